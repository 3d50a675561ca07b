"""ctypes binding of libmica_w8a8.so (declarations in include/mica_w8a8.h).

The reference binds its kernels the same way -- ctypes into the CUDA driver, launching
AOT cubins (v0.5/serving/lib/int8_kernels.py:27-64) -- but keeps the launch logic in
Python. Here Python only passes pointers, strides and the current stream; argument
checking, TMA descriptor encoding and tile choice live in the C++ side.

There is no fallback: if the library is missing or fails to load, `lib()` raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_NAME = 'libmica_w8a8.so'
ENV_LIB = 'MICA_B200_LIB'

OK = 0
ERRORS = {
    1: 'ERR_ARG',
    2: 'ERR_SHAPE',
    3: 'ERR_ALIGN',
    4: 'ERR_ARCH',
    5: 'ERR_CUDA',
    6: 'ERR_RANGE',
    7: 'ERR_WORKSPACE',
    8: 'ERR_UNSUPPORTED',
}
DT_BF16, DT_FP16, DT_FP32 = 0, 1, 2
ROUND_HALF_AWAY, ROUND_HALF_EVEN = 0, 1
NORM_OFFSET, NORM_WEIGHT = 0, 1
DEV_ERRORS = {
    0: 'ok',
    1: 'timeout_producer',
    2: 'timeout_mma',
    3: 'timeout_epilogue',
    4: 'timeout_grid',
    5: 'timeout_drain',
    6: 'timeout_selftest',
    7: 'timeout_streamk',
    8: 'bad_launch',
}
SPLIT_STREAM_K = -1

# name -> (restype, argtypes); mirrors include/mica_w8a8.h
_P, _I, _L, _F, _Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_float, ctypes.c_size_t


class Caps(ctypes.Structure):
    _fields_ = [
        ('device', _I),
        ('cc_major', _I),
        ('cc_minor', _I),
        ('sm_count', _I),
        ('supported', _I),
        ('max_smem_optin', _I),
        ('abi_version', _I),
        ('pair_clusters', _I),
    ]


SIGNATURES = {
    'mica_query': (_I, [_I, ctypes.POINTER(Caps)]),
    'mica_preload': (_I, [ctypes.POINTER(_I)]),
    'mica_last_cuda_error': (ctypes.c_char_p, []),
    'mica_device_error': (_I, [ctypes.POINTER(_I), _P]),
    'mica_act_quant': (_I, [_P, _I, _L, _P, _P, _L, _P, _I, _I, _I, _P]),
    'mica_rmsnorm_quant': (
        _I,
        [_P, _I, _L, _P, _L, _P, _I, _F, _P, _P, _L, _P, _L, _P, _L, _P, _I, _I, _I, _P],
    ),
    'mica_w8a8_gemm': (_I, [_P, _L, _P, _L, _P, _P, _P, _P, _I, _L, _I, _I, _I, _P]),
    'mica_w8a8_gemm_cfg': (_I, [_P, _L, _P, _L, _P, _P, _P, _P, _I, _L, _I, _I, _I, _I, _I, _I, _I, _P]),
    'mica_w8a8_gemm_ex': (_I, [_P, _L, _P, _L, _P, _P, _P, _P, _I, _L, _I, _I, _I, _I, _I, _I, _I, _P, _Z, _P]),
    'mica_w8a8_gemm_workspace_bytes': (_Z, [_I, _I, _I, _I, _I, _I, _I]),
    'mica_swiglu_workspace_bytes': (_Z, [_I]),
    'mica_w8a8_gemm_swiglu_quant': (
        _I,
        [_P, _L, _P, _L, _P, _P, _P, _P, _P, _L, _P, _L, _P, _I, _I, _I, _I, _P, _Z, _P],
    ),
    'mica_w8a8_gemm_swiglu_quant_noalloc': (
        _I,
        [_P, _L, _P, _L, _P, _P, _P, _P, _P, _L, _P, _L, _P, _I, _I, _I, _I, _P],
    ),
    'mica_swiglu_quant': (_I, [_P, _L, _P, _L, _I, _P, _P, _L, _P, _L, _P, _I, _I, _I, _P]),
    'mica_option_logits': (_I, [_P, _I, _L, _P, _I, _F, _P, _I, _I, _P, _P, _P, _P, _I, _P]),
    'mica_qk_norm_rope': (_I, [_P, _L, _P, _P, _P, _P, _P, _L, _I, _I, _I, _I, _F, _P]),
    'mica_attention_prefill': (_I, [_P, _L, _P, _L, _I, _I, _I, _I, _I, _F, _P]),
    'mica_selftest_wait_timeout': (_I, [_P, _I, _P]),
}

_LIB = None
_LOCK = threading.Lock()


def lib_path() -> Path:
    env = os.environ.get(ENV_LIB)
    return Path(env) if env else Path(__file__).resolve().parent / LIB_NAME


class NativeError(RuntimeError):
    """A libmica_w8a8 entry point returned a non-zero status."""

    def __init__(self, name, rc, detail=''):
        self.name, self.rc = name, rc
        super().__init__(f'{name} failed: {ERRORS.get(rc, rc)}' + (f' ({detail})' if detail else ''))


def lib():
    """The loaded library; raises OSError when it is missing (run mica_b200.build.build())."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            p = lib_path()
            if not p.is_file():
                raise OSError(f'{p} not found: build it with `python -c "import mica_b200.build as b; b.build()"`')
            handle = ctypes.CDLL(str(p))
            for name, (res, args) in SIGNATURES.items():
                f = getattr(handle, name)
                f.restype, f.argtypes = res, args
            _LIB = handle
    return _LIB


def exported_symbols():
    return sorted(SIGNATURES)


def check(name, rc):
    if rc != OK:
        detail = ''
        if rc == 5:
            detail = lib().mica_last_cuda_error().decode(errors='replace')
        raise NativeError(name, rc, detail)
    return rc


def call(name, *args):
    """Call entry point `name` and raise NativeError on a non-zero status."""
    return check(name, getattr(lib(), name)(*args))
