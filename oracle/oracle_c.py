"""numpy-facing wrapper of oracle_cpu.c (the plain-C oracle) -- TEST INFRASTRUCTURE ONLY.

Built by `make -C oracle` (called from __graft_entry__.build()) into oracle/_build/. Used by
tests/ to cross-check the numpy oracle and by bench.py's CPU-baseline / reference legs.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / '_build' / 'liboracle_cpu.so'
_P, _L = ctypes.c_void_p, ctypes.c_long
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.is_file():
            raise OSError(f'{LIB} missing: run `make -C {HERE}`')
        h = ctypes.CDLL(str(LIB))
        h.oracle_threads.restype = ctypes.c_int
        h.oracle_set_threads.argtypes = [ctypes.c_int]
        h.oracle_quant_act.argtypes = [_P, _P, _L, _L, ctypes.c_int, _P, _P]
        h.oracle_int_gemm.argtypes = [_P, _P, _L, _L, _L, _P]
        h.oracle_dequant.argtypes = [_P, _P, _P, _P, _L, _L, _P]
        _lib = h
    return _lib


def available() -> bool:
    try:
        lib()
        return True
    except OSError:
        return False


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def quant_act(x, inv=None, mode='half_away'):
    x = _c(x, np.float32)
    m, k = x.shape
    inv_a = None if inv is None else _c(inv, np.float32)
    q = np.empty((m, k), np.int8)
    s = np.empty((m,), np.float32)
    lib().oracle_quant_act(x.ctypes.data, None if inv_a is None else inv_a.ctypes.data, m, k,
                           1 if mode == 'half_even' else 0, q.ctypes.data, s.ctypes.data)
    return q, s


def int_gemm(qx, qw):
    a, b = _c(qx, np.int8), _c(qw, np.int8)
    m, k = a.shape
    n = b.shape[0]
    out = np.empty((m, n), np.int32)
    lib().oracle_int_gemm(a.ctypes.data, b.ctypes.data, m, n, k, out.ctypes.data)
    return out


def dequant_bf16_bits(acc, sa, sb, bias=None):
    acc = _c(acc, np.int32)
    m, n = acc.shape
    sa, sb = _c(sa, np.float32), _c(sb, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    out = np.empty((m, n), np.uint16)
    lib().oracle_dequant(acc.ctypes.data, sa.ctypes.data, sb.ctypes.data, None if b is None else b.ctypes.data, m, n,
                         out.ctypes.data)
    return out


def threads() -> int:
    return int(lib().oracle_threads())


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))
