"""The C ABI: libmica_w8a8.so loads and exports exactly what include/mica_w8a8.h declares (no
compute without a GPU), and the ctypes binding covers every declaration."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'mica_w8a8.h'


def declared():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(mica_[a-z0-9_]+)\s*\(', text)))


@pytest.fixture(scope='module')
def lib_path():
    from mica_b200 import build
    return build.build()


def test_header_declares_the_entry_points():
    names = declared()
    for n in ('mica_act_quant', 'mica_w8a8_gemm', 'mica_rmsnorm_quant', 'mica_w8a8_gemm_swiglu_quant',
              'mica_option_logits', 'mica_query', 'mica_preload'):
        assert n in names


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(['nm', '-D', '--defined-only', str(lib_path)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r'\bT (mica_[a-z0-9_]+)', out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
    lib = ctypes.CDLL(str(lib_path))
    for n in declared():
        assert getattr(lib, n) is not None


def test_ctypes_binding_covers_the_header(lib_path):
    from mica_b200 import _native as N
    assert sorted(N.SIGNATURES) == declared()
    lib = N.lib()
    assert lib.mica_swiglu_workspace_bytes(4096) == 4096 * 4 + 16
    assert lib.mica_swiglu_workspace_bytes(3) == 16 + 16


def test_entry_points_reject_bad_arguments_without_touching_a_gpu(lib_path):
    """Argument checks run before any CUDA call, so they work on a CPU-only host."""
    from mica_b200 import _native as N
    lib = N.lib()
    assert lib.mica_act_quant(None, 0, 64, None, None, 64, None, 4, 64, 0, None) == 1          # ERR_ARG
    assert lib.mica_act_quant(16, 0, 64, None, 16, 64, 16, 4, 12, 0, None) == 2                # K % 8
    assert lib.mica_act_quant(17, 0, 64, None, 16, 64, 16, 4, 64, 0, None) == 3                # misaligned
    assert lib.mica_w8a8_gemm(16, 24, 16, 24, 16, 16, None, 16, 0, 8, 4, 8, 24, None) == 2     # K % 16
    assert lib.mica_w8a8_gemm(16, 32, 16, 32, 16, 16, None, 16, 0, 4, 4, 4, 32, None) == 3     # ldc*2 % 16
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 0, 96, 0, 0, None) == 1  # block_n
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 192, 0, 0, 0, None) == 1  # block_m
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 256, 64, 0, 0, None) == 1
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 128, 64, 0, 9, None) == 1  # splits
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 256, 256, 0, 2, None) == 1
    # 128 x 320 tiles: single CTAs only, no K split
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 256, 320, 0, 0, None) == 1
    assert lib.mica_w8a8_gemm_cfg(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 128, 320, 0, 2, None) == 1
    # stream-K: not on CTA pairs, not with a capped grid, splits below -1 rejected; workspace alignment
    sk = N.SPLIT_STREAM_K
    assert lib.mica_w8a8_gemm_ex(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 256, 256, 0, sk, None, 0, None) == 1
    assert lib.mica_w8a8_gemm_ex(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 128, 256, 4, sk, None, 0, None) == 1
    assert lib.mica_w8a8_gemm_ex(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 128, 256, 0, -2, None, 0, None) == 1
    assert lib.mica_w8a8_gemm_ex(16, 32, 16, 32, 16, 16, None, 16, 0, 8, 4, 8, 32, 128, 256, 0, sk, 24, 4096,
                                 None) == 3
    assert lib.mica_w8a8_gemm_workspace_bytes(512, 9728, 2560, 0, 0, 0, 0) == 0      # no device here
    assert lib.mica_w8a8_gemm_swiglu_quant(16, 32, 16, 32, 16, 16, None, None, 16, 32, 16, 32, 16, 4, 32, 32, 0,
                                           16, 8, None) == 7                                   # workspace
    # the allocation-free SwiGLU entry point checks its arguments like the workspace one, then its
    # row limit, all before any CUDA call
    na = lib.mica_w8a8_gemm_swiglu_quant_noalloc
    assert na(None, 32, 16, 32, 16, 16, None, None, 16, 32, 16, 32, 16, 4, 32, 32, 0, None) == 1   # ERR_ARG
    assert na(16, 32, 16, 32, 16, 16, None, None, 16, 32, 16, 32, 16, 4, 32, 32, 3, None) == 1     # round mode
    assert na(16, 32, 16, 32, 16, 16, None, None, 16, 32, 16, 32, 16, 4, 24, 32, 0, None) == 2     # I % 16
    assert na(17, 32, 16, 32, 16, 16, None, None, 16, 32, 16, 32, 16, 4, 32, 32, 0, None) == 3     # misaligned
    assert na(16, 32, 16, 32, 16, 16, None, None, 16, 32, 16, 32, 16, 65537, 32, 32, 0, None) == 7  # rows > limit
    assert lib.mica_option_logits(16, 0, 64, None, 0, 1e-6, 16, 0, 64, None, None, 16, 16, 1, None) == 2
    assert lib.mica_selftest_wait_timeout(None, 10, None) == 1
