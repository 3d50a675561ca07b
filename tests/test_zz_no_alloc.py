"""The allocation-free SwiGLU entry point (mica_w8a8_gemm_swiglu_quant_noalloc).

It exists for callers that cannot call cudaMalloc: a host whose memory planner already owns
all of device memory, or a plugin host that forbids allocation on its serving path. It
takes its scratch from a fixed array inside the library instead of a caller-supplied
workspace. This test calls it through the C ABI and compares it with the workspace entry
point on the same inputs, twice in a row. The second call has smaller activations, so a
stale row maximum left by the first call would change the scales and codes.

Collected last on purpose (file name), so a failure here comes after every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import ORACLE as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def lib():
    from mica_b200 import _native as N
    import mica_b200.int8_kernels as K
    ok, why = K.available('cuda')
    assert ok, why
    return N


def _inputs(m, i, k, seed, x_scale):
    g = torch.Generator().manual_seed(seed)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    sx = (torch.rand(m, generator=g) * 0.02 + 1e-3) * x_scale
    wg = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    wu = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    sg = torch.rand(i, generator=g) * 9e-3 + 1e-3
    su = torch.rand(i, generator=g) * 9e-3 + 1e-3
    qw = torch.from_numpy(O.interleave_gate_up(wg.numpy(), wu.numpy())).contiguous()
    sw = torch.from_numpy(O.interleave_gate_up(sg.numpy(), su.numpy())).contiguous()
    return [t.cuda() for t in (qx, sx, qw, sw)]


def _outputs(m, i):
    return (torch.empty(m, i, dtype=torch.bfloat16, device='cuda'), torch.empty(m, i, dtype=torch.int8, device='cuda'),
            torch.empty(m, dtype=torch.float32, device='cuda'))


def _call_workspace(N, qx, sx, qw, sw, m, i, k):
    h, q, s = _outputs(m, i)
    ws = torch.empty(N.lib().mica_swiglu_workspace_bytes(m), dtype=torch.uint8, device='cuda')
    N.call('mica_w8a8_gemm_swiglu_quant', qx.data_ptr(), k, qw.data_ptr(), k, sx.data_ptr(), sw.data_ptr(), None,
           None, h.data_ptr(), i, q.data_ptr(), i, s.data_ptr(), m, i, k, 0, ws.data_ptr(), ws.numel(),
           torch.cuda.current_stream().cuda_stream)
    return h, q, s


def _call_noalloc(N, qx, sx, qw, sw, m, i, k):
    h, q, s = _outputs(m, i)
    N.call('mica_w8a8_gemm_swiglu_quant_noalloc', qx.data_ptr(), k, qw.data_ptr(), k, sx.data_ptr(), sw.data_ptr(),
           None, None, h.data_ptr(), i, q.data_ptr(), i, s.data_ptr(), m, i, k, 0, torch.cuda.current_stream().cuda_stream)
    return h, q, s


def _close(a, b):
    hf_a, hf_b = a[0].float(), b[0].float()
    # the tolerance the other SwiGLU tests use for h (1e-2 relative); codes and scales exact
    assert torch.allclose(hf_a, hf_b, rtol=1e-2, atol=1e-2 * float(hf_b.abs().max()))
    assert torch.equal(a[1], b[1])
    assert torch.equal(a[2], b[2])


def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row(lib):
    m, i, k = 300, 512, 1024
    first = _inputs(m, i, k, seed=1, x_scale=8.0)
    second = _inputs(m, i, k, seed=2, x_scale=0.25)
    a1 = _call_noalloc(lib, *first, m, i, k)
    a2 = _call_noalloc(lib, *second, m, i, k)
    b1 = _call_workspace(lib, *first, m, i, k)
    b2 = _call_workspace(lib, *second, m, i, k)
    torch.cuda.synchronize()
    _close(a1, b1)
    _close(a2, b2)
    assert not torch.equal(a1[2], a2[2])
    code = ctypes.c_int(-1)
    lib.call('mica_device_error', ctypes.byref(code), torch.cuda.current_stream().cuda_stream)
    assert code.value == 0


def test_noalloc_rejects_rows_beyond_its_fixed_scratch(lib):
    m, i, k = 65537, 128, 64     # one row over MICA_NOALLOC_MAX_ROWS; refused before any launch
    dummy = torch.empty(16, dtype=torch.int8, device='cuda')
    rc = lib.lib().mica_w8a8_gemm_swiglu_quant_noalloc(dummy.data_ptr(), k, dummy.data_ptr(), k, dummy.data_ptr(),
                                                        dummy.data_ptr(), None, None, dummy.data_ptr(), i,
                                                        dummy.data_ptr(),
                                                        i, dummy.data_ptr(), m, i, k, 0,
                                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 7   # MICA_ERR_WORKSPACE


@pytest.mark.parametrize('m,i,k', [(2048, 9728, 2560), (65536, 64, 64)])
def test_noalloc_matches_workspace_entry_point_at_its_limits(lib, m, i, k):
    """A grid large enough for the 256-wide tiles, and the maximum row count, where the grid
    barrier's counter sits in the last bytes of the fixed scratch; codes and scales exact."""
    x = _inputs(m, i, k, seed=3 + m, x_scale=1.0)
    a = _call_noalloc(lib, *x, m, i, k)
    b = _call_workspace(lib, *x, m, i, k)
    torch.cuda.synchronize()
    _close(a, b)
    code = ctypes.c_int(-1)
    lib.call('mica_device_error', ctypes.byref(code), torch.cuda.current_stream().cuda_stream)
    assert code.value == 0
