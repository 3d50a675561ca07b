"""GPU parity at BASELINE's full sizes (the largest config-1 shapes, M = 32768).

The oracle cannot compute a whole 32768 x 19456 x 2560 product in seconds, so these tests use
properties that hold at any size, plus full rows sampled from the product:
  * the exact int32 row and column checksums of the product: sum_n C[m, n] = A[m] . colsum(B)
    and sum_m C[m, n] = B[n] . colsum(A), evaluated in float64, which is exact for integers
    below 2^53;
  * full rows picked at random, bit-exact against the oracle;
  * quantiser invariants on every row: the scale is max|x| / 127 in IEEE fp32, |q| <= 127, and
    the absmax element of each row quantises to +-127.
"""
import numpy as np
import pytest
import torch

from conftest import ORACLE as O

pytestmark = pytest.mark.gpu

M_FULL = 32768


@pytest.fixture(scope='module')
def K():
    import mica_b200.int8_kernels as K
    ok, why = K.available('cuda')
    assert ok, why
    K.preload('cuda')
    return K


def _rows(seed, n=48):
    g = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, M_FULL - 1], g.integers(0, M_FULL, n)]))


def _to_f32(t):
    return O.bf16_bits_to_f32(t.cpu().view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize('tile', [0, 128256, 256256])
def test_gemm_full_size_int32_checksums_and_rows(K, tile):
    """gate_up shape at M = 32768. Operands in [-31, 31] keep every |acc| <= 2560 * 31^2 below
    2^24, so the fp32 output with unit scales is the exact int32 accumulator."""
    n, k = 19456, 2560
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(4242 + tile)
    a = torch.randint(-31, 32, (M_FULL, k), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-31, 32, (n, k), generator=g, device=dev, dtype=torch.int8)
    y = torch.ops.mica.w8a8_gemm(a, torch.ones(M_FULL, device=dev), b, torch.ones(n, device=dev), None, 2, tile)
    torch.cuda.synchronize()
    row_sum = y.double().sum(dim=1)
    col_sum = y.double().sum(dim=0)
    assert torch.equal(row_sum, a.double() @ b.double().sum(dim=0))
    assert torch.equal(col_sum, b.double() @ a.double().sum(dim=0))
    rows = _rows(tile)
    acc = O.int_gemm_exact(a[rows].cpu().numpy(), b.cpu().numpy())
    assert np.array_equal(y[rows].cpu().numpy().astype(np.int64), acc.astype(np.int64))


@pytest.mark.parametrize('n,k', [(19456, 2560), (2560, 9728)])
def test_gemm_full_size_bf16_rows_bit_exact(K, n, k):
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(n + k)
    a = torch.randint(-127, 128, (M_FULL, k), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
    sa = torch.rand(M_FULL, generator=g, device=dev) * 0.05 + 1e-3
    sb = torch.rand(n, generator=g, device=dev) * 9e-3 + 1e-3
    y = K.mm_i8(a, sa, b, sb, None, torch.bfloat16)
    assert y is not None
    rows = _rows(n)
    ref = O.dequant_out(O.int_gemm_exact(a[rows].cpu().numpy(), b.cpu().numpy()), sa[rows].cpu().numpy(),
                        sb.cpu().numpy(), None, out='bf16')
    assert np.array_equal(_to_f32(y[rows]), ref)
    assert torch.isfinite(y.float()).all()


def _check_codes(x, q, s, mode, rows):
    """Invariants on every row, then sampled rows bit-exact against the oracle."""
    amax = x.float().abs().amax(dim=1)
    # tensor / tensor: torch divides by a Python scalar on CUDA as a multiply by its reciprocal
    assert torch.equal(s, torch.clamp(amax, min=1e-8) / torch.full_like(amax, 127.0))
    qa = q.abs().amax(dim=1)
    assert int(qa.max()) <= 127
    assert bool((qa[amax >= 1e-8] == 127).all())
    qo, so = O.quant_act(x[rows].float().cpu().numpy(), None, mode)
    assert np.array_equal(s[rows].cpu().numpy(), so)
    assert np.array_equal(q[rows].cpu().numpy(), qo)


@pytest.mark.parametrize('mode', ['half_away', 'half_even'])
def test_act_quant_full_size(K, mode):
    """down_proj input at 32k tokens: 32768 x 9728, row magnitudes over 8 decades, outlier channels."""
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(9728)
    x = torch.randn(M_FULL, 9728, generator=g, device=dev)
    x *= torch.pow(10.0, torch.rand(M_FULL, 1, generator=g, device=dev) * 8 - 4)
    x[:, torch.randperm(9728, generator=g, device=dev)[:8]] *= 50
    x = x.to(torch.bfloat16)
    K.ROUND['mode'] = mode
    try:
        q, s = K.act_quant(x)
    finally:
        K.ROUND['mode'] = 'half_away'
    _check_codes(x, q, s, mode, _rows(7))


def test_gemm_swiglu_quant_full_size(K):
    """gate_up + SwiGLU + requant at M = 32768, I = 9728: sampled rows of h against the oracle
    chain, and the fused requantisation checked on every row against the kernel's own h."""
    m, i, k = M_FULL, 9728, 2560
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(31)
    qx = torch.randint(-127, 128, (m, k), generator=g, device=dev, dtype=torch.int8)
    sx = torch.rand(m, generator=g, device=dev) * 0.02 + 1e-3
    wg = torch.randint(-127, 128, (i, k), generator=g, device=dev, dtype=torch.int8)
    wu = torch.randint(-127, 128, (i, k), generator=g, device=dev, dtype=torch.int8)
    sg = torch.rand(i, generator=g, device=dev) * 9e-3 + 1e-3
    su = torch.rand(i, generator=g, device=dev) * 9e-3 + 1e-3
    wg_n, wu_n, sg_n, su_n = (t.cpu().numpy() for t in (wg, wu, sg, su))
    qw = torch.from_numpy(O.interleave_gate_up(wg_n, wu_n)).contiguous().to(dev)
    sw = torch.from_numpy(O.interleave_gate_up(sg_n, su_n)).contiguous().to(dev)
    h, q, s = K.mm_i8_swiglu_quant(qx, sx, qw, sw)
    rows = _rows(3, n=24)
    h_ref, _, _ = O.gate_up_swiglu_quant(qx[rows].cpu().numpy(), sx[rows].cpu().numpy(), wg_n, sg_n, wu_n, su_n)
    hk = _to_f32(h[rows])
    assert np.allclose(hk, h_ref, rtol=1e-2, atol=1e-2 * np.abs(h_ref).max())
    assert (hk != h_ref).mean() < 0.01
    _check_codes(h, q, s, 'half_away', rows)
