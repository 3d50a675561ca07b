"""GPU parity on the W8A8 shapes of the shipped Qwen3.5-4B hybrid model (24 Gated-DeltaNet +
8 full-attention layers, hidden 2560, FFN 9216): the (N, K) pairs and quantiser widths of the
reference's sm100 specialisations (v0.5/serving/kernel_src/specs/sm100.json), the GDN q/k/v
projection split by QLinear.rows_forward (v0.5/serving/lib/fork.py:46-68,
lib/int8_runtime.py:153-170), with and without smoothing. Bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from conftest import ORACLE as O

pytestmark = pytest.mark.gpu

# GDN in_proj_a/b (32), attention k/v (1024), out/o proj (2560 <- 4096), down (2560 <- 9216),
# in_proj_z / q (4096), in_proj_qkv (8192 = 2 x 2048 keys + 4096 values), gate / up (9216)
HYBRID_NK = ((32, 2560), (1024, 2560), (2560, 4096), (2560, 9216), (4096, 2560), (8192, 2560), (9216, 2560))


@pytest.fixture(scope='module')
def K():
    import mica_b200.int8_kernels as K
    ok, why = K.available('cuda')
    assert ok, why
    K.preload('cuda')
    return K


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize('m', [1, 17, 200, 1500])
@pytest.mark.parametrize('n,k', HYBRID_NK)
def test_hybrid_linear_bit_exact(K, n, k, m):
    from mica_b200.int8_runtime import QLinear
    g = torch.Generator().manual_seed(n + k + m)
    lin = torch.nn.Linear(k, n, bias=False)
    lin.weight.data = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    q = QLinear(lin).cuda()
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    y = q(x.cuda())
    ref = O.w8a8_linear(x.float().numpy(), q.qweight.cpu().numpy(), q.wscale.cpu().numpy())[0]
    assert np.array_equal(_bits(y), O.f32_to_bf16_bits(ref))


@pytest.mark.parametrize('smooth', [False, True])
@pytest.mark.parametrize('m', [3, 640])
def test_gdn_qkv_rows_forward_split(K, m, smooth):
    """One quantisation of x, three GEMMs over the key / key / value row ranges of in_proj_qkv."""
    from mica_b200.int8_runtime import QLinear
    n, k, kd = 8192, 2560, 2048
    g = torch.Generator().manual_seed(m + smooth)
    lin = torch.nn.Linear(k, n, bias=False)
    lin.weight.data = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    sm = torch.exp(torch.randn(k, generator=g) * 0.5) if smooth else None
    q = QLinear(lin, sm).cuda()
    x = torch.randn(2, m, k, generator=g).to(torch.bfloat16).cuda()
    ranges = ((0, kd), (kd, 2 * kd), (2 * kd, n))
    parts = q.rows_forward(x, ranges)
    full = q(x)
    for (lo, hi), part in zip(ranges, parts):
        assert part.shape == (2, m, hi - lo)
        assert torch.equal(part, full[..., lo:hi])
    inv = None if q.inv_smooth is None else q.inv_smooth.cpu().numpy()
    ref = O.w8a8_linear(x.reshape(-1, k).float().cpu().numpy(), q.qweight.cpu().numpy(), q.wscale.cpu().numpy(),
                        inv_smooth=inv)[0]
    assert np.array_equal(_bits(full.reshape(-1, n)), O.f32_to_bf16_bits(ref))


@pytest.mark.parametrize('mode', ['half_away', 'half_even'])
@pytest.mark.parametrize('k', [2560, 4096, 9216])
def test_hybrid_act_quant_widths(K, k, mode):
    g = torch.Generator().manual_seed(k)
    x = (torch.randn(300, k, generator=g) * torch.pow(10.0, torch.rand(300, 1, generator=g) * 4 - 2)).to(torch.bfloat16)
    inv = torch.exp(torch.randn(k, generator=g) * 0.5)
    K.ROUND['mode'] = mode
    try:
        q, s = K.act_quant(x.cuda(), inv.cuda())
    finally:
        K.ROUND['mode'] = 'half_away'
    qo, so = O.quant_act(x.float().numpy(), inv.numpy(), mode)
    assert np.array_equal(s.cpu().numpy(), so)
    assert np.array_equal(q.cpu().numpy(), qo)


def test_hybrid_fused_mlp_ffn9216(K):
    """gate_up (2 x 9216 <- 2560) + SwiGLU + requant in one launch, at the hybrid FFN width."""
    m, i, k = 513, 9216, 2560
    g = torch.Generator().manual_seed(9216)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    sx = torch.rand(m, generator=g) * 0.02 + 1e-3
    wg = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    wu = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    sg = torch.rand(i, generator=g) * 9e-3 + 1e-3
    su = torch.rand(i, generator=g) * 9e-3 + 1e-3
    qw = torch.from_numpy(O.interleave_gate_up(wg.numpy(), wu.numpy())).contiguous()
    sw = torch.from_numpy(O.interleave_gate_up(sg.numpy(), su.numpy())).contiguous()
    h, q, s = K.mm_i8_swiglu_quant(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda())
    h_ref, _, _ = O.gate_up_swiglu_quant(qx.numpy(), sx.numpy(), wg.numpy(), sg.numpy(), wu.numpy(), su.numpy())
    hk = O.bf16_bits_to_f32(_bits(h))
    assert np.allclose(hk, h_ref, rtol=1e-2, atol=1e-2 * np.abs(h_ref).max())
    assert (hk != h_ref).mean() < 0.01
    q2, s2 = O.quant_act_half_away(hk)
    assert np.array_equal(s.cpu().numpy(), s2)
    assert np.array_equal(q.cpu().numpy(), q2)
