"""GPU parity: libmica_w8a8 kernels (through the reference-facing surface and the C ABI)
against the CPU oracle on the same seeded inputs.

Bars: int8 codes, token scales and int32 accumulators bit-exact; bf16 GEMM outputs
bit-exact against the oracle's fp32 epilogue (so within 1e-2 relative of the reference);
norm outputs within 1 bf16 ulp; option probabilities within 1e-3 absolute.
"""
import numpy as np
import pytest
import torch

from conftest import golden, ORACLE as O

pytestmark = pytest.mark.gpu

ROWS = (1, 3, 17, 48, 200, 608, 1500)   # the reference self-test rows (int8_runtime.py:288)


@pytest.fixture(scope='module')
def K():
    import mica_b200.int8_kernels as K
    ok, why = K.available('cuda')
    assert ok, why
    assert K.preload('cuda') > 0
    return K


def bf16(a):
    return torch.from_numpy(O.f32_to_bf16_bits(a).view(np.int16)).view(torch.bfloat16)


def to_np(t):
    if t.dtype == torch.bfloat16:
        return O.bf16_bits_to_f32(t.cpu().view(torch.int16).numpy().view(np.uint16))
    return t.cpu().numpy()


def dev_error():
    from mica_b200 import _native as N
    code = N.ctypes.c_int(-1)
    N.call('mica_device_error', N.ctypes.byref(code), torch.cuda.current_stream().cuda_stream)
    return code.value


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize('mode', ['half_away', 'half_even'])
@pytest.mark.parametrize('case', ['a', 'b', 'c', 'd', 'e', 'f'])
def test_act_quant_golden(K, case, mode):
    g = golden('act_quant')
    x = torch.from_numpy(g[f'{case}/x'].view(np.int16)).view(torch.bfloat16).cuda()
    inv = g[f'{case}/inv']
    inv_t = torch.from_numpy(inv).cuda() if inv.size else None
    K.ROUND['mode'] = mode
    try:
        q, s = K.act_quant(x, inv_t)
    finally:
        K.ROUND['mode'] = 'half_away'
    suffix = 'away' if mode == 'half_away' else 'even'
    assert np.array_equal(s.cpu().numpy(), g[f'{case}/s_{suffix}'])
    assert np.array_equal(q.cpu().numpy(), g[f'{case}/q_{suffix}'])


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize('m', ROWS)
@pytest.mark.parametrize('k', [64, 2560, 9728])
def test_act_quant_random(K, m, k, dtype):
    g = torch.Generator().manual_seed(m * 31 + k)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[:8]] *= 50
    x = x.to(dtype)
    inv = torch.rand(k, generator=g) + 0.5 if m % 2 else None
    q, s = K.act_quant(x.cuda(), inv.cuda() if inv is not None else None)
    qo, so = O.quant_act_half_away(x.float().numpy(), None if inv is None else inv.numpy())
    assert np.array_equal(s.cpu().numpy(), so)
    assert np.array_equal(q.cpu().numpy(), qo)


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize('case', ['a', 'b', 'c', 'd'])
def test_gemm_golden(K, case):
    g = golden('gemm')
    qx = torch.from_numpy(g[f'{case}/qx']).cuda()
    sx = torch.from_numpy(g[f'{case}/sx']).cuda()
    qw = torch.from_numpy(g[f'{case}/qw']).cuda()
    sw = torch.from_numpy(g[f'{case}/sw']).cuda()
    b = g[f'{case}/bias']
    bias = torch.from_numpy(b).cuda() if b.size else None
    y32 = K.mm_i8(qx, sx, qw, sw, bias, torch.float32)
    assert np.array_equal(y32.cpu().numpy(), g[f'{case}/y_triton_f32'])   # reference Triton kernel, bit-exact
    y = K.mm_i8(qx, sx, qw, sw, bias, torch.bfloat16)
    assert np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), g[f'{case}/y_qlinear'])


TILES = [128064, 128128, 128256, 256128, 256256]   # block_m * 1000 + block_n


@pytest.mark.parametrize('tile', TILES)
@pytest.mark.parametrize('m,n', [(1, 64), (3, 256), (130, 192), (200, 512), (1500, 320), (513, 1024)])
def test_gemm_int32_accumulators_exact(K, m, n, tile):
    """K=1024 keeps |acc| < 2^24, so float(acc) in the fp32 output is the exact int32."""
    k = 1024
    g = torch.Generator().manual_seed(m + n + tile)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    one_m, one_n = torch.ones(m), torch.ones(n)
    y = torch.ops.mica.w8a8_gemm(qx.cuda(), one_m.cuda(), qw.cuda(), one_n.cuda(), None, 2, tile)
    acc = O.int_gemm_exact(qx.numpy(), qw.numpy())
    assert np.array_equal(y.cpu().numpy().astype(np.int64), acc.astype(np.int64))


@pytest.mark.parametrize('out', ['bf16', 'fp16'])
@pytest.mark.parametrize('m,n,k', [(17, 96, 2560), (256, 6144, 2560), (130, 2560, 4096), (48, 2560, 9728),
                                   (512, 9728, 2560), (5, 40, 48), (300, 104, 16)])
def test_gemm_random_vs_oracle(K, m, n, k, out):
    g = torch.Generator().manual_seed(m * 7 + n + k)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sx = torch.rand(m, generator=g) * 0.05 + 1e-3
    sw = torch.rand(n, generator=g) * 9e-3 + 1e-3
    bias = torch.randn(n, generator=g) * 0.1 if n % 3 == 0 else None
    dt = torch.bfloat16 if out == 'bf16' else torch.float16
    y = K.mm_i8(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda(), None if bias is None else bias.cuda(), dt)
    assert y is not None
    ref = O.dequant_out(O.int_gemm_exact(qx.numpy(), qw.numpy()), sx.numpy(), sw.numpy(),
                        None if bias is None else bias.numpy(), out=out)
    assert np.array_equal(to_np(y.float()), ref)


@pytest.mark.parametrize('tile', TILES)
@pytest.mark.parametrize('out', [0, 1, 2])
@pytest.mark.parametrize('m,n,k', [(4096, 6144, 2560), (777, 2560, 9728), (256, 19456, 2560)])
def test_gemm_tiles_bit_exact_vs_oracle(K, m, n, k, tile, out):
    g = torch.Generator().manual_seed(m + n + k + tile + out)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sx = torch.rand(m, generator=g) * 0.05 + 1e-3
    sw = torch.rand(n, generator=g) * 9e-3 + 1e-3
    bias = torch.randn(n, generator=g) * 0.1
    y = torch.ops.mica.w8a8_gemm(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda(), bias.cuda(), out, tile)
    ref = O.dequant_out(O.int_gemm_exact(qx.numpy(), qw.numpy()), sx.numpy(), sw.numpy(), bias.numpy(),
                        out=('bf16', 'fp16', 'fp32')[out])
    assert np.array_equal(to_np(y.float()), ref)
    assert dev_error() == 0


def test_gemm_misses_match_reference_contract(K):
    qx = torch.zeros(4, 24, dtype=torch.int8, device='cuda')          # K % 16 != 0
    qw = torch.zeros(8, 24, dtype=torch.int8, device='cuda')
    s4, s8 = torch.ones(4, device='cuda'), torch.ones(8, device='cuda')
    before = dict(K.STATS['fallback'])
    assert K.mm_i8(qx, s4, qw, s8) is None
    assert K.STATS['fallback'].get('align', 0) == before.get('align', 0) + 1
    assert K.mm_i8(qx.float(), s4, qw, s8) is None                    # dtype miss


# ---------------------------------------------------------------------------------------
# (1, 9728, 2560): the last layer's single scored row, 128-wide tiles, 152 tiles on 148 SMs (two on some CTAs)
@pytest.mark.parametrize('m,i,k', [(1, 128, 256), (37, 256, 2560), (300, 512, 1024), (1, 9728, 2560),
                                   (1024, 9728, 2560)])
def test_gemm_swiglu_quant(K, m, i, k):
    g = torch.Generator().manual_seed(m + i + k)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    sx = torch.rand(m, generator=g) * 0.02 + 1e-3
    wg = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    wu = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    sg = torch.rand(i, generator=g) * 9e-3 + 1e-3
    su = torch.rand(i, generator=g) * 9e-3 + 1e-3
    qw = torch.from_numpy(O.interleave_gate_up(wg.numpy(), wu.numpy())).contiguous()
    sw = torch.from_numpy(O.interleave_gate_up(sg.numpy(), su.numpy())).contiguous()
    h, q, s = K.mm_i8_swiglu_quant(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda())
    h_ref, q_ref, s_ref = O.gate_up_swiglu_quant(qx.numpy(), sx.numpy(), wg.numpy(), sg.numpy(), wu.numpy(),
                                                 su.numpy())
    hk = to_np(h)
    # SwiGLU: within 1e-2 relative (exp rounding may move the bf16 silu by one ulp)
    assert np.allclose(hk, h_ref, rtol=1e-2, atol=1e-2 * np.abs(h_ref).max())
    assert (hk != h_ref).mean() < 0.01
    # the fused requantisation is bit-exact given the kernel's own h
    q2, s2 = O.quant_act_half_away(hk)
    assert np.array_equal(s.cpu().numpy(), s2)
    assert np.array_equal(q.cpu().numpy(), q2)
    assert dev_error() == 0


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize('case', ['a', 'b', 'c'])
def test_rmsnorm_quant_golden(K, case):
    g = golden('norm')
    x = torch.from_numpy(g[f'{case}/x'].view(np.int16)).view(torch.bfloat16).cuda()
    r = g[f'{case}/r']
    rt = torch.from_numpy(r.view(np.int16)).view(torch.bfloat16).cuda() if r.size else None
    w = torch.from_numpy(g[f'{case}/w'].view(np.int16)).view(torch.bfloat16).cuda()
    q, s, y, summed = K.rmsnorm_quant(x, w, float(g[f'{case}/eps']), rt, want_y=True)
    yk = y.cpu().view(torch.int16).numpy().view(np.uint16)
    ulp = np.abs(yk.astype(int) - g[f'{case}/y_cpu'].astype(int))
    assert ulp.max() <= 1 and (ulp > 0).mean() < 0.01
    if rt is not None:
        assert np.array_equal(summed.cpu().view(torch.int16).numpy().view(np.uint16), g[f'{case}/sum_cpu'])
    q2, s2 = O.quant_act_half_away(O.bf16_bits_to_f32(yk))
    assert np.array_equal(q.cpu().numpy(), q2) and np.array_equal(s.cpu().numpy(), s2)
    # HF Qwen3RMSNorm convention on the same stream
    gam = torch.from_numpy(g[f'{case}/gamma'].view(np.int16)).view(torch.bfloat16).cuda()
    src = summed if rt is not None else x
    _, _, yh, _ = K.rmsnorm_quant(src.contiguous(), gam, float(g[f'{case}/eps']), None, style=1, want_y=True,
                                  want_q=False)
    ulp = np.abs(yh.cpu().view(torch.int16).numpy().view(np.uint16).astype(int) - g[f'{case}/y_hf'].astype(int))
    assert ulp.max() <= 1 and (ulp > 0).mean() < 0.01


@pytest.mark.parametrize('k', [1024, 4096, 8192])
def test_rmsnorm_quant_widths(K, k):
    """Rows up to 4096 wide take the warp-per-row kernel (two register sizings), wider rows the
    block-per-row kernel; both against the oracle, with a residual and the summed stream."""
    m = 300
    g = torch.Generator().manual_seed(k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    r = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gam = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    q, s, y, summed = K.rmsnorm_quant(x.cuda(), gam.cuda(), 1e-6, r.cuda(), style=1, want_y=True)
    yo, so = O.rms_norm(x.float().numpy(), gam.float().numpy(), 1e-6, r.float().numpy(), style='weight')
    assert np.array_equal(to_np(summed), so)
    yk = to_np(y)
    ulp = np.abs(O.f32_to_bf16_bits(yk).astype(int) - O.f32_to_bf16_bits(yo).astype(int))
    assert ulp.max() <= 2 and (ulp > 0).mean() < 0.01
    q2, s2 = O.quant_act_half_away(yk)
    assert np.array_equal(q.cpu().numpy(), q2) and np.array_equal(s.cpu().numpy(), s2)


@pytest.mark.parametrize('m', [1, 33, 4096])
def test_rmsnorm_quant_outliers(K, m):
    k = 2560
    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, k, generator=g)
    ch = torch.randperm(k, generator=g)[:8]
    x[:, ch] *= 50
    x = x.to(torch.bfloat16)
    gam = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    q, s, y, _ = K.rmsnorm_quant(x.cuda(), gam.cuda(), 1e-6, None, style=1, want_y=True)
    yo, _ = O.rms_norm(x.float().numpy(), gam.float().numpy(), 1e-6, None, style='weight')
    yk = to_np(y)
    # HF style rounds twice (normalised value, then times gamma): a 1-ulp difference in
    # the first rounding (summation order) can become 2 ulp after the second, i.e. at most
    # 2^-6 relative just above a power of two
    ulp = np.abs(O.f32_to_bf16_bits(yk).astype(int) - O.f32_to_bf16_bits(yo).astype(int))
    assert ulp.max() <= 2 and (ulp > 0).mean() < 0.01
    assert np.allclose(yk, yo, rtol=2.0 ** -6, atol=0)
    q2, s2 = O.quant_act_half_away(yk)
    assert np.array_equal(q.cpu().numpy(), q2) and np.array_equal(s.cpu().numpy(), s2)


# ---------------------------------------------------------------------------------------
def test_option_logits_golden(K):
    g = golden('readout')
    h = torch.from_numpy(g['a/h'].view(np.int16)).view(torch.bfloat16).cuda()
    gam = torch.from_numpy(g['a/gamma'].view(np.int16)).view(torch.bfloat16).cuda()
    rows = torch.from_numpy(g['a/rows']).cuda()
    lo = torch.from_numpy(g['a/lo']).cuda()
    hi = torch.from_numpy(g['a/hi']).cuda()
    z, p = K.option_logits(h, rows, gam, lo, hi, eps=1e-6, style=1)
    assert np.allclose(z.cpu().numpy(), g['a/logits'], rtol=1e-4, atol=1e-4)
    assert np.abs(p.cpu().numpy() - g['a/probs']).max() < 1e-3


@pytest.mark.parametrize('b,r', [(1, 257), (7, 40), (64, 255)])
def test_option_logits_random(K, b, r):
    d = 2560
    g = torch.Generator().manual_seed(b * r)
    h = torch.randn(b, d, generator=g).to(torch.bfloat16)
    rows = torch.randn(r, d, generator=g) * 0.02
    lo = torch.randint(0, 3, (b,), generator=g, dtype=torch.int32)
    hi = torch.minimum(lo + torch.randint(2, r, (b,), generator=g, dtype=torch.int32), torch.tensor(r, dtype=torch.int32))
    z, p = K.option_logits(h.cuda(), rows.cuda(), None, lo.cuda(), hi.cuda())
    zo, po = O.option_probs(to_np(h), rows.numpy(), lo.numpy(), hi.numpy())
    assert np.allclose(z.cpu().numpy(), zo, rtol=1e-4, atol=1e-4)
    assert np.abs(p.cpu().numpy() - po).max() < 1e-3


# ---------------------------------------------------------------------------------------
def test_bounded_wait_returns_error_status_and_context_survives(K):
    from mica_b200 import _native as N
    st = torch.full((1,), -1, dtype=torch.int32, device='cuda')
    N.call('mica_selftest_wait_timeout', st.data_ptr(), 20000, torch.cuda.current_stream().cuda_stream)
    assert int(st.item()) == 6          # MICA_DEV_TIMEOUT_SELFTEST
    assert dev_error() == 6             # recorded in the device error word, then cleared
    assert dev_error() == 0
    x = torch.randn(4, 64, device='cuda').to(torch.bfloat16)
    assert K.act_quant(x) is not None    # context still usable
    torch.cuda.synchronize()


@pytest.mark.parametrize('mode', ['half_away', 'half_even'])
def test_act_quant_large_random_scales_bit_exact(K, mode):
    """20M quotients with row magnitudes spanning 12 decades: the per-row reciprocal +
    residual division must give the IEEE quotient everywhere (a 1-ulp error would move
    codes that sit within an ulp of a rounding boundary)."""
    m, k = 2048, 9728
    g = torch.Generator().manual_seed(77)
    x = torch.randn(m, k, generator=g) * torch.pow(10.0, torch.rand(m, 1, generator=g) * 12 - 6)
    x[:, torch.randperm(k, generator=g)[:8]] *= 50
    x = x.to(torch.bfloat16)
    K.ROUND['mode'] = mode
    try:
        q, s = K.act_quant(x.cuda())
    finally:
        K.ROUND['mode'] = 'half_away'
    qo, so = O.quant_act(x.float().numpy(), None, mode)
    assert np.array_equal(s.cpu().numpy(), so)
    assert np.array_equal(q.cpu().numpy(), qo)


def test_act_quant_exact_ties_and_boundaries(K):
    """Quotients exactly on .5 boundaries and one ulp either side of them."""
    k = 256
    rows = []
    # x = n/4 for |n| <= 254 (plus one zero): absmax 63.5 gives scale exactly 1/2, so v = n/2
    base = torch.cat([torch.arange(-254, 256, 2, dtype=torch.float32) / 4, torch.zeros(1)])
    for delta in (0.0, 2 ** -7, -(2 ** -7)):
        r = (base + delta).clone()
        r[0] = 63.5                                                            # absmax -> scale exactly 1/2
        rows.append(r)
    x = torch.stack(rows).to(torch.bfloat16)
    for mode in ('half_away', 'half_even'):
        K.ROUND['mode'] = mode
        try:
            q, s = K.act_quant(x.cuda())
        finally:
            K.ROUND['mode'] = 'half_away'
        qo, so = O.quant_act(x.float().numpy(), None, mode)
        assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy(), so)


# ---------------------------------------------------------------------------------------
# SwiGLU + requantisation for MLPs whose gate and up projections are smoothed differently
# (mica_swiglu_quant), and down_proj's smoothing inside the fused gate_up kernel.
@pytest.mark.parametrize('mode', ['half_away', 'half_even'])
@pytest.mark.parametrize('smooth', [False, True])
@pytest.mark.parametrize('m,i', [(1, 64), (37, 256), (608, 9728)])
def test_swiglu_quant_vs_oracle(K, m, i, smooth, mode):
    g = torch.Generator().manual_seed(m + i + smooth)
    gate = (torch.randn(m, i, generator=g) * 3).to(torch.bfloat16)
    up = (torch.randn(m, i, generator=g) * 2).to(torch.bfloat16)
    inv = torch.exp(torch.randn(i, generator=g)) if smooth else None
    K.ROUND['mode'] = mode
    try:
        h, q, s = K.swiglu_quant(gate.cuda(), up.cuda(), None if inv is None else inv.cuda(), want_h=True)
        h_only = K.swi_glu(gate.cuda(), up.cuda())
    finally:
        K.ROUND['mode'] = 'half_away'
    h_ref = O.silu_mul(gate.float().numpy(), up.float().numpy())
    hk = to_np(h)
    assert np.allclose(hk, h_ref, rtol=1e-2, atol=1e-2 * np.abs(h_ref).max())
    assert (hk != h_ref).mean() < 0.01
    assert torch.equal(h_only, h)
    q2, s2 = O.quant_act(hk, None if inv is None else inv.numpy(), mode)
    assert np.array_equal(s.cpu().numpy(), s2)
    assert np.array_equal(q.cpu().numpy(), q2)


@pytest.mark.parametrize('m,i,k', [(37, 256, 2560), (1024, 9728, 2560)])
def test_gemm_swiglu_quant_down_smoothing(K, m, i, k):
    """inv_h (down_proj's inv_smooth): the fused requantisation quantises h * inv_h."""
    g = torch.Generator().manual_seed(m * 3 + i)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    sx = torch.rand(m, generator=g) * 0.02 + 1e-3
    wg = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    wu = torch.randint(-127, 128, (i, k), generator=g, dtype=torch.int8)
    sg = torch.rand(i, generator=g) * 9e-3 + 1e-3
    su = torch.rand(i, generator=g) * 9e-3 + 1e-3
    inv = torch.exp(torch.randn(i, generator=g))
    qw = torch.from_numpy(O.interleave_gate_up(wg.numpy(), wu.numpy())).contiguous()
    sw = torch.from_numpy(O.interleave_gate_up(sg.numpy(), su.numpy())).contiguous()
    h, q, s = K.mm_i8_swiglu_quant(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda(), None, inv.cuda())
    h_ref, _, _ = O.gate_up_swiglu_quant(qx.numpy(), sx.numpy(), wg.numpy(), sg.numpy(), wu.numpy(), su.numpy())
    hk = to_np(h)
    assert np.allclose(hk, h_ref, rtol=1e-2, atol=1e-2 * np.abs(h_ref).max())
    q2, s2 = O.quant_act_half_away(hk, inv.numpy())
    assert np.array_equal(s.cpu().numpy(), s2)
    assert np.array_equal(q.cpu().numpy(), q2)
    assert dev_error() == 0


def test_gemm_into_column_slices_bit_exact(K):
    """w8a8_gemm_into writes each projection into its column slice of one q|k|v buffer."""
    m, k = 300, 512
    g = torch.Generator().manual_seed(5)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8).cuda()
    sx = (torch.rand(m, generator=g) * 0.05 + 1e-3).cuda()
    out = torch.full((m, 384), 7.0, dtype=torch.bfloat16, device='cuda')
    refs = []
    for lo, hi in ((0, 256), (256, 320), (320, 384)):
        w = torch.randint(-127, 128, (hi - lo, k), generator=g, dtype=torch.int8).cuda()
        sw = (torch.rand(hi - lo, generator=g) * 9e-3 + 1e-3).cuda()
        torch.ops.mica.w8a8_gemm_into(qx, sx, w, sw, None, out[:, lo:hi], 0)
        refs.append(torch.ops.mica.w8a8_gemm(qx, sx, w, sw, None, 0, 0))
    assert torch.equal(out, torch.cat(refs, dim=1))


# ---------------------------------------------------------------------------------------
# Split-K across a cluster (the K loop of one tile over S CTAs, partials summed in
# distributed shared memory): every forced split factor is bit-exact.
def _valid_split(k, s):
    kb = (k + 127) // 128
    per = (kb + s - 1) // s
    return (s - 1) * per < kb


@pytest.mark.parametrize('splits', [1, 2, 3, 5, 8])
@pytest.mark.parametrize('bn', [64, 128, 256])
@pytest.mark.parametrize('m,n,k', [(1, 256, 4096), (130, 320, 2560), (256, 2560, 9728), (77, 96, 1040)])
def test_gemm_split_k_bit_exact(K, m, n, k, bn, splits):
    if not _valid_split(k, splits):
        pytest.skip('a rank would get no k-block')
    g = torch.Generator().manual_seed(m + n + k + bn + splits)
    lo = 31 if k > 1024 else 127                    # |acc| < 2^24: the fp32 output is the exact int32
    qx = torch.randint(-lo, lo + 1, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-lo, lo + 1, (n, k), generator=g, dtype=torch.int8)
    tile = splits * 1000000 + 128000 + bn
    y = torch.ops.mica.w8a8_gemm(qx.cuda(), torch.ones(m).cuda(), qw.cuda(), torch.ones(n).cuda(), None, 2, tile)
    acc = O.int_gemm_exact(qx.numpy(), qw.numpy())
    assert np.array_equal(y.cpu().numpy().astype(np.int64), acc.astype(np.int64))
    # dequant epilogue with bias, bf16
    sx = torch.rand(m, generator=g) * 0.05 + 1e-3
    sw = torch.rand(n, generator=g) * 9e-3 + 1e-3
    bias = torch.randn(n, generator=g) * 0.1
    yb = torch.ops.mica.w8a8_gemm(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda(), bias.cuda(), 0, tile)
    ref = O.dequant_out(acc, sx.numpy(), sw.numpy(), bias.numpy(), out='bf16')
    assert np.array_equal(to_np(yb.float()), ref)
    assert dev_error() == 0


# ---------------------------------------------------------------------------------------
# Stream-K (one CTA per SM, equal runs of (tile, k-block) units, a cut tile finished from its
# neighbour's int32 partial): bit-exact against the oracle and the data-parallel kernel.
@pytest.mark.parametrize('bn', [128, 256])
@pytest.mark.parametrize('m,n,k', [(512, 9728, 2560), (2048, 2560, 4096), (1000, 9704, 2576), (77, 96, 1040),
                                   (256, 19456, 2560)])
def test_gemm_stream_k_bit_exact(K, m, n, k, bn):
    g = torch.Generator().manual_seed(m + n + k + bn)
    lo = 31 if k > 1024 else 127                    # |acc| < 2^24: the fp32 output is the exact int32
    qx = torch.randint(-lo, lo + 1, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-lo, lo + 1, (n, k), generator=g, dtype=torch.int8)
    sk, dp = 9000000 + 128000 + bn, 1000000 + 128000 + bn
    qxc, qwc = qx.cuda(), qw.cuda()
    y = torch.ops.mica.w8a8_gemm(qxc, torch.ones(m).cuda(), qwc, torch.ones(n).cuda(), None, 2, sk)
    acc = O.int_gemm_exact(qx.numpy(), qw.numpy())
    assert np.array_equal(y.cpu().numpy().astype(np.int64), acc.astype(np.int64))
    sx = (torch.rand(m, generator=g) * 0.05 + 1e-3).cuda()
    sw = (torch.rand(n, generator=g) * 9e-3 + 1e-3).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).cuda()
    yb = torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, 0, sk)
    ref = O.dequant_out(acc, sx.cpu().numpy(), sw.cpu().numpy(), bias.cpu().numpy(), out='bf16')
    assert np.array_equal(to_np(yb.float()), ref)
    for code in (0, 1):
        assert torch.equal(torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, code, sk),
                           torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, code, dp))
    assert dev_error() == 0


def test_gemm_stream_k_library_choice(K):
    """A grid of one to two waves with a long, mostly empty second wave that 128 x 320 tiles
    cannot fit in one wave (M 2048, N 3072, K 9728: 192 tiles of 128 x 256 on 148 SMs, 76
    k-blocks each) runs as stream-K by default, with the data-parallel kernel's output; so does
    the strided-output form. Grids that 128 x 320 tiles cover in one wave (config 0, M 2048 with
    N 2560) and many-wave grids use no workspace. Without a workspace the forced form is refused
    and the library choice runs data-parallel."""
    from mica_b200 import _native as N
    lib = N.lib()
    assert lib.mica_w8a8_gemm_workspace_bytes(512, 9728, 2560, 0, 0, 0, 0) == 0
    assert lib.mica_w8a8_gemm_workspace_bytes(2048, 2560, 9728, 0, 0, 0, 0) == 0
    assert lib.mica_w8a8_gemm_workspace_bytes(32768, 2560, 9728, 0, 0, 0, 0) == 0
    assert lib.mica_w8a8_gemm_workspace_bytes(512, 9728, 2560, 128, 256, 0, N.SPLIT_STREAM_K) > 0
    m, n, k = 2048, 3072, 9728
    assert lib.mica_w8a8_gemm_workspace_bytes(m, n, k, 0, 0, 0, 0) > 0
    assert lib.mica_w8a8_gemm_workspace_bytes(m, n, k, 0, 0, 0, 1) == 0
    g = torch.Generator(device='cuda').manual_seed(3)
    qx = torch.randint(-127, 128, (m, k), generator=g, device='cuda', dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, device='cuda', dtype=torch.int8)
    sx = torch.rand(m, generator=g, device='cuda') * 0.05 + 1e-3
    sw = torch.rand(n, generator=g, device='cuda') * 9e-3 + 1e-3
    y0 = torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, 0)
    y1 = torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, 1128256)
    assert torch.equal(y0, y1)
    out = torch.zeros((m, n + 64), dtype=torch.bfloat16, device='cuda')
    torch.ops.mica.w8a8_gemm_into(qx, sx, qw, sw, None, out[:, 32:32 + n], 0)
    assert torch.equal(out[:, 32:32 + n], y1) and not out[:, :32].any() and not out[:, 32 + n:].any()
    y2 = torch.empty_like(y1)
    stream = torch.cuda.current_stream().cuda_stream
    args = (qx.data_ptr(), k, qw.data_ptr(), k, sx.data_ptr(), sw.data_ptr(), None, y2.data_ptr(), 0, n, m, n, k)
    assert N.lib().mica_w8a8_gemm_cfg(*args, 128, 256, 0, N.SPLIT_STREAM_K, stream) == 7     # ERR_WORKSPACE
    assert N.lib().mica_w8a8_gemm_ex(*args, 0, 0, 0, 0, None, 0, stream) == 0              # data-parallel
    torch.cuda.synchronize()
    assert torch.equal(y2, y1)
    assert dev_error() == 0


def test_gemm_stream_k_in_a_cuda_graph(K):
    """The stream-K plan (flag clear + cooperative launch, workspace from the graph's pool)
    captures into a CUDA graph; replays on new inputs give the data-parallel kernel's output."""
    m, n, k = 2048, 3072, 9728
    g = torch.Generator(device='cuda').manual_seed(9)
    qx = torch.randint(-127, 128, (m, k), generator=g, device='cuda', dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, device='cuda', dtype=torch.int8)
    sx = torch.rand(m, generator=g, device='cuda') * 0.05 + 1e-3
    sw = torch.rand(n, generator=g, device='cuda') * 9e-3 + 1e-3
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, 0)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, 0)
    for seed in (1, 2):
        gg = torch.Generator(device='cuda').manual_seed(seed)
        qx.copy_(torch.randint(-127, 128, (m, k), generator=gg, device='cuda', dtype=torch.int8))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, 1128256)), seed
    del graph
    assert dev_error() == 0


# ---------------------------------------------------------------------------------------
# 128 x 320 tiles (two 160-wide MMAs per k-step, one accumulator buffer, one tile per CTA):
# the library's choice when 128 x 256 tiles just exceed one wave (config 0). Bit-exact.
@pytest.mark.parametrize('m,n,k', [(512, 9728, 2560), (2048, 2560, 4096), (500, 9000, 2576), (77, 96, 1040),
                                   (256, 19456, 2560)])
def test_gemm_wide_tile_bit_exact(K, m, n, k):
    g = torch.Generator().manual_seed(m + 2 * n + k)
    lo = 31 if k > 1024 else 127                    # |acc| < 2^24: the fp32 output is the exact int32
    qx = torch.randint(-lo, lo + 1, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-lo, lo + 1, (n, k), generator=g, dtype=torch.int8)
    qxc, qwc = qx.cuda(), qw.cuda()
    y = torch.ops.mica.w8a8_gemm(qxc, torch.ones(m).cuda(), qwc, torch.ones(n).cuda(), None, 2, 128320)
    acc = O.int_gemm_exact(qx.numpy(), qw.numpy())
    assert np.array_equal(y.cpu().numpy().astype(np.int64), acc.astype(np.int64))
    sx = (torch.rand(m, generator=g) * 0.05 + 1e-3).cuda()
    sw = (torch.rand(n, generator=g) * 9e-3 + 1e-3).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).cuda()
    yb = torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, 0, 128320)
    ref = O.dequant_out(acc, sx.cpu().numpy(), sw.cpu().numpy(), bias.cpu().numpy(), out='bf16')
    assert np.array_equal(to_np(yb.float()), ref)
    for code in (0, 1):
        assert torch.equal(torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, code, 128320),
                           torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, code, 1128256))
    assert torch.equal(torch.ops.mica.w8a8_gemm(qxc, sx, qwc, sw, bias, 0, 0), yb)   # library choice
    assert dev_error() == 0


def test_gemm_wide_tile_needs_one_wave(K):
    """A forced 128 x 320 tile on a grid larger than one wave is refused before any launch."""
    from mica_b200 import _native as N
    m, n, k = 32768, 2560, 256
    qx = torch.zeros((m, k), dtype=torch.int8, device='cuda')
    qw = torch.zeros((n, k), dtype=torch.int8, device='cuda')
    s = torch.ones(max(m, n), device='cuda')
    y = torch.empty((m, n), dtype=torch.bfloat16, device='cuda')
    st = torch.cuda.current_stream().cuda_stream
    rc = N.lib().mica_w8a8_gemm_cfg(qx.data_ptr(), k, qw.data_ptr(), k, s.data_ptr(), s.data_ptr(), None,
                                    y.data_ptr(), 0, n, m, n, k, 128, 320, 0, 0, st)
    assert rc == 8                                   # MICA_ERR_UNSUPPORTED
    assert dev_error() == 0


def test_automatic_width_keeps_256_when_the_caller_forces_a_split_or_caps_the_grid(K):
    """Config 0's shape (M 512, N 9728, K 2560) is where the library choice takes 128 x 320
    tiles. With the width left to the library but a forced cluster split, a forced stream-K or
    a grid cap below one wave, it must keep a 256-wide path: a 320-wide choice would refuse
    each of these (MICA_ERR_UNSUPPORTED). Every form is bit-exact against the oracle."""
    from mica_b200 import _native as N
    lib = N.lib()
    m, n, k = 512, 9728, 2560
    g = torch.Generator().manual_seed(512)
    qx = torch.randint(-31, 32, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-31, 32, (n, k), generator=g, dtype=torch.int8)
    acc = O.int_gemm_exact(qx.numpy(), qw.numpy()).astype(np.int64)
    qxc, qwc = qx.cuda(), qw.cuda()
    ones = torch.ones(max(m, n), device='cuda')
    st = torch.cuda.current_stream().cuda_stream
    F32 = 2
    for max_ctas, splits in ((0, 2), (0, 4), (100, 0), (0, 1)):
        y = torch.full((m, n), -1.0, dtype=torch.float32, device='cuda')
        rc = lib.mica_w8a8_gemm_cfg(qxc.data_ptr(), k, qwc.data_ptr(), k, ones.data_ptr(), ones.data_ptr(), None,
                                    y.data_ptr(), F32, n, m, n, k, 0, 0, max_ctas, splits, st)
        assert rc == 0, (max_ctas, splits, rc)
        assert np.array_equal(y.cpu().numpy().astype(np.int64), acc), (max_ctas, splits)
    need = lib.mica_w8a8_gemm_workspace_bytes(m, n, k, 0, 0, 0, -1)
    assert need > 0                                  # stream-K planned: a 256- or 128-wide tile
    ws = torch.empty(need, dtype=torch.uint8, device='cuda')
    y = torch.full((m, n), -1.0, dtype=torch.float32, device='cuda')
    rc = lib.mica_w8a8_gemm_ex(qxc.data_ptr(), k, qwc.data_ptr(), k, ones.data_ptr(), ones.data_ptr(), None,
                               y.data_ptr(), F32, n, m, n, k, 0, 0, 0, -1, ws.data_ptr(), need, st)
    assert rc == 0
    assert np.array_equal(y.cpu().numpy().astype(np.int64), acc)
    assert dev_error() == 0
