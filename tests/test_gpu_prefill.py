"""Prefill scoring on the W8A8 kernels: option probabilities against the reference's own
scoring of the same tiny Qwen3 model (tests/golden/model.npz, made by running the
reference's int8_runtime.convert + readout), plus size-independent checks at full dims."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

TINY = dict(hidden=128, inter=256, layers=3, heads=2, kv_heads=1, head_dim=64, vocab=512, eps=1e-6,
            rope_theta=1e6, tie_embeddings=True)


def _bf16(a):
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)


@pytest.fixture(scope='module')
def tiny():
    from mica_b200 import prefill as P
    g = golden('model')
    state = {k[len('m/state/'):]: _bf16(g[k]) for k in g.files if k.startswith('m/state/')}
    cfg = P.DecoderConfig(**TINY)
    model = P.from_hf_state(state, cfg, torch.device('cuda'))
    return P.Prefill(model, torch.from_numpy(g['m/options']), max_len=512), g


@pytest.mark.parametrize('i', [0, 1])
def test_tiny_model_probs_match_reference(tiny, i):
    import mica_b200.int8_kernels as K
    pf, g = tiny
    ids = torch.from_numpy(g[f'm/ids{i}']).cuda()
    lo, hi = (int(v) for v in g[f'm/slice{i}'])
    K.ROUND['mode'] = 'half_even'      # the reference's QLinear 'emulate' path rounds half to even
    try:
        z, p = pf.score(ids, lo, hi, graphs=False)
        z_full, p_full = pf.probs(pf.hidden_last(ids, last_only=False), torch.tensor([lo], dtype=torch.int32,
                                  device='cuda'), torch.tensor([hi], dtype=torch.int32, device='cuda'))
    finally:
        K.ROUND['mode'] = 'half_away'
    ref_p, ref_z = g[f'm/probs{i}'], g[f'm/logits{i}']
    assert np.abs(p.cpu().numpy() - ref_p).max() < 1e-3
    assert np.abs(z.cpu().numpy() - ref_z).max() < 2e-2 * max(1.0, float(np.abs(ref_z).max()))
    assert np.abs(p_full.cpu().numpy() - ref_p).max() < 1e-3
    assert abs(float(p.sum()) - 1.0) < 1e-5


def test_tiny_graph_replay_matches_eager(tiny):
    pf, g = tiny
    ids = torch.from_numpy(g['m/ids1']).cuda()          # 100 tokens -> bucket 128
    z_e, p_e = pf.score(ids, 0, 40, graphs=False)
    pf.capture(128)
    z_g, p_g = (t.clone() for t in pf.score(ids, 0, 40))
    assert torch.allclose(p_g, p_e, atol=1e-3, rtol=0)
    # a second request through the same graph (other length, other slice)
    ids2 = torch.from_numpy(g['m/ids0']).cuda()
    z2, p2 = (t.clone() for t in pf.score(ids2, 2, 19))
    z2e, p2e = pf.score(ids2, 2, 19, graphs=False)
    assert torch.allclose(p2, p2e, atol=1e-3, rtol=0)
    assert float(p2[0, :2].abs().sum()) == 0.0 and float(p2[0, 19:].abs().sum()) == 0.0
    pf.release()


def test_full_dims_last_row_path_matches_full_path():
    """4B dims (2 layers): the last-layer row restriction gives the full computation's row."""
    from mica_b200 import prefill as P
    cfg = P.DecoderConfig(layers=2, vocab=4096)
    model = P.random_decoder(cfg, torch.device('cuda'), seed=3)
    options = torch.arange(2, 259)
    pf = P.Prefill(model, options, max_len=4096)
    ids = torch.randint(0, cfg.vocab, (1500,), generator=torch.Generator().manual_seed(5)).cuda()
    z1, p1 = pf.score(ids, graphs=False)
    z2, p2 = pf.probs(pf.hidden_last(ids, last_only=False))
    assert torch.isfinite(p1).all()
    assert abs(float(p1.sum()) - 1.0) < 1e-4
    assert torch.allclose(p1, p2, atol=1e-3, rtol=0)


def test_full_dims_36_layers_scores_finite_and_deterministic():
    from mica_b200 import prefill as P
    cfg = P.DecoderConfig(vocab=8192)
    model = P.random_decoder(cfg, torch.device('cuda'), seed=11)
    pf = P.Prefill(model, torch.arange(0, 257), max_len=4096)
    ids = torch.randint(0, cfg.vocab, (4000,), generator=torch.Generator().manual_seed(6)).cuda()
    a = pf.score(ids, 2, 257, graphs=False)[1].clone()
    b = pf.score(ids, 2, 257, graphs=False)[1].clone()
    assert torch.isfinite(a).all() and abs(float(a.sum()) - 1.0) < 1e-4
    assert torch.equal(a, b)


@pytest.mark.parametrize('S,H,KV', [(333, 32, 8), (64, 4, 2)])
def test_qk_norm_rope_bit_exact_against_fixed_order_restatement(S, H, KV):
    """The D = 128 kernel equals the oracle's restatement of the HF op sequence bit for bit
    (the restatement fixes the sum of squares to the kernel's order): no step may be fused or
    re-rounded. Rows scaled by 1e-3 and 50 and scattered positions included."""
    from conftest import ORACLE as O
    from mica_b200 import ops  # noqa: F401
    from mica_b200 import prefill as P
    D = 128
    g = torch.Generator(device='cuda').manual_seed(S + 3 * H)
    qkv = (torch.randn(S, (H + 2 * KV) * D, generator=g, device='cuda') * 3).to(torch.bfloat16)
    qkv[:5] *= 1e-3
    qkv[5:7] *= 50
    qw = (1 + 0.1 * torch.randn(D, generator=g, device='cuda')).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device='cuda')).to(torch.bfloat16)
    cos, sin = P.rope_tables(P.DecoderConfig(head_dim=D), 8192, torch.device('cuda'))
    pos = torch.randint(0, 8192, (S,), generator=g, device='cuda')
    before = qkv.float().cpu().numpy()
    torch.ops.mica.qk_norm_rope(qkv, qw, kw, cos, sin, pos, 0, H, KV, 1e-6)
    after = qkv.float().cpu().numpy()
    c = cos[pos].float().cpu().numpy()
    sn = sin[pos].float().cpu().numpy()
    for h in range(H + KV):
        w = (qw if h < H else kw).float().cpu().numpy()
        want = O.qk_norm_rope(before[:, h * D:(h + 1) * D], w, c, sn, 1e-6)
        assert np.array_equal(after[:, h * D:(h + 1) * D], want), h
    assert np.array_equal(after[:, (H + KV) * D:], before[:, (H + KV) * D:])


def _hf_qk(x, w, cos, sin, eps):
    """HF Qwen3 q_norm/k_norm + apply_rotary_pos_emb as torch bf16 ops (the reference)."""
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    y = w * n
    h = y.shape[-1] // 2
    rot = torch.cat((-y[..., h:], y[..., :h]), dim=-1)
    return (y * cos[:, None, :]) + (rot * sin[:, None, :])


@pytest.mark.parametrize('S,H,KV', [(1, 32, 8), (333, 32, 8), (2048, 4, 2)])
def test_qk_norm_rope_matches_hf_torch_ops(S, H, KV):
    from mica_b200 import ops  # noqa: F401
    from mica_b200 import prefill as P
    D = 128
    g = torch.Generator(device='cuda').manual_seed(S + H)
    qkv = (torch.randn(S, (H + 2 * KV) * D, generator=g, device='cuda') * 3).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(D, generator=g, device='cuda')).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device='cuda')).to(torch.bfloat16)
    cfg = P.DecoderConfig(head_dim=D)
    cos, sin = P.rope_tables(cfg, 4096, torch.device('cuda'))
    pos0 = 100
    ref_q = _hf_qk(qkv[:, :H * D].view(S, H, D), qw, cos[pos0:pos0 + S], sin[pos0:pos0 + S], 1e-6)
    ref_k = _hf_qk(qkv[:, H * D:(H + KV) * D].view(S, KV, D), kw, cos[pos0:pos0 + S], sin[pos0:pos0 + S], 1e-6)
    v_before = qkv[:, (H + KV) * D:].clone()
    torch.ops.mica.qk_norm_rope(qkv, qw, kw, cos, sin, None, pos0, H, KV, 1e-6)
    got_q = qkv[:, :H * D].view(S, H, D)
    got_k = qkv[:, H * D:(H + KV) * D].view(S, KV, D)
    for got, ref in ((got_q, ref_q), (got_k, ref_k)):
        # the rotation adds two rounded terms; near cancellation a 1-ulp difference in the
        # normalised input is many ulps of the small sum, so compare values, not ulps
        assert torch.allclose(got.float(), ref.float(), rtol=1e-2, atol=2e-2)
        assert float((got != ref).float().mean()) < 0.01
    assert torch.equal(qkv[:, (H + KV) * D:], v_before)


def test_eager_padding_matches_unpadded_run(tiny):
    """Eager requests are padded to a 256-token bucket with `limit`: same scores as the
    unpadded computation (within attention-kernel rounding)."""
    pf, g = tiny
    ids = torch.from_numpy(g['m/ids1']).cuda()                 # 100 tokens -> padded to 256
    z_pad, p_pad = (t.clone() for t in pf.score(ids, 0, 40, graphs=False))
    z_raw, p_raw = pf.probs(pf.hidden_last(ids), torch.tensor([0], dtype=torch.int32, device='cuda'),
                            torch.tensor([40], dtype=torch.int32, device='cuda'))
    assert pf.eager_bucket(100) == 256
    assert torch.allclose(p_pad, p_raw, atol=1e-3, rtol=0)


def test_startup_selftest_like_the_reference():
    from mica_b200 import int8_runtime as rt
    res = rt.selftest([(6144, 2560, False), (2560, 4096, True), (2560, 9728, False)], 'cuda')
    assert res['ok'], res
    assert res['checked'] == 3 * 2 * len(rt.SELFTEST_ROWS)
    assert res['worst_ratio'] <= rt.SELFTEST_TOL


@pytest.mark.parametrize('attention', ['sdpa', 'mica'])
def test_batched_scoring_matches_single_requests(attention):
    """[B, L] batches (padded, per-request limits and option slices) give each request the
    probabilities it gets alone (within attention-kernel rounding), with either attention."""
    from mica_b200 import prefill as P
    cfg = P.DecoderConfig(layers=3, vocab=4096)
    model = P.random_decoder(cfg, torch.device('cuda'), seed=21)
    pf = P.Prefill(model, torch.arange(0, 257), max_len=4096, attention=attention)
    gen = torch.Generator().manual_seed(8)
    lens = [300, 511, 64, 1000, 777]
    ids = [torch.randint(0, cfg.vocab, (n,), generator=gen).cuda() for n in lens]
    slices = [(2, 2 + 10 * (i + 1)) for i in range(len(lens))]
    zb, pb = pf.score_batch(ids, slices)
    for i, t in enumerate(ids):
        z1, p1 = pf.score(t, *slices[i], graphs=False)
        assert torch.allclose(pb[i:i + 1], p1, atol=2e-3, rtol=0), i
        assert abs(float(pb[i].sum()) - 1.0) < 1e-4


@pytest.mark.parametrize('attention', ['sdpa', 'mica'])
def test_batch_graph_replay_matches_eager_batch(attention):
    """A captured [B, L] batch graph replays each new batch (ids, limits and option slices
    copied into its static buffers) with the eager batch's results, and its outputs are the
    caller's own (a later replay does not overwrite them)."""
    from mica_b200 import prefill as P
    cfg = P.DecoderConfig(layers=3, vocab=4096)
    model = P.random_decoder(cfg, torch.device('cuda'), seed=22)
    pf = P.Prefill(model, torch.arange(0, 257), max_len=4096, attention=attention)
    gen = torch.Generator().manual_seed(12)
    batches = [[300, 511, 64, 1000], [1024, 700, 1, 999]]
    ids = [[torch.randint(0, cfg.vocab, (n,), generator=gen).cuda() for n in lens] for lens in batches]
    slices = [[(2, 2 + 10 * (i + 1)) for i in range(4)], [(0, 257), (5, 6), (2, 100), (2, 257)]]
    with pytest.raises(ValueError):
        pf.capture_batch(4, 1000)
    pf.capture_batch(4, 1024)
    got = [pf.score_batch(t, s) for t, s in zip(ids, slices)]
    for (zg, pg), t, s in zip(got, ids, slices):
        ze, pe = pf.score_batch(t, s, graphs=False)
        assert torch.allclose(pg, pe, atol=1e-3, rtol=0)
        assert torch.allclose(zg, ze, atol=2e-2, rtol=1e-2)
        for i, (lo, hi) in enumerate(s):
            assert abs(float(pg[i].sum()) - 1.0) < 1e-4
            assert float(pg[i, :lo].abs().sum()) == 0.0 and float(pg[i, hi:].abs().sum()) == 0.0
    assert not torch.equal(got[0][1], got[1][1])
    pf.release()
    assert not pf.batch_graphs


# ---------------------------------------------------------------------------------------
# A model read from an int8-w8a8/1 weights folder written by the reference's convert with
# activation statistics: per-projection smoothing (split q/k/v and gate/up paths), down and
# o smoothing, tied lm_head. Probabilities against the converted reference model's own.
@pytest.fixture(scope='module')
def int8_file_model():
    from conftest import GOLDEN
    from mica_b200 import prefill as P
    g = golden('model_int8')
    model = P.load_model(GOLDEN / 'model_int8', 'cuda')
    return P.Prefill(model, torch.from_numpy(g['m/options']), max_len=512), g


@pytest.mark.parametrize('i', [0, 1])
def test_int8_file_model_probs_match_reference(int8_file_model, i):
    import mica_b200.int8_kernels as K
    pf, g = int8_file_model
    ids = torch.from_numpy(g[f'm/ids{i}']).cuda()
    lo, hi = (int(v) for v in g[f'm/slice{i}'])
    K.ROUND['mode'] = 'half_even'      # the reference's QLinear 'emulate' path rounds half to even
    try:
        z, p = pf.score(ids, lo, hi, graphs=False)
        pf.capture(pf.bucket(int(ids.shape[0])))
        zg, pg = (t.clone() for t in pf.score(ids, lo, hi, graphs=True))
        pf.release()
        z_full, p_full = pf.probs(pf.hidden_last(ids, last_only=False), torch.tensor([lo], dtype=torch.int32,
                                                                                      device='cuda'),
                                  torch.tensor([hi], dtype=torch.int32, device='cuda'))
    finally:
        K.ROUND['mode'] = 'half_away'
    ref_p, ref_z = g[f'm/probs{i}'], g[f'm/logits{i}']
    assert np.abs(p.cpu().numpy() - ref_p).max() < 1e-3
    assert np.abs(z.cpu().numpy() - ref_z).max() < 2e-2 * max(1.0, float(np.abs(ref_z).max()))
    assert torch.allclose(pg, p, atol=1e-3, rtol=0)                     # graph replay vs eager
    assert np.abs(p_full.cpu().numpy() - p.cpu().numpy()).max() < 1e-3   # last-row restriction


def test_mica_attention_matches_sdpa_in_the_prefill():
    """The same 3-layer 4B-width decoder scored with this library's attention and with SDPA
    (cuDNN). Per-token int8 requantisation turns attention rounding into quantisation-noise-sized
    differences, so the bar is the spread between two of torch's own attention kernels (cuDNN
    against flash, or the math kernel where flash is absent) on the same model: within 3x that,
    plus 1e-3."""
    from torch.nn.attention import SDPBackend
    from mica_b200 import prefill as P
    cfg = P.DecoderConfig(layers=3, vocab=4096)
    model = P.random_decoder(cfg, torch.device('cuda'), seed=23)
    cudnn = P.Prefill(model, torch.arange(0, 257), max_len=4096, attn_backends=[SDPBackend.CUDNN_ATTENTION])
    eff = P.Prefill(model, torch.arange(0, 257), max_len=4096,
                    attn_backends=[SDPBackend.FLASH_ATTENTION, SDPBackend.MATH])
    mica = P.Prefill(model, torch.arange(0, 257), max_len=4096, attention='mica')
    gen = torch.Generator().manual_seed(13)
    for n in (2048, 4000):
        ids = torch.randint(0, cfg.vocab, (n,), generator=gen).cuda()
        _, pc = cudnn.score(ids, 2, 257, graphs=False)
        _, pe = eff.score(ids, 2, 257, graphs=False)
        _, pm = mica.score(ids, 2, 257, graphs=False)
        spread = float((pe - pc).abs().max())
        dp = float((pm - pc).abs().max())
        print(f'{n} tokens: mica vs cuDNN {dp:.3g}, flash vs cuDNN {spread:.3g}')
        assert dp <= 3 * spread + 1e-3, (dp, spread)
        assert abs(float(pm.sum()) - 1.0) < 1e-5
    with pytest.raises(ValueError):
        P.Prefill(model, torch.arange(0, 257), max_len=4096, attention='flash')
