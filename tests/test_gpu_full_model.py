"""The north-star correctness target at BASELINE scale: the 4B-dims, 36-layer, vocab-151936
decoder (config 3's model) scored by this library against the reference's own scoring of the
same weights and requests. Both sides regenerate the weights from full_model.py's seeds.

Goldens (tests/golden/, made by make_golden.py running the reference on the CPU):
  model_full.npz       HF Qwen3ForCausalLM + the reference's int8_runtime.convert ('emulate')
                       + the restated readout, SDPA attention, at 2048 and 32768 tokens;
  model_full_band.npz  the same reference with its attention computed in fp32;
  model_layer0.npz     layer 0's intermediates (last 4 rows) of the 2048-token request.

Why the full-depth bar is the reference's own spread and not 1e-3: the reference moves its
own option probabilities by 6.9e-3 (2048 tokens) and 1.5e-2 (32768 tokens) when only its
attention's rounding changes (bf16 SDPA -> fp32). Every per-token int8 quantisation of a
random-init layer turns an ulp-level input change into a change of the size of its own
quantisation noise, and 36 layers carry that to the logits. So no two valid implementations
(the reference's two attentions, this library's cuDNN or fp32 attention) agree to 1e-3 at this
depth; measured pairwise, they differ by 5e-3 to 2.7e-2. The bar is therefore 2x the
reference's self-spread (two valid implementations can sit on opposite sides of it), and the
strict checks move to layer 0 at full dims: given the reference's input to each step, this
library's step reproduces the reference's output bit for bit (or within the one ulp that the
norm's summation order and silu's exp allow). The full-depth probabilities say little on their
own: leaving the last of the 36 layers out moves them by only 9.5e-3 at 2048 tokens."""
import sys

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN, ORACLE, golden

pytestmark = pytest.mark.gpu

if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))
import full_model as FM  # noqa: E402


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope='module')
def full():
    from mica_b200 import prefill as P
    for name in ('model_full', 'model_full_band'):
        if not (GOLDEN / f'{name}.npz').is_file():
            pytest.fail(f'tests/golden/{name}.npz is missing (make_golden.py ... {name})')
    cfg = P.DecoderConfig()
    assert (cfg.hidden, cfg.inter, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab) == (
        FM.HF_CONFIG['hidden_size'], FM.HF_CONFIG['intermediate_size'], FM.HF_CONFIG['num_hidden_layers'],
        FM.HF_CONFIG['num_attention_heads'], FM.HF_CONFIG['num_key_value_heads'], FM.HF_CONFIG['head_dim'],
        FM.HF_CONFIG['vocab_size'])
    model = P.from_hf_state(FM.state(), cfg, torch.device('cuda'))
    yield model, golden('model_full'), golden('model_full_band')
    del model
    torch.cuda.empty_cache()


@pytest.mark.parametrize('attention', ['sdpa', 'mica'])
@pytest.mark.parametrize('n', FM.LENGTHS)
def test_full_scale_option_probs_within_the_reference_self_spread(full, n, attention):
    """attention 'mica' runs the 35 full-length layers' attention on this library's tcgen05
    kernel instead of cuDNN: the same bar holds."""
    import mica_b200.int8_kernels as K
    from mica_b200 import prefill as P
    model, g, band = full
    ids, rows = FM.request(n)
    assert np.array_equal(ids.numpy(), g[f'n{n}/ids']) and np.array_equal(rows.numpy(), g[f'n{n}/rows'])
    lo, hi = (int(v) for v in g[f'n{n}/slice'])
    pf = P.Prefill(model, rows, max_len=max(FM.LENGTHS), attention=attention)
    K.ROUND['mode'] = 'half_even'      # the reference's QLinear 'emulate' path rounds half to even
    try:
        z, p = pf.score(ids.cuda(), lo, hi, graphs=False)
    finally:
        K.ROUND['mode'] = 'half_away'
    p, z = p.cpu().numpy(), z.cpu().numpy()
    ref_p, ref_z = g[f'n{n}/probs'], g[f'n{n}/logits']
    self_p = np.abs(ref_p - band[f'n{n}/probs']).max()        # the reference against itself
    self_z = np.abs(ref_z - band[f'n{n}/logits']).max()
    dp, dz = np.abs(p - ref_p).max(), np.abs(z - ref_z).max()
    print(f'{n} tokens, {attention}: max |dp| {dp:.3g} (reference self-spread {self_p:.3g}, probs up to {ref_p.max():.3g}); '
          f'max |dz| {dz:.3g} (self-spread {self_z:.3g})')
    assert dp <= 2 * self_p
    assert dz <= 2 * self_z
    assert abs(float(p.sum()) - 1.0) < 1e-5
    assert float(np.abs(p[:, :lo]).sum()) == 0.0 and float(np.abs(p[:, hi:]).sum()) == 0.0


def test_full_scale_weights_quantise_like_the_reference(full):
    """The int8 weights and channel scales built on the GPU equal the reference quantiser's
    (int8_quant.quant_weight, restated by the oracle) on the CPU, for one layer's projections."""
    model, _, _ = full
    lay = model.layers[7]
    specs = {name: (i, shape, kind) for i, (name, shape, kind) in enumerate(FM.tensor_specs())}
    p = 'model.layers.7.'
    w = torch.cat([FM.make_tensor(*specs[p + f'self_attn.{n}_proj.weight']) for n in 'qkv'])
    q_ref, s_ref = ORACLE.quant_weight(w.float().numpy())
    assert np.array_equal(lay.qkv_w.cpu().numpy(), q_ref)
    assert np.array_equal(lay.qkv_s.cpu().numpy(), s_ref)
    d = FM.make_tensor(*specs[p + 'mlp.down_proj.weight'])
    q_ref, s_ref = ORACLE.quant_weight(d.float().numpy())
    assert np.array_equal(lay.down_w.cpu().numpy(), q_ref)
    assert np.array_equal(lay.down_s.cpu().numpy(), s_ref)


def test_layer0_at_full_dims_reproduces_the_reference_step_by_step():
    """Layer 0 of the full-dims decoder, last 4 rows of the 2048-token request: fed the
    reference's input to each step, each of this library's steps gives the reference's output.
    o_proj (quantiser + W8A8 GEMM) and down_proj are bit-exact, the residual-added RMSNorm is
    within 1 ulp, the fused gate_up + SwiGLU within 1e-2 with at most 1 % of elements one ulp
    off (silu's exp), and the layer output is bit-exact."""
    import mica_b200.int8_kernels as K
    from mica_b200 import _native as N
    from mica_b200 import prefill as P
    g = golden('model_layer0')
    dev = torch.device('cuda')
    cfg = P.DecoderConfig(layers=1)
    m = P.from_hf_state(FM.state(1), cfg, dev)
    lay = m.layers[0]
    pf = P.Prefill(m, torch.arange(0, 8), max_len=2048)
    ids, _ = FM.request(2048)
    emb = F.embedding(ids[-4:].to(dev), m.embed)
    K.ROUND['mode'] = 'half_even'
    try:
        attn = _bf16(g['l0/attn']).to(dev)
        qa, sa = torch.ops.mica.act_quant(attn, None, K._round_code())
        o = pf._gemm(qa, sa, lay.o_w, lay.o_s)
        assert np.array_equal(_bits(o), g['l0/o_proj'])
        _, _, y, summed = torch.ops.mica.rmsnorm_quant(o, emb, lay.post_norm, None, cfg.eps, N.NORM_WEIGHT,
                                                        K._round_code(), True, True)
        ulp = np.abs(_bits(y).astype(int) - g['l0/ln2'].astype(int))
        assert ulp.max() <= 1 and (ulp > 0).mean() < 0.01
        ln2 = _bf16(g['l0/ln2']).to(dev)
        q2, s2 = torch.ops.mica.act_quant(ln2, None, K._round_code())
        h, _, _ = torch.ops.mica.gemm_swiglu_quant(q2, s2, lay.gu_w, lay.gu_s, None, None, K._round_code())
        hk, hr = h.float().cpu().numpy(), ORACLE.bf16_bits_to_f32(g['l0/h'])
        assert np.allclose(hk, hr, rtol=1e-2, atol=1e-2 * np.abs(hr).max())
        assert (hk != hr).mean() < 0.01
        qh, sh = torch.ops.mica.act_quant(_bf16(g['l0/h']).to(dev), None, K._round_code())
        d = pf._gemm(qh, sh, lay.down_w, lay.down_s)
        assert np.array_equal(_bits(d), g['l0/down'])
        out = summed + d
        ref_mid = (_bf16(g['l0/o_proj']).float() + emb.cpu().float()).to(torch.bfloat16)
        assert np.array_equal(_bits(summed), _bits(ref_mid))
        assert np.array_equal(_bits(out), g['l0/layer_out'])
    finally:
        K.ROUND['mode'] = 'half_away'
