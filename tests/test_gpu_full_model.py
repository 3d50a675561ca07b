"""The north-star correctness target at BASELINE scale: option probabilities of the 4B-dims,
36-layer, vocab-151936 decoder (config 3's model) scored by this library, against the
reference's own scoring of the same weights and requests (tests/golden/model_full.npz, made
by make_golden.py with HF Qwen3ForCausalLM + the reference's int8_runtime.convert 'emulate'
+ the restated readout). Both sides regenerate the weights from full_model.py's seeds.

Bar: max |dp| < 1e-3 over the 255 options, at 2048 and at 32768 tokens."""
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden

pytestmark = pytest.mark.gpu

if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))
import full_model as FM  # noqa: E402


@pytest.fixture(scope='module')
def full():
    from mica_b200 import prefill as P
    if not (GOLDEN / 'model_full.npz').is_file():
        pytest.fail('tests/golden/model_full.npz is missing (make_golden.py ... model_full)')
    cfg = P.DecoderConfig()
    assert (cfg.hidden, cfg.inter, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab) == (
        FM.HF_CONFIG['hidden_size'], FM.HF_CONFIG['intermediate_size'], FM.HF_CONFIG['num_hidden_layers'],
        FM.HF_CONFIG['num_attention_heads'], FM.HF_CONFIG['num_key_value_heads'], FM.HF_CONFIG['head_dim'],
        FM.HF_CONFIG['vocab_size'])
    model = P.from_hf_state(FM.state(), cfg, torch.device('cuda'))
    yield model, golden('model_full')
    del model
    torch.cuda.empty_cache()


@pytest.mark.parametrize('n', FM.LENGTHS)
def test_full_scale_option_probs_match_reference(full, n):
    import mica_b200.int8_kernels as K
    from mica_b200 import prefill as P
    model, g = full
    ids, rows = FM.request(n)
    assert np.array_equal(ids.numpy(), g[f'n{n}/ids']) and np.array_equal(rows.numpy(), g[f'n{n}/rows'])
    lo, hi = (int(v) for v in g[f'n{n}/slice'])
    pf = P.Prefill(model, rows, max_len=max(FM.LENGTHS))
    K.ROUND['mode'] = 'half_even'      # the reference's QLinear 'emulate' path rounds half to even
    try:
        z, p = pf.score(ids.cuda(), lo, hi, graphs=False)
    finally:
        K.ROUND['mode'] = 'half_away'
    p = p.cpu().numpy()
    z = z.cpu().numpy()
    ref_p, ref_z = g[f'n{n}/probs'], g[f'n{n}/logits']
    dp = np.abs(p - ref_p).max()
    dz = np.abs(z - ref_z).max()
    print(f'{n} tokens: max |dp| {dp:.2e} (probs up to {ref_p.max():.2e}), max |dz| {dz:.2e}')
    assert dp < 1e-3
    assert dz < 5e-2 * max(1.0, float(np.abs(ref_z).max()))
    assert abs(float(p.sum()) - 1.0) < 1e-5
    assert float(np.abs(p[:, :lo]).sum()) == 0.0


def test_full_scale_weights_quantise_like_the_reference(full):
    """The int8 weights and channel scales built on the GPU equal the reference quantiser's
    (int8_quant.quant_weight, restated by the oracle) on the CPU, for one layer's projections."""
    from conftest import ORACLE as O
    model, _ = full
    lay = model.layers[7]
    specs = {name: (i, shape, kind) for i, (name, shape, kind) in enumerate(FM.tensor_specs())}
    p = 'model.layers.7.'
    w = torch.cat([FM.make_tensor(*specs[p + f'self_attn.{n}_proj.weight']) for n in 'qkv'])
    q_ref, s_ref = O.quant_weight(w.float().numpy())
    assert np.array_equal(lay.qkv_w.cpu().numpy(), q_ref)
    assert np.array_equal(lay.qkv_s.cpu().numpy(), s_ref)
    d = FM.make_tensor(*specs[p + 'mlp.down_proj.weight'])
    q_ref, s_ref = O.quant_weight(d.float().numpy())
    assert np.array_equal(lay.down_w.cpu().numpy(), q_ref)
    assert np.array_equal(lay.down_s.cpu().numpy(), s_ref)
