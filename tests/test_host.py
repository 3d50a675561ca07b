"""Host-side logic that needs no GPU: the reference-facing surface's miss contract, weight
conversion, gate/up interleave, tile table, and the failure paths."""
import numpy as np
import pytest
import torch

from conftest import ORACLE as O


def test_available_reports_no_cuda_here_or_sm100_there():
    import mica_b200.int8_kernels as K
    ok, why = K.available()
    if not torch.cuda.is_available():
        assert not ok and 'CUDA' in why
    else:
        assert isinstance(ok, bool)


def test_misses_return_none_and_count_reasons_like_the_reference():
    import mica_b200.int8_kernels as K
    before = dict(K.STATS['fallback'])
    assert K.act_quant(torch.zeros(4, 64)) is None                      # CPU tensor
    assert K.mm_i8(torch.zeros(4, 64), torch.ones(4), torch.zeros(8, 64, dtype=torch.int8), torch.ones(8)) is None
    assert K.attn_fwd(None, None, None, 1.0) is None
    after = K.STATS['fallback']
    assert after['act_input'] == before.get('act_input', 0) + 1
    assert after['mm_input'] == before.get('mm_input', 0) + 1
    assert after['no_cubin'] == before.get('no_cubin', 0) + 1
    assert K.attn_keys() == []


def test_qlinear_weight_conversion_matches_reference_quant_weight():
    from mica_b200.int8_runtime import QLinear
    g = torch.Generator().manual_seed(0)
    lin = torch.nn.Linear(256, 48, bias=True)
    lin.weight.data = (torch.randn(48, 256, generator=g) * 0.05).to(torch.bfloat16)
    lin.bias.data = torch.randn(48, generator=g).to(torch.bfloat16)
    q = QLinear(lin)
    qo, so = O.quant_weight(lin.weight.detach().float().numpy())
    assert np.array_equal(q.qweight.numpy(), qo) and np.array_equal(q.wscale.numpy(), so)
    assert q.bias.dtype == torch.float32 and q.inv_smooth is None
    assert q.out_dtype == torch.bfloat16 and q.in_features == 256 and q.out_features == 48
    w = q.weight
    assert w.shape == (48, 256) and w.dtype == torch.bfloat16


def test_qlinear_smoothing_folds_into_weights():
    from mica_b200.int8_runtime import QLinear, smooth_factors
    g = torch.Generator().manual_seed(1)
    lin = torch.nn.Linear(128, 32, bias=False)
    lin.weight.data = torch.randn(32, 128, generator=g) * 0.05
    amax = torch.rand(128, generator=g) * 4 + 0.05
    sm = smooth_factors(amax, lin.weight.detach())
    smo = O.smooth_factors(amax.numpy(), lin.weight.detach().numpy())
    assert np.allclose(sm.numpy(), smo, rtol=1e-6)
    q = QLinear(lin, sm)
    assert torch.allclose(q.inv_smooth * sm, torch.ones(128), rtol=1e-6)


def test_qlinear_empty_has_meta_buffers():
    from mica_b200.int8_runtime import QLinear
    q = QLinear.empty(2560, 9728, smooth=True, bias=False)
    assert q.qweight.device.type == 'meta' and q.qweight.shape == (9728, 2560) and q.inv_smooth.shape == (2560,)


def test_qlinear_rejects_emulate_backend():
    from mica_b200.int8_runtime import QLinear
    with pytest.raises(ValueError):
        QLinear(torch.nn.Linear(16, 16), backend='emulate')


def test_qlinear_forward_raises_loudly_without_the_gpu_path():
    from mica_b200.int8_runtime import KernelMiss, QLinear
    q = QLinear(torch.nn.Linear(64, 32))
    with pytest.raises(KernelMiss):
        q(torch.randn(3, 64).to(torch.bfloat16))


def test_interleave_gate_up_matches_oracle_layout():
    from mica_b200.int8_runtime import interleave_gate_up
    g = torch.arange(64 * 5).reshape(64, 5)
    u = -g
    assert np.array_equal(interleave_gate_up(g, u).numpy(), O.interleave_gate_up(g.numpy(), u.numpy()))
    s = torch.arange(64.0)
    assert np.array_equal(interleave_gate_up(s, -s).numpy(), O.interleave_gate_up(s.numpy(), -s.numpy()))
    with pytest.raises(ValueError):
        interleave_gate_up(torch.zeros(24, 3), torch.zeros(24, 3))


def test_fused_mlp_builds_from_hf_qwen3_mlp():
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3MLP

    from mica_b200.int8_runtime import FusedMLP
    cfg = Qwen3Config(hidden_size=128, intermediate_size=256)
    mlp = Qwen3MLP(cfg)
    f = FusedMLP(mlp)
    assert f.qweight_gu.shape == (512, 128) and f.wscale_gu.shape == (512,)
    assert f.down.qweight.shape == (128, 256)
    # the first 16 rows are gate rows, the next 16 up rows
    qg, _ = O.quant_weight(mlp.gate_proj.weight.detach().numpy())
    qu, _ = O.quant_weight(mlp.up_proj.weight.detach().numpy())
    assert np.array_equal(f.qweight_gu[:16].numpy(), qg[:16]) and np.array_equal(f.qweight_gu[16:32].numpy(), qu[:16])


def test_convert_replaces_every_projection():
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3Model

    from mica_b200.int8_runtime import FusedMLP, QLinear, convert
    cfg = Qwen3Config(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, vocab_size=100)
    body = Qwen3Model(cfg)
    n, sm = convert(body, None)
    assert (n, sm) == (14, 0)
    assert isinstance(body.layers[0].self_attn.q_proj, QLinear)
    body2 = Qwen3Model(cfg)
    n, _ = convert(body2, None, fuse_mlp=True)
    assert n == 14 and isinstance(body2.layers[1].mlp, FusedMLP)


def test_tile_table_keys_use_reference_m_classes(tmp_path):
    from mica_b200 import tiles
    assert [tiles.m_class(m) for m in (1, 128, 129, 384, 385, 1024, 1025)] == ['s', 's', 'm', 'm', 'n', 'n', 'l']
    assert tiles.key(6144, 2560, 4096) == 'mm|N6144|K2560|cl'
    (tmp_path / tiles.STATE_NAME).write_text('{"format": "mica-tiles/1", "entries": {"mm|N64|K64|cs": 256128}}')
    tiles.set_state_dir(tmp_path)
    try:
        assert tiles.tile(64, 64, 7) == 256128
        assert tiles.tile(64, 64, 700) == 0
    finally:
        tiles.set_state_dir(None)


def test_native_errors_name_the_status():
    from mica_b200 import _native as N
    with pytest.raises(N.NativeError, match='ERR_SHAPE'):
        N.check('mica_x', 2)


def test_decoder_from_hf_state_quantises_like_reference_qlinear():
    """The golden tiny model's weights, converted on CPU, give the reference QLinear codes."""
    from conftest import golden
    from mica_b200 import prefill as P
    g = golden('model')
    bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    state = {k[len('m/state/'):]: bf(g[k]) for k in g.files if k.startswith('m/state/')}
    cfg = P.DecoderConfig(hidden=128, inter=256, layers=3, heads=2, kv_heads=1, head_dim=64, vocab=512)
    m = P.from_hf_state(state, cfg, torch.device('cpu'))
    assert len(m.layers) == 3 and m.lm_head is None
    lay = m.layers[1]
    assert lay.qkv_w.shape == (256, 128) and lay.gu_w.shape == (512, 128) and lay.down_w.shape == (128, 256)
    q_ref, s_ref = O.quant_weight(state['model.layers.1.self_attn.k_proj.weight'].float().numpy())
    assert np.array_equal(lay.qkv_w[128:192].numpy(), q_ref) and np.array_equal(lay.qkv_s[128:192].numpy(), s_ref)
    g_ref, _ = O.quant_weight(state['model.layers.1.mlp.gate_proj.weight'].float().numpy())
    assert np.array_equal(lay.gu_w[:16].numpy(), g_ref[:16]) and np.array_equal(lay.gu_w[32:48].numpy(), g_ref[16:32])
    cos, sin = P.rope_tables(cfg, 16, torch.device('cpu'))
    assert cos.shape == (16, 64) and cos.dtype == torch.bfloat16 and float(cos[0, 0]) == 1.0


def test_tile_codes_decode_to_the_c_arguments():
    """splits * 10**6 + block_m * 1000 + block_n; splits digit 9 asks for stream-K."""
    from mica_b200 import _native as N
    from mica_b200.ops import _tile_args
    assert _tile_args(0) == (0, 0, 0, 0)
    assert _tile_args(128256) == (128, 256, 0, 0)
    assert _tile_args(128320) == (128, 320, 0, 0)
    assert _tile_args(256256) == (256, 256, 0, 0)
    assert _tile_args(1128064) == (128, 64, 0, 1)
    assert _tile_args(4128256) == (128, 256, 0, 4)
    assert _tile_args(9128256) == (128, 256, 0, N.SPLIT_STREAM_K)


def test_workspace_size_memo_is_bounded():
    """The per-shape memo of stream-K workspace sizes stays bounded however many token counts
    a server sees (here the library answers 0: no device)."""
    from mica_b200 import ops
    ops._WS_BYTES.clear()
    for m in range(1, ops._WS_CACHE_MAX + 500):
        assert ops._workspace_bytes(0, m, 2560, 9728, 0) == 0
    assert 0 < len(ops._WS_BYTES) <= ops._WS_CACHE_MAX
    ops._WS_BYTES.clear()


def test_fused_kernels_drop_in_has_no_cpu_path():
    """fused_kernels.rms_norm / swi_glu keep the reference's names and arguments but, unlike
    the reference module, serve CUDA tensors only: a CPU tensor raises RuntimeError (which
    the reference's caller, fork.rms_norm_fused, catches) instead of computing on the CPU."""
    from mica_b200 import fused_kernels as ffk
    x = torch.zeros(2, 3, 64, dtype=torch.bfloat16)
    w = torch.zeros(64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match='CUDA'):
        ffk.rms_norm(x, w, 1e-6)
    with pytest.raises(RuntimeError, match='CUDA'):
        ffk.rms_norm(x, w, 1e-6, torch.zeros_like(x))
    with pytest.raises(RuntimeError, match='CUDA'):
        ffk.swi_glu(x, x)
    import inspect
    assert list(inspect.signature(ffk.rms_norm).parameters) == ['x', 'weight', 'eps', 'residual']
    assert list(inspect.signature(ffk.swi_glu).parameters) == ['gate', 'up']


def test_tile_codes_the_tuner_weighs_are_all_valid_and_the_table_drops_others(tmp_path):
    """The tuner's candidates cover every kind of tile the library has (library choice,
    128-row 64/128/256/320, CTA pairs, never-split, forced K splits 2..8, stream-K); a state
    file's unknown codes are ignored, and a 320-wide entry applies only where its grid fits
    one wave (elsewhere the call takes the library's choice)."""
    from mica_b200 import tiles
    assert all(tiles.valid(c) for c in tiles.CHOICES)
    kinds = {c // 1000000 for c in tiles.CHOICES}
    assert kinds == set(range(0, 9)) | {9}
    assert 128320 in tiles.CHOICES and 0 in tiles.CHOICES and 256256 in tiles.CHOICES
    for bad in (-1, 128000, 128512, 256064, 256320, 2256256, 2128320, 9128064, 10128128, 128096):
        assert not tiles.valid(bad), bad
    assert all(tiles.valid(v) for v in tiles._load(tiles.PINNED).values())
    (tmp_path / tiles.STATE_NAME).write_text(
        '{"format": "mica-tiles/1", "entries": {"mm|N64|K64|cs": 2256256, "mm|N64|K64|cm": "x", '
        '"mm|N9728|K2560|cm": 128320, "mm|N64|K64|cl": 9128256}}')
    loaded = tiles._load(tmp_path / tiles.STATE_NAME)
    assert loaded == {'mm|N9728|K2560|cm': 128320, 'mm|N64|K64|cl': 9128256}
    tiles.set_state_dir(tmp_path)
    try:
        assert tiles.tile(9728, 2560, 300, sms=148) == 128320       # 3 x 31 = 93 tiles: one wave
        assert tiles.tile(9728, 2560, 384, sms=148) == 128320
        assert tiles.effective(128320, 9728, 640, 148) == 0           # 5 x 31 = 155 tiles
        assert tiles.tile(9728, 2560, 300) == 128320                   # no SM count: as stored
        assert tiles.tile(64, 64, 5000, sms=148) == 9128256
    finally:
        tiles.set_state_dir(None)
