"""The INT8 weights file (int8-w8a8/1, the reference's lib/int8_runtime.py:639-726) on CPU:
reading, ties, validation errors, and how a file's smoothing maps onto the decoder's fused
and split paths. The golden folder tests/golden/model_int8/ was written by the reference's
own convert (tests/golden/make_golden.py)."""
import json

import pytest
import torch

from conftest import GOLDEN

from mica_b200 import int8_runtime as R
from mica_b200 import prefill as P

FOLDER = GOLDEN / 'model_int8'


def test_reads_the_reference_converted_file():
    t, ties = R.read_int8_file(FOLDER)
    assert ties == {'lm_head.weight': 'model.embed_tokens.weight'}
    assert t['lm_head.weight'] is t['model.embed_tokens.weight']
    assert t['model.layers.0.self_attn.q_proj.qweight'].dtype == torch.int8
    assert t['model.layers.1.mlp.gate_proj.inv_smooth'].dtype == torch.float32
    assert 'model.layers.0.mlp.gate_proj.inv_smooth' not in t


def test_config_from_file_matches_config_json():
    t, ties = R.read_int8_file(FOLDER)
    from_json = P.config_from_hf(json.loads((FOLDER / 'config.json').read_text()))
    assert P.config_from_int8(t, ties) == from_json


def test_smoothing_selects_fused_or_split_paths():
    m = P.load_model(FOLDER, 'cpu')
    l0, l1, l2 = m.layers
    # layer 0: no smoothing -> one q|k|v part, fused gate|up
    assert l0.parts() == [(0, l0.qkv_w.shape[0], None)] and l0.split_mlp is None and l0.down_inv is None
    # layer 1: per-projection smoothing -> three q/k/v parts, split gate/up
    assert [(a, b) for a, b, _ in l1.parts()] == [(0, 128), (128, 192), (192, 256)]
    assert all(inv is not None for _, _, inv in l1.parts())
    assert l1.gu_w is None and l1.split_mlp is not None and l1.distinct_mlp_invs() == 2
    assert l1.o_inv is not None and l1.down_inv is not None
    # layer 2: only o and down smoothed -> fused paths, down smoothing in the requant
    assert l2.qkv_parts is None and l2.split_mlp is None and l2.down_inv is not None and l2.o_inv is not None
    assert m.lm_head is None                                    # tied to the embedding
    # the stored int8 weights are used as they are
    t, _ = R.read_int8_file(FOLDER)
    assert torch.equal(l1.qkv_w[128:192], t['model.layers.1.self_attn.k_proj.qweight'])
    assert torch.equal(l1.split_mlp[4], t['model.layers.1.mlp.up_proj.qweight'])
    assert torch.equal(l0.gu_w, R.interleave_gate_up(t['model.layers.0.mlp.gate_proj.qweight'],
                                                     t['model.layers.0.mlp.up_proj.qweight']))


def test_write_read_round_trip(tmp_path):
    t, ties = R.read_int8_file(FOLDER)
    R.write_int8_file(tmp_path / R.FILE, t, ties)
    t2, ties2 = R.read_int8_file(tmp_path)
    assert ties2 == ties and set(t2) == set(t)
    assert all(torch.equal(t[k], t2[k]) for k in t)


def _rewrite(tmp_path, edit, ties=None, meta_format=None):
    t, tz = R.read_int8_file(FOLDER)
    t = dict(t)
    edit(t)
    tz = tz if ties is None else ties
    path = tmp_path / R.FILE
    if meta_format is None:
        R.write_int8_file(path, t, tz)
    else:
        from safetensors.torch import save_file
        save_file({k: v.contiguous() for k, v in t.items() if k not in tz}, str(path),
                  metadata={'format': meta_format, 'ties': json.dumps(tz)})
    return tmp_path


@pytest.mark.parametrize('case', ['format', 'tie', 'dtype', 'shape', 'gdn_key', 'missing'])
def test_invalid_files_raise_invalid_model(tmp_path, case):
    def nothing(t):
        pass

    if case == 'format':
        folder = _rewrite(tmp_path, nothing, meta_format='int8-w8a8/0')
    elif case == 'tie':
        folder = _rewrite(tmp_path, nothing, ties={'lm_head.weight': 'model.nowhere.weight'})
    elif case == 'dtype':
        folder = _rewrite(tmp_path, lambda t: t.update({'model.layers.0.mlp.up_proj.wscale':
                                                        t['model.layers.0.mlp.up_proj.wscale'].double()}))
    elif case == 'shape':
        folder = _rewrite(tmp_path, lambda t: t.update({'model.layers.2.self_attn.o_proj.inv_smooth':
                                                        torch.ones(7)}))
    elif case == 'gdn_key':      # a hybrid (GDN) layer's projection: not a dense decoder
        folder = _rewrite(tmp_path, lambda t: t.update({'model.layers.0.linear_attn.in_proj_qkv.qweight':
                                                        torch.zeros(16, 128, dtype=torch.int8)}))
    else:
        folder = _rewrite(tmp_path, lambda t: t.pop('model.layers.1.self_attn.k_norm.weight'))
    with pytest.raises(R.InvalidModel, match='invalid_model'):
        P.load_model(folder, 'cpu', cfg=P.config_from_hf(json.loads((FOLDER / 'config.json').read_text())))
