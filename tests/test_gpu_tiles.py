"""`--kernel-tune full` on the device (the reference's kernel_state pin/restore/capture,
v0.5/serving/lib/kernel_state.py:111-256): the tuner times every tile kind on two small
shapes, persists the winners in a state dir, and the serving path (int8_kernels.mm_i8) then
runs the chosen codes bit-exact against the oracle."""
import json

import numpy as np
import pytest
import torch

from conftest import ORACLE as O

pytestmark = pytest.mark.gpu


def test_tune_two_shapes_into_a_state_dir_and_serve_them(tmp_path):
    import mica_b200.int8_kernels as K
    from mica_b200 import tiles
    shapes = [(2560, 4096, 2048), (2560, 9728, 256)]        # O at M 2048 (class l), down at M 256 (class m)
    try:
        res = tiles.tune(shapes, reps=3, state_dir=tmp_path)
        saved = json.loads((tmp_path / tiles.STATE_NAME).read_text())['entries']
        assert set(res) == {tiles.key(n, k, m) for n, k, m in shapes} and saved == res
        assert all(tiles.valid(c) for c in res.values())
        for n, k, m in shapes:
            assert K.gemm_tile(n, k, m) == tiles.effective(res[tiles.key(n, k, m)], n, m, K.caps().sm_count)
            g = torch.Generator().manual_seed(n + m)
            x = torch.randn(m, k, generator=g).to(torch.bfloat16)
            qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
            sw = torch.rand(n, generator=g) * 9e-3 + 1e-3
            q, s = K.act_quant(x.cuda())
            y = K.mm_i8(q, s, qw.cuda(), sw.cuda())
            qo, so = O.quant_act_half_away(x.float().numpy())
            ref = O.dequant_out(O.int_gemm_exact(qo, qw.numpy()), so, sw.numpy())
            assert np.array_equal(y.float().cpu().numpy(), ref)
    finally:
        tiles.set_state_dir(None)


@pytest.mark.parametrize('m', [300, 512, 1024, 2048])
def test_pinned_wide_tile_entries_follow_the_library_where_they_do_not_fit(m):
    """A 128 x 320 entry serves only M whose grid fits one wave; at other M of the same class
    the call takes the library's choice, and both are bit-exact."""
    import mica_b200.int8_kernels as K
    from mica_b200 import tiles
    n, k = 9728, 2560
    sms = K.caps().sm_count
    code = tiles.effective(128320, n, m, sms)
    assert code == (128320 if ((m + 127) // 128) * ((n + 319) // 320) <= sms else 0)
    g = torch.Generator().manual_seed(m)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sx = torch.rand(m, generator=g) * 1e-2 + 1e-3
    sw = torch.rand(n, generator=g) * 9e-3 + 1e-3
    y = torch.ops.mica.w8a8_gemm(qx.cuda(), sx.cuda(), qw.cuda(), sw.cuda(), None, 0, code)
    ref = O.dequant_out(O.int_gemm_exact(qx.numpy(), qw.numpy()), sx.numpy(), sw.numpy())
    assert np.array_equal(y.float().cpu().numpy(), ref)
