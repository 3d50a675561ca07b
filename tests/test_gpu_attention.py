"""The tcgen05 attention forward (mica_attention_prefill) against an fp32 attention of the same
bf16 q, k, v: causal, grouped-query, per request of a [B, L] batch, read in place from a QKV
projection buffer. Tolerance: the kernel rounds P to bf16 for the second MMA and its output to
bf16, so outputs are compared within 2e-2 of the largest |o| (mean error below 2e-3 of it)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _reference(qkv, B, L, H, KV, D, scale):
    q, k, v = qkv.float().split([H * D, KV * D, KV * D], dim=1)
    q = q.view(B, L, H, D).transpose(1, 2)
    k = k.view(B, L, KV, D).transpose(1, 2).repeat_interleave(H // KV, dim=1)
    v = v.view(B, L, KV, D).transpose(1, 2).repeat_interleave(H // KV, dim=1)
    s = (q @ k.transpose(-1, -2)) * scale
    mask = torch.ones(L, L, dtype=torch.bool, device=qkv.device).tril()
    p = s.masked_fill(~mask, float('-inf')).softmax(-1)
    return (p @ v).transpose(1, 2).reshape(B * L, H * D)


@pytest.mark.parametrize('B,L,H,KV', [(1, 128, 4, 2), (1, 333, 32, 8), (2, 256, 8, 8), (3, 200, 16, 4),
                                      (1, 2048, 32, 8), (2, 1000, 4, 1), (1, 1, 8, 2), (2, 127, 4, 4),
                                      (1, 129, 4, 2), (3, 257, 8, 2)])
def test_attention_matches_fp32_reference(B, L, H, KV):
    from mica_b200 import ops  # noqa: F401
    D = 128
    g = torch.Generator(device='cuda').manual_seed(B * 7919 + L + H)
    qkv = torch.randn(B * L, (H + 2 * KV) * D, generator=g, device='cuda').to(torch.bfloat16)
    scale = D ** -0.5
    o = torch.ops.mica.attention_prefill(qkv, B, L, H, KV, scale)
    ref = _reference(qkv, B, L, H, KV, D, scale)
    err = (o.float() - ref).abs()
    big = float(ref.abs().max())
    assert float(err.max()) < 2e-2 * big, (float(err.max()), big)
    assert float(err.mean()) < 2e-3 * big


def test_attention_matches_sdpa_on_a_strided_qkv_buffer():
    """q/k/v taken in place from a wider buffer (row stride above (H + 2 KV) D), as the prefill's
    per-part GEMMs can leave it; the same result as torch SDPA on the extracted heads."""
    from mica_b200 import ops  # noqa: F401
    B, L, H, KV, D = 2, 384, 8, 2, 128
    g = torch.Generator(device='cuda').manual_seed(3)
    wide = torch.randn(B * L, (H + 2 * KV) * D + 64, generator=g, device='cuda').to(torch.bfloat16)
    qkv = wide[:, :(H + 2 * KV) * D]
    o = torch.ops.mica.attention_prefill(qkv, B, L, H, KV, D ** -0.5)
    q, k, v = qkv.split([H * D, KV * D, KV * D], dim=1)
    ref = F.scaled_dot_product_attention(q.reshape(B, L, H, D).transpose(1, 2), k.reshape(B, L, KV, D).transpose(1, 2),
                                         v.reshape(B, L, KV, D).transpose(1, 2), is_causal=True, enable_gqa=True)
    ref = ref.transpose(1, 2).reshape(B * L, H * D).float()
    err = (o.float() - ref).abs()
    assert float(err.max()) < 2e-2 * float(ref.abs().max())


def test_attention_rejects_bad_arguments():
    from mica_b200 import _native as N
    lib = N.lib()
    buf = torch.empty(16, dtype=torch.bfloat16, device='cuda')
    st = torch.cuda.current_stream().cuda_stream
    assert lib.mica_attention_prefill(None, 1536, buf.data_ptr(), 1024, 1, 8, 8, 2, 128, 0.1, st) == 1   # null
    assert lib.mica_attention_prefill(buf.data_ptr(), 1536, buf.data_ptr(), 1024, 1, 8, 8, 3, 128, 0.1, st) == 2  # H % KV
    assert lib.mica_attention_prefill(buf.data_ptr(), 1536, buf.data_ptr(), 1024, 1, 8, 8, 2, 64, 0.1, st) == 2   # D
    assert lib.mica_attention_prefill(buf.data_ptr(), 1535, buf.data_ptr(), 1024, 1, 8, 4, 2, 128, 0.1, st) == 3  # stride


def test_attention_of_an_empty_batch_is_a_no_op():
    """B = 0 or L = 0: nothing to compute; the call succeeds and launches nothing."""
    from mica_b200 import _native as N
    lib = N.lib()
    buf = torch.zeros(16, dtype=torch.bfloat16, device='cuda')
    st = torch.cuda.current_stream().cuda_stream
    assert lib.mica_attention_prefill(buf.data_ptr(), 1536, buf.data_ptr(), 1024, 0, 8, 8, 2, 128, 0.1, st) == 0
    assert lib.mica_attention_prefill(buf.data_ptr(), 1536, buf.data_ptr(), 1024, 2, 0, 8, 2, 128, 0.1, st) == 0
    torch.cuda.synchronize()
    assert float(buf.float().abs().sum()) == 0.0
