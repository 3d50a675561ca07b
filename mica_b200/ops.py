"""PyTorch custom ops over the libmica_w8a8 C ABI.

Each op allocates its outputs with torch (so CUDA-graph capture draws them from the
graph's pool, as the reference's torch.empty outputs do, v0.5/serving/lib/
int8_kernels.py:343-344, :376) and launches on torch's current stream of the input's
device (:261-265). Fake (meta) implementations let torch.compile and graph tooling see
shapes without running anything.

    torch.ops.mica.act_quant(x, inv, round_mode)                       -> (q, s)
    torch.ops.mica.rmsnorm_quant(x, residual, gamma, inv, eps, style, round_mode, want_y)
                                                                        -> (q, s, y, sum)
    torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, bias, out_dtype, tile)     -> y
    torch.ops.mica.w8a8_gemm_into(qx, sx, qw, sw, bias, out, tile)      (writes out, a row-strided view)
    torch.ops.mica.gemm_swiglu_quant(qx, sx, qw_gu, sw_gu, bias, inv_h, round_mode) -> (h, q, s)
    torch.ops.mica.swiglu_quant(g, u, inv, round_mode, want_h, want_q) -> (h, q, s)
    torch.ops.mica.option_logits(h, rows, gamma, lo, hi, eps, style)    -> (logits, probs)
    torch.ops.mica.qk_norm_rope(qkv, q_w, k_w, cos, sin, pos, pos0, heads, kv_heads, eps)  (in place)
    torch.ops.mica.attention_prefill(qkv, B, L, heads, kv_heads, scale)  -> o [B * L, heads * D]
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _native as N

DTYPE_CODE = {torch.bfloat16: N.DT_BF16, torch.float16: N.DT_FP16, torch.float32: N.DT_FP32}
OUT_DTYPES = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class _on:
    """Makes the tensor's device current for the C side (cudaGetDevice)."""

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.idx:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev != self.idx:
            torch.cuda.set_device(self.prev)


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::act_quant', mutates_args=())
def act_quant(x: torch.Tensor, inv: Optional[torch.Tensor], round_mode: int) -> tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    with _on(x):
        N.call('mica_act_quant', x.data_ptr(), DTYPE_CODE[x.dtype], x.stride(0), _ptr(inv), q.data_ptr(), q.stride(0),
               s.data_ptr(), m, k, round_mode, _stream(x))
    return q, s


@act_quant.register_fake
def _(x, inv, round_mode):
    m, k = x.shape
    return x.new_empty((m, k), dtype=torch.int8), x.new_empty((m,), dtype=torch.float32)


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::rmsnorm_quant', mutates_args=())
def rmsnorm_quant(x: torch.Tensor, residual: Optional[torch.Tensor], gamma: torch.Tensor, inv: Optional[torch.Tensor],
                  eps: float, style: int, round_mode: int, want_y: bool, want_q: bool
                  ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    m, k = x.shape
    dev = x.device
    q = torch.empty((m, k) if want_q else (0,), dtype=torch.int8, device=dev)
    s = torch.empty((m,) if want_q else (0,), dtype=torch.float32, device=dev)
    y = torch.empty((m, k) if want_y else (0,), dtype=x.dtype, device=dev)
    sm = torch.empty((m, k) if residual is not None else (0,), dtype=x.dtype, device=dev)
    with _on(x):
        N.call('mica_rmsnorm_quant', x.data_ptr(), DTYPE_CODE[x.dtype], x.stride(0),
               _ptr(residual), residual.stride(0) if residual is not None else 0,
               gamma.data_ptr(), style, eps, _ptr(inv),
               y.data_ptr() if want_y else None, k if want_y else 0,
               sm.data_ptr() if residual is not None else None, k if residual is not None else 0,
               q.data_ptr() if want_q else None, k if want_q else 0, s.data_ptr() if want_q else None,
               m, k, round_mode, _stream(x))
    return q, s, y, sm


@rmsnorm_quant.register_fake
def _(x, residual, gamma, inv, eps, style, round_mode, want_y, want_q):
    m, k = x.shape
    return (x.new_empty((m, k) if want_q else (0,), dtype=torch.int8),
            x.new_empty((m,) if want_q else (0,), dtype=torch.float32),
            x.new_empty((m, k) if want_y else (0,)),
            x.new_empty((m, k) if residual is not None else (0,)))


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::w8a8_gemm', mutates_args=())
def w8a8_gemm(qx: torch.Tensor, sx: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor, bias: Optional[torch.Tensor],
              out_dtype: int, tile: int) -> torch.Tensor:
    """tile = splits * 10**6 + block_m * 1000 + block_n (e.g. 256256 = CTA pair, 256 x 256;
    1128064 = 128 x 64 never split; 4128256 = 128 x 256 split four ways; 9128256 = 128 x 256
    stream-K), 0 = library choice."""
    m, k = qx.shape
    n = qw.shape[0]
    out = torch.empty((m, n), dtype=OUT_DTYPES[out_dtype], device=qx.device)
    _gemm(qx, sx, qw, sw, bias, out, out_dtype, tile)
    return out


def _tile_args(tile: int):
    """(block_m, block_n, max_ctas, splits) of a tile code (splits digit 9 = stream-K)."""
    splits = tile // 1000000
    return (tile // 1000) % 1000, tile % 1000, 0, N.SPLIT_STREAM_K if splits == 9 else splits


_WS_BYTES = {}
_WS_CACHE_MAX = 4096       # shapes remembered; a server sees many token counts, so it is bounded


def _workspace_bytes(device_index, m, n, k, tile):
    """Workspace bytes of mica_w8a8_gemm_ex for this call (its device must be current),
    remembered per (device, shape, tile); the memo is cleared when it reaches _WS_CACHE_MAX."""
    key = (device_index, m, n, k, tile)
    need = _WS_BYTES.get(key)
    if need is None:
        if len(_WS_BYTES) >= _WS_CACHE_MAX:
            _WS_BYTES.clear()
        need = _WS_BYTES[key] = int(N.lib().mica_w8a8_gemm_workspace_bytes(m, n, k, *_tile_args(tile)))
    return need


def _gemm(qx, sx, qw, sw, bias, out, out_code, tile):
    """One mica_w8a8_gemm_ex call; the stream-K workspace, when the plan uses one, comes from
    torch's allocator on the current stream (reserved until the kernel is done with it)."""
    m, k = qx.shape
    n = qw.shape[0]
    args = _tile_args(tile)
    with _on(qx):
        need = _workspace_bytes(qx.device.index, m, n, k, tile)
        ws = torch.empty((need,), dtype=torch.uint8, device=qx.device) if need else None
        N.call('mica_w8a8_gemm_ex', qx.data_ptr(), qx.stride(0), qw.data_ptr(), qw.stride(0), sx.data_ptr(),
               sw.data_ptr(), _ptr(bias), out.data_ptr(), out_code, out.stride(0), m, n, k, *args,
               _ptr(ws), need, _stream(qx))


@w8a8_gemm.register_fake
def _(qx, sx, qw, sw, bias, out_dtype, tile):
    return qx.new_empty((qx.shape[0], qw.shape[0]), dtype=OUT_DTYPES[out_dtype])


_OUT_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


@torch.library.custom_op('mica::w8a8_gemm_into', mutates_args=('out',))
def w8a8_gemm_into(qx: torch.Tensor, sx: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor,
                   bias: Optional[torch.Tensor], out: torch.Tensor, tile: int) -> None:
    """As w8a8_gemm, writing into `out` [M, N] (unit column stride, any row stride): e.g. the
    q, k and v slices of one qkv buffer when the three projections quantise their input
    differently."""
    _gemm(qx, sx, qw, sw, bias, out, _OUT_CODE[out.dtype], tile)


@w8a8_gemm_into.register_fake
def _(qx, sx, qw, sw, bias, out, tile):
    return None


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::gemm_swiglu_quant', mutates_args=())
def gemm_swiglu_quant(qx: torch.Tensor, sx: torch.Tensor, qw_gu: torch.Tensor, sw_gu: torch.Tensor,
                      bias: Optional[torch.Tensor], inv_h: Optional[torch.Tensor], round_mode: int
                      ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    m, k = qx.shape
    i = qw_gu.shape[0] // 2
    dev = qx.device
    h = torch.empty((m, i), dtype=torch.bfloat16, device=dev)
    q = torch.empty((m, i), dtype=torch.int8, device=dev)
    s = torch.empty((m,), dtype=torch.float32, device=dev)
    ws_bytes = N.lib().mica_swiglu_workspace_bytes(m)
    ws = torch.empty((max(ws_bytes, 16),), dtype=torch.uint8, device=dev)
    with _on(qx):
        N.call('mica_w8a8_gemm_swiglu_quant', qx.data_ptr(), qx.stride(0), qw_gu.data_ptr(), qw_gu.stride(0),
               sx.data_ptr(), sw_gu.data_ptr(), _ptr(bias), _ptr(inv_h), h.data_ptr(), h.stride(0), q.data_ptr(),
               q.stride(0),
               s.data_ptr(), m, i, k, round_mode, ws.data_ptr(), ws.numel(), _stream(qx))
    return h, q, s


@gemm_swiglu_quant.register_fake
def _(qx, sx, qw_gu, sw_gu, bias, inv_h, round_mode):
    m, i = qx.shape[0], qw_gu.shape[0] // 2
    return (qx.new_empty((m, i), dtype=torch.bfloat16), qx.new_empty((m, i), dtype=torch.int8),
            qx.new_empty((m,), dtype=torch.float32))


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::swiglu_quant', mutates_args=())
def swiglu_quant(g: torch.Tensor, u: torch.Tensor, inv: Optional[torch.Tensor], round_mode: int, want_h: bool,
                 want_q: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    m, i = g.shape
    dev = g.device
    h = torch.empty((m, i) if want_h else (0,), dtype=g.dtype, device=dev)
    q = torch.empty((m, i) if want_q else (0,), dtype=torch.int8, device=dev)
    s = torch.empty((m,) if want_q else (0,), dtype=torch.float32, device=dev)
    with _on(g):
        N.call('mica_swiglu_quant', g.data_ptr(), g.stride(0), u.data_ptr(), u.stride(0), DTYPE_CODE[g.dtype],
               _ptr(inv), h.data_ptr() if want_h else None, i if want_h else 0, q.data_ptr() if want_q else None,
               i if want_q else 0, s.data_ptr() if want_q else None, m, i, round_mode, _stream(g))
    return h, q, s


@swiglu_quant.register_fake
def _(g, u, inv, round_mode, want_h, want_q):
    m, i = g.shape
    return (g.new_empty((m, i) if want_h else (0,)), g.new_empty((m, i) if want_q else (0,), dtype=torch.int8),
            g.new_empty((m,) if want_q else (0,), dtype=torch.float32))


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::option_logits', mutates_args=())
def option_logits(h: torch.Tensor, rows: torch.Tensor, gamma: Optional[torch.Tensor], lo: Optional[torch.Tensor],
                  hi: Optional[torch.Tensor], eps: float, style: int) -> tuple[torch.Tensor, torch.Tensor]:
    b, d = h.shape
    r = rows.shape[0]
    logits = torch.empty((b, r), dtype=torch.float32, device=h.device)
    probs = torch.empty((b, r), dtype=torch.float32, device=h.device)
    with _on(h):
        N.call('mica_option_logits', h.data_ptr(), DTYPE_CODE[h.dtype], h.stride(0), _ptr(gamma), style, eps,
               rows.data_ptr(), r, d, _ptr(lo), _ptr(hi), logits.data_ptr(), probs.data_ptr(), b, _stream(h))
    return logits, probs


@option_logits.register_fake
def _(h, rows, gamma, lo, hi, eps, style):
    b, r = h.shape[0], rows.shape[0]
    return h.new_empty((b, r), dtype=torch.float32), h.new_empty((b, r), dtype=torch.float32)


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::qk_norm_rope', mutates_args=('qkv',))
def qk_norm_rope(qkv: torch.Tensor, q_w: Optional[torch.Tensor], k_w: Optional[torch.Tensor], cos: torch.Tensor,
                 sin: torch.Tensor, pos: Optional[torch.Tensor], pos0: int, heads: int, kv_heads: int,
                 eps: float) -> None:
    d = cos.shape[1]
    with _on(qkv):
        N.call('mica_qk_norm_rope', qkv.data_ptr(), qkv.stride(0), _ptr(q_w), _ptr(k_w), cos.data_ptr(),
               sin.data_ptr(), _ptr(pos), pos0, qkv.shape[0], heads, kv_heads, d, eps, _stream(qkv))


@qk_norm_rope.register_fake
def _(qkv, q_w, k_w, cos, sin, pos, pos0, heads, kv_heads, eps):
    return None


# ---------------------------------------------------------------------------------------
@torch.library.custom_op('mica::attention_prefill', mutates_args=())
def attention_prefill(qkv: torch.Tensor, batch: int, length: int, heads: int, kv_heads: int,
                      scale: float) -> torch.Tensor:
    """Causal GQA attention of a [batch, length] prefill on the QKV projection output (D = 128)."""
    d = qkv.shape[1] // (heads + 2 * kv_heads)
    out = torch.empty((qkv.shape[0], heads * d), dtype=torch.bfloat16, device=qkv.device)
    with _on(qkv):
        N.call('mica_attention_prefill', qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), batch, length,
               heads, kv_heads, d, scale, _stream(qkv))
    return out


@attention_prefill.register_fake
def _(qkv, batch, length, heads, kv_heads, scale):
    d = qkv.shape[1] // (heads + 2 * kv_heads)
    return qkv.new_empty((qkv.shape[0], heads * d))
