"""Drop-in for the reference's kernel-call surface, v0.5/serving/lib/int8_kernels.py.

Same names, arguments and contract as the reference module:
  * act_quant(x, inv_smooth=None) -> (q int8 [M,K], s fp32 [M]) or None      (:325-353)
  * mm_i8(qx, sx, qw, sw, bias=None, out_dtype=torch.bfloat16) -> y or None  (:359-406)
  * available(device=None) -> (bool, str)                                    (:146-159)
  * preload(device=None) -> int                                              (:217-224)
  * kernel_dir(), PACKED, STATS, ATTN, GEMM_CLASSES, attn_fwd, attn_keys
A request the kernels cannot serve returns None and counts the reason in
STATS['fallback'] (:19-24), so QLinear's own fallback logic is unchanged. Hard errors
(CUDA failures) raise. Unlike the reference, no cubin container is read: the kernels
live in libmica_w8a8.so, built from csrc/ for sm_100a.

Additions used by the fused paths: rmsnorm_quant, mm_i8_swiglu_quant, swiglu_quant / swi_glu,
option_logits.
"""
from __future__ import annotations

import threading
from pathlib import Path

import torch

from . import _native as N
from . import ops  # noqa: F401  (registers torch.ops.mica.*)
from . import tiles

DT = {torch.bfloat16: 'bf16', torch.float16: 'fp16', torch.float32: 'fp32'}
I32 = 2**31
STATS = {'launch': 0, 'fallback': {}}
GEMM_CLASSES = ((128, 's'), (384, 'm'), (1024, 'n'))
PACKED = N.LIB_NAME
ATTN = {'enabled': False}
# Rounding of activation codes: 'half_away' is the reference GPU kernel
# (v0.5/serving/kernel_src/kernels.py:35), 'half_even' its torch path (lib/int8_quant.py:70).
ROUND = {'mode': 'half_away'}
_ROUND_CODE = {'half_away': N.ROUND_HALF_AWAY, 'half_even': N.ROUND_HALF_EVEN}
_LOCK = threading.Lock()


def _miss(reason):
    STATS['fallback'][reason] = STATS['fallback'].get(reason, 0) + 1
    return None


def _launched(n=1):
    STATS['launch'] += n


def kernel_dir():
    return Path(N.lib_path()).parent


def _dev(device):
    dev = torch.device(device) if device is not None else torch.device('cuda')
    if dev.type == 'cuda' and dev.index is None:
        dev = torch.device('cuda', torch.cuda.current_device())
    return dev


_CAPS = {}


def caps(device=None):
    dev = _dev(device)
    if dev.index not in _CAPS:
        c = N.Caps()
        N.call('mica_query', dev.index, c)
        _CAPS[dev.index] = c
    return _CAPS[dev.index]


def available(device=None):
    if not torch.cuda.is_available():
        return (False, 'CUDA not available')
    dev = _dev(device)
    if dev.type != 'cuda':
        return (False, f'{dev} is not CUDA')
    try:
        c = caps(dev)
    except (OSError, N.NativeError) as exc:
        return (False, f'library: {exc!r}'[:200])
    if not c.supported:
        return (False, f'capability sm_{c.cc_major}{c.cc_minor} is not sm_100 ({N.lib_path()})')
    return (True, f'sm_100a from {N.lib_path()}')


def preload(device=None):
    dev = _dev(device)
    ok, _ = available(dev)
    if not ok:
        return 0
    n = N.ctypes.c_int(0)
    with torch.cuda.device(dev):
        N.call('mica_preload', n)
    return n.value


def gemm_tile(n, k, m, device=None):
    """The tuning table's tile code for this GEMM on `device` (tiles.tile with its SM count)."""
    return tiles.tile(n, k, m, caps(device).sm_count)


def _round_code():
    return _ROUND_CODE[ROUND['mode']]


def _aligned(*ts):
    return all(t.data_ptr() % 16 == 0 for t in ts if t is not None)


def _supported(dev):
    ok, _ = available(dev)
    return ok


def act_quant(x, inv_smooth=None):
    """Per-token int8 quantisation; mirrors v0.5/serving/lib/int8_kernels.py:325-353."""
    if x.dim() != 2 or x.device.type != 'cuda' or x.dtype not in DT:
        return _miss('act_input')
    m, k = x.shape
    if x.stride(1) != 1 or x.stride(0) != k:
        return _miss('act_contiguous')
    if not _supported(x.device):
        return _miss('no_container')
    if inv_smooth is not None and (
        inv_smooth.dtype != torch.float32
        or not inv_smooth.is_contiguous()
        or inv_smooth.numel() != k
        or inv_smooth.device != x.device
    ):
        return _miss('act_inv')
    if m * k >= I32:
        return _miss('i32_range')
    if k % 16 or not _aligned(x, *(() if inv_smooth is None else (inv_smooth,))):
        return _miss('align')
    if m == 0:
        return (x.new_empty((0, k), dtype=torch.int8), x.new_empty((0,), dtype=torch.float32))
    q, s = torch.ops.mica.act_quant(x, inv_smooth, _round_code())
    _launched()
    return (q, s)


def mm_i8(qx, sx, qw, sw, bias=None, out_dtype=torch.bfloat16):
    """W8A8 GEMM with dequant epilogue; mirrors v0.5/serving/lib/int8_kernels.py:359-406."""
    if qx.dim() != 2 or qw.dim() != 2 or qx.dtype != torch.int8 or qw.dtype != torch.int8 or out_dtype not in DT:
        return _miss('mm_input')
    m, k = qx.shape
    n = qw.shape[0]
    if qw.shape[1] != k or qx.stride(1) != 1 or qw.stride(1) != 1 or qx.stride(0) != k or qw.stride(0) != k:
        return _miss('mm_contiguous')
    for t, size in ((sx, m), (sw, n)) + (((bias, n),) if bias is not None else ()):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != size or t.device != qx.device:
            return _miss('mm_scales')
    if qw.device != qx.device or qx.device.type != 'cuda':
        return _miss('mm_device')
    if not _supported(qx.device):
        return _miss('no_container')
    if m * max(k, n) >= I32:
        return _miss('i32_range')
    es = 4 if out_dtype == torch.float32 else 2
    if k % 16 or (n * es) % 16 or not _aligned(qx, qw):
        return _miss('align')
    if m == 0:
        return qx.new_empty((0, n), dtype=out_dtype)
    y = torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, bias, ops.DTYPE_CODE[out_dtype], gemm_tile(n, k, m, qx.device))
    _launched()
    return y


def rmsnorm_quant(x, weight, eps, residual=None, inv_smooth=None, style=N.NORM_OFFSET, want_y=False, want_q=True):
    """Fused (residual add +) RMSNorm (+ per-token quantisation).

    Returns (q, s, y, summed): q/s are empty when want_q is False, y is empty unless want_y,
    summed is the residual-added stream (empty without a residual)."""
    if x.dim() != 2 or x.device.type != 'cuda' or x.dtype not in (torch.bfloat16, torch.float16):
        return _miss('norm_input')
    m, k = x.shape
    if x.stride(1) != 1 or x.stride(0) != k or (residual is not None and not residual.is_contiguous()):
        return _miss('norm_contiguous')
    if weight.dtype != x.dtype or weight.numel() != k or not weight.is_contiguous():
        return _miss('norm_weight')
    if k % 16 or not _aligned(x, weight):
        return _miss('align')
    if not _supported(x.device):
        return _miss('no_container')
    r = torch.ops.mica.rmsnorm_quant(x, residual, weight, inv_smooth, float(eps), int(style), _round_code(),
                                     bool(want_y), bool(want_q))
    _launched()
    return r


def mm_i8_swiglu_quant(qx, sx, qw_gu, sw_gu, bias=None, inv_h=None):
    """gate_up GEMM + SwiGLU + per-token requantisation of the product (one kernel).

    qw_gu/sw_gu hold gate and up rows interleaved in groups of 16 (int8_runtime.interleave_gate_up).
    inv_h [I] is down_proj's inv_smooth (the requantisation quantises h * inv_h), or None.
    Returns (h bf16 [M, I], q int8 [M, I], s fp32 [M])."""
    if qx.dim() != 2 or qx.dtype != torch.int8 or qw_gu.dtype != torch.int8 or qw_gu.shape[0] % 32:
        return _miss('swiglu_input')
    m, k = qx.shape
    if qw_gu.shape[1] != k or not qx.is_contiguous() or not qw_gu.is_contiguous():
        return _miss('swiglu_contiguous')
    if inv_h is not None and (inv_h.dtype != torch.float32 or inv_h.numel() != qw_gu.shape[0] // 2):
        return _miss('act_inv')
    if k % 16 or not _aligned(qx, qw_gu, inv_h):
        return _miss('align')
    if not _supported(qx.device):
        return _miss('no_container')
    r = torch.ops.mica.gemm_swiglu_quant(qx, sx, qw_gu, sw_gu, bias, inv_h, _round_code())
    _launched()
    return r


def swiglu_quant(gate, up, inv=None, want_h=False, want_q=True):
    """h = bf16(bf16(silu(gate)) * up) (fused_kernels.swi_glu, lib/fused_kernels.py:85-96), then
    down_proj's per-token quantisation of h * inv (one kernel). For MLPs whose gate and up
    projections quantise their input differently. Returns (h, q, s); h is empty unless
    want_h, q/s are empty unless want_q."""
    if gate.dim() != 2 or gate.shape != up.shape or gate.dtype != up.dtype or gate.dtype not in (
            torch.bfloat16, torch.float16) or gate.device.type != 'cuda':
        return _miss('swiglu_input')
    m, i = gate.shape
    if gate.stride(1) != 1 or up.stride(1) != 1:
        return _miss('swiglu_contiguous')
    if inv is not None and (inv.dtype != torch.float32 or inv.numel() != i):
        return _miss('act_inv')
    if i % 8 or (gate.stride(0) * 2) % 16 or (up.stride(0) * 2) % 16 or not _aligned(gate, up, inv):
        return _miss('align')
    if not _supported(gate.device):
        return _miss('no_container')
    r = torch.ops.mica.swiglu_quant(gate, up, inv, _round_code(), bool(want_h), bool(want_q))
    _launched()
    return r


def swi_glu(gate, up):
    """fused_kernels.swi_glu drop-in (lib/fused_kernels.py:85-96): bf16(bf16(silu(gate)) * up)."""
    r = swiglu_quant(gate, up, None, want_h=True, want_q=False)
    return None if r is None else r[0]


def option_logits(h, rows, gamma=None, lo=None, hi=None, eps=1e-6, style=N.NORM_WEIGHT):
    """Gathered lm_head GEMV for the last position + per-request softmax slice.

    h [B, D] (bf16/fp16/fp32), rows fp32 [R, D]; lo/hi int32 [B] or None. Returns (logits, probs)."""
    if h.dim() != 2 or rows.dim() != 2 or rows.dtype != torch.float32 or h.shape[1] != rows.shape[1]:
        return _miss('readout_input')
    if not h.is_contiguous() or not rows.is_contiguous():
        return _miss('readout_contiguous')
    if not _supported(h.device):
        return _miss('no_container')
    r = torch.ops.mica.option_logits(h, rows, gamma, lo, hi, float(eps), int(style))
    _launched(2)
    return r


def attn_key(hq, rep, d, scale, small):
    return 'attn|bf16|hd%d|hq%d|r%d|s%.8g|%s' % (d, hq, rep, scale, 'm16' if small else 'm64')


def attn_keys(device=None):
    """No attention kernel ships here: attention stays on torch SDPA (flash/cuDNN)."""
    return []


def attn_fwd(q, k, v, scale):
    """Reference :430-481. Out of this library's scope; the miss makes callers use SDPA."""
    return _miss('no_cubin')
