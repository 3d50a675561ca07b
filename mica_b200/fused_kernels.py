"""Drop-in for the reference's fused_kernels module (v0.5/serving/lib/fused_kernels.py): the
RMSNorm and SwiGLU calls the serving runtime installs on the model (lib/fork.py:179-204
install_norms / rms_norm_fused, lib/fast_runtime.py:126-147 install_swiglu / _fused_mlp).
Same names, arguments and returns:

  rms_norm(x, weight, eps, residual=None) -> y, or (y, x + residual)      (:50-83)
      y = cast(x * rsqrt(mean(x^2) + eps) * (1 + weight)), any leading dims; with a
      residual the sum is rounded to x's dtype first and returned as the second value.
  swi_glu(gate, up) -> cast(cast(silu(gate)) * up)                          (:85-96)

Both run this library's kernels: mica_rmsnorm_quant with the quantiser off, and
mica_swiglu_quant writing only h. Errors follow the reference: a non-unit feature stride
raises ValueError (rms_norm), non-contiguous projections raise ValueError (swi_glu). What the
kernels cannot serve (a CPU tensor, a dtype other than bf16/fp16, a width that is not a
multiple of 8, a weight of another dtype) raises RuntimeError, which the reference's own
caller catches before it uses its torch form (fork.rms_norm_fused). There is no CPU branch
here: the reference's CPU branch is its fallback, and the oracle restates it for the tests.
"""
from __future__ import annotations

import torch

from . import _native as N
from . import int8_kernels as K
from . import ops  # noqa: F401  (registers torch.ops.mica.*)

_DTYPES = (torch.bfloat16, torch.float16)


def _served(name, *ts):
    for t in ts:
        if t is None:
            continue
        if t.device.type != 'cuda':
            raise RuntimeError(f'fused_kernels.{name}: CUDA tensors only (this library has no CPU path)')
        if t.dtype not in _DTYPES:
            raise RuntimeError(f'fused_kernels.{name}: {t.dtype} is not served (bf16 or fp16)')
    ok, why = K.available(ts[0].device)
    if not ok:
        raise RuntimeError(f'fused_kernels.{name}: {why}')


def _rows(t, d):
    """t as [rows, d] with 16-byte aligned rows (a copy only when the view is not)."""
    flat = t.view(-1, d)
    if flat.data_ptr() % 16 or (flat.stride(0) * flat.element_size()) % 16 or flat.stride(1) != 1:
        flat = flat.clone(memory_format=torch.contiguous_format)
    return flat


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor = None):
    """fused_kernels.rms_norm with the (1 + weight) convention (lib/fused_kernels.py:50-83)."""
    _served('rms_norm', x, weight, residual)
    if x.stride(-1) != 1:
        raise ValueError('fused RMSNorm requires unit feature stride')
    d = x.shape[-1]
    if weight.dtype != x.dtype or weight.numel() != d:
        raise RuntimeError(f'fused_kernels.rms_norm: weight {weight.dtype} [{weight.numel()}] for x {x.dtype} [..., {d}]')
    if d % 8:
        raise RuntimeError(f'fused_kernels.rms_norm: width {d} is not a multiple of 8')
    if residual is not None and residual.shape != x.shape:
        residual = residual.view_as(x)
    if x.numel() == 0:
        y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        return y if residual is None else (y, torch.empty_like(y))
    flat = _rows(x, d)
    res = None if residual is None else _rows(residual, d)
    w = weight.contiguous()
    if w.data_ptr() % 16:
        w = w.clone()
    _, _, y, summed = torch.ops.mica.rmsnorm_quant(flat, res, w, None, float(eps), N.NORM_OFFSET,
                                                   K._round_code(), True, False)
    K._launched()
    y = y.view(x.shape)
    return y if residual is None else (y, summed.view(x.shape))


def swi_glu(gate: torch.Tensor, up: torch.Tensor):
    """fused_kernels.swi_glu (lib/fused_kernels.py:85-96): cast(cast(silu(gate)) * up)."""
    _served('swi_glu', gate, up)
    if not gate.is_contiguous() or not up.is_contiguous():
        raise ValueError('fused gate-up kernel requires dense projections')
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise RuntimeError(f'fused_kernels.swi_glu: gate {gate.dtype} {tuple(gate.shape)} vs up {up.dtype} '
                           f'{tuple(up.shape)}')
    n = gate.numel()
    if n == 0:
        return torch.empty_like(gate)
    d = gate.shape[-1] if gate.dim() and gate.shape[-1] % 8 == 0 else 8
    if n % d:
        raise RuntimeError(f'fused_kernels.swi_glu: {n} elements do not split into rows of 8')
    g, u = _rows(gate.reshape(-1, d), d), _rows(up.reshape(-1, d), d)
    h, _, _ = torch.ops.mica.swiglu_quant(g, u, None, K._round_code(), True, False)
    K._launched()
    return h.view(gate.shape)
