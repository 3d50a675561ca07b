"""Drop-in for the reference's quantised-module surface, v0.5/serving/lib/int8_runtime.py.

QLinear keeps the reference's buffers and attributes (qweight int8 [N,K], wscale fp32 [N],
inv_smooth fp32 [K] | None, bias fp32 [N] | None, w16, in_features, out_features, out_dtype,
backend, mode; :108-192) so weights converted or loaded for the reference load here
unchanged. forward() runs two kernels -- per-token quantiser and W8A8 GEMM -- through
int8_kernels (:172-192).

Differences, by design:
  * backend 'aot' only. A kernel miss raises KernelMiss (the reference silently falls back
    to torch ops; set FALLBACK['allowed'] = True to get that behaviour, on the GPU).
  * FusedMLP replaces gate_proj / up_proj / act / down_proj with the fused gate_up GEMM
    (SwiGLU + requantisation in its epilogue) and the down GEMM: 2 kernels instead of the
    reference's 2 quantisers + 3 GEMMs + SwiGLU (lib/fast_runtime.py:126-132).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from . import int8_kernels as aot

ALPHA = 0.5
EPS = 1e-08
PRECISION = {'mode': 'int8'}
FALLBACK = {'allowed': False}
GDN = ('in_proj_qkv', 'in_proj_z', 'in_proj_a', 'in_proj_b', 'out_proj')
ATTN = ('q_proj', 'k_proj', 'v_proj', 'o_proj')
MLP = ('gate_proj', 'up_proj', 'down_proj')
GROUPS = {'gdn': GDN, 'attn': ATTN, 'mlp': MLP, 'ffn': MLP, 'all': GDN + ATTN + MLP}


class KernelMiss(RuntimeError):
    """The W8A8 kernels could not serve a call (reason as in int8_kernels.STATS['fallback'])."""


def quant_weight(w: torch.Tensor):
    """Per-output-row int8 weights, the reference's int8_quant.quant_weight (lib/int8_quant.py:54-62).
    The scale divides by a tensor of 127s: torch on CUDA turns a division by a Python scalar
    into a multiply by its rounded reciprocal, which can move a scale by one ulp from the
    reference's (CPU) result; an elementwise tensor division is correctly rounded everywhere."""
    wf = w.float()
    amax = wf.abs().amax(1).clamp_min(EPS)
    s = amax / torch.full_like(amax, 127.0)
    q = torch.round(wf / s[:, None]).clamp(-127, 127).to(torch.int8)
    return q, s


def smooth_factors(act_amax, w, alpha=ALPHA, lo=1e-4, hi=1e4):
    """SmoothQuant factors, the reference's int8_quant.smooth_factors (lib/int8_quant.py:80-86)."""
    a = act_amax.float().to(w.device)
    wmax = w.float().abs().amax(0)
    s = a.clamp_min(EPS).pow(alpha) / wmax.clamp_min(EPS).pow(1.0 - alpha)
    s = torch.where((a > 0) & (wmax > 0), s, torch.ones_like(s))
    return s.clamp(lo, hi)


def _last_miss(before):
    now = aot.STATS['fallback']
    return ', '.join(f'{k}+{v - before.get(k, 0)}' for k, v in now.items() if v != before.get(k, 0)) or 'unknown'


def _torch_fallback(x2, inv, qweight, wscale, bias, out_dtype):
    """The reference's own fallback (int8_quant.quant_act + torch._int_mm + dequant,
    lib/int8_runtime.py:181-192), on the GPU; only reached with FALLBACK['allowed']."""
    xf = x2.float() * inv if inv is not None else x2.float()
    s = xf.abs().amax(-1).clamp_min(EPS) / 127.0
    q = torch.round(xf / s[:, None]).clamp(-127, 127).to(torch.int8)
    m = q.shape[0]
    qp = torch.cat((q, q.new_zeros(32 - m, q.shape[1])), 0) if m <= 16 else q
    y = torch._int_mm(qp, qweight.t())[:m].float() * s[:, None] * wscale[None, :]
    return (y + bias if bias is not None else y).to(out_dtype)


class QLinear(nn.Module):
    def __init__(self, linear, smooth=None, backend='aot', keep_bf16=False):
        super().__init__()
        if backend != 'aot':
            raise ValueError("mica_b200 QLinear serves backend='aot' only (the CPU emulation is the test oracle)")
        w = linear.weight.detach()
        self.register_buffer('w16', w.contiguous() if keep_bf16 else None)
        self.in_features, self.out_features = (w.shape[1], w.shape[0])
        self.out_dtype, self.backend, self.mode = (w.dtype, backend, 'int8')
        wf = w.float()
        if smooth is not None:
            smooth = smooth.float().to(w.device)
            wf = wf * smooth[None, :]
            self.register_buffer('inv_smooth', (1.0 / smooth).contiguous())
        else:
            self.inv_smooth = None
        q, s = quant_weight(wf)
        self.register_buffer('qweight', q.contiguous())
        self.register_buffer('wscale', s.contiguous())
        self.register_buffer('bias', None if linear.bias is None else linear.bias.detach().float().contiguous())

    @classmethod
    def empty(cls, in_features, out_features, out_dtype=torch.bfloat16, backend='aot', smooth=True, bias=False):
        """Shape-only module for file loading (reference :130-144)."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.register_buffer('w16', None)
        self.in_features, self.out_features = (in_features, out_features)
        self.out_dtype, self.backend, self.mode = (out_dtype, backend, 'int8')
        meta = lambda *shape, dtype=torch.float32: torch.empty(*shape, dtype=dtype, device='meta')  # noqa: E731
        if smooth:
            self.register_buffer('inv_smooth', meta(in_features))
        else:
            self.inv_smooth = None
        self.register_buffer('qweight', meta(out_features, in_features, dtype=torch.int8))
        self.register_buffer('wscale', meta(out_features))
        self.register_buffer('bias', meta(out_features) if bias else None)
        return self

    @property
    def weight(self):
        w = self.qweight.float() * self.wscale.reshape(-1, 1)
        return (w * self.inv_smooth[None, :] if self.inv_smooth is not None else w).to(self.out_dtype)

    def _quant(self, x2):
        before = dict(aot.STATS['fallback'])
        r = aot.act_quant(x2.contiguous(), self.inv_smooth)
        if r is None and not FALLBACK['allowed']:
            raise KernelMiss(f'act_quant miss ({_last_miss(before)}) for x {tuple(x2.shape)} {x2.dtype}')
        return r

    def rows_forward(self, x, ranges):
        """One quantisation, several GEMMs over row ranges of the weight (reference :153-170)."""
        if self.w16 is not None and PRECISION['mode'] == 'bf16':
            return None
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        r = self._quant(x2)
        outs = []
        for lo, hi in ranges:
            w, s = (self.qweight[lo:hi], self.wscale[lo:hi])
            b = None if self.bias is None else self.bias[lo:hi]
            y = None
            if r is not None:
                before = dict(aot.STATS['fallback'])
                y = aot.mm_i8(r[0], r[1], w, s, b, self.out_dtype)
                if y is None and not FALLBACK['allowed']:
                    raise KernelMiss(f'mm_i8 miss ({_last_miss(before)}) for rows {lo}:{hi}')
            if y is None:
                y = _torch_fallback(x2, self.inv_smooth, w, s, b, self.out_dtype)
            outs.append(y.reshape(*shape[:-1], hi - lo))
        return outs

    def forward(self, x):
        if self.w16 is not None and PRECISION['mode'] == 'bf16':
            return nn.functional.linear(x, self.w16, None if self.bias is None else self.bias.to(self.w16.dtype))
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.shape[0] == 0:
            return x.new_zeros(*shape[:-1], self.out_features, dtype=self.out_dtype)
        r = self._quant(x2)
        y = None
        if r is not None:
            before = dict(aot.STATS['fallback'])
            y = aot.mm_i8(r[0], r[1], self.qweight, self.wscale, self.bias, self.out_dtype)
            if y is None and not FALLBACK['allowed']:
                raise KernelMiss(f'mm_i8 miss ({_last_miss(before)}) for N {self.out_features} K {self.in_features}')
        if y is None:
            y = _torch_fallback(x2, self.inv_smooth, self.qweight, self.wscale, self.bias, self.out_dtype)
        return y.reshape(*shape[:-1], self.out_features)


def same_smoothing(a, b) -> bool:
    """True when two projections quantise their (shared) input identically."""
    if a is None or b is None:
        return a is None and b is None
    return a.shape == b.shape and bool(torch.equal(a, b))


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = 16) -> torch.Tensor:
    """Fused gate_up row order: `group` gate rows, then the same `group` up rows, repeated
    (what the SwiGLU epilogue of mica_w8a8_gemm_swiglu_quant expects). [I, ...] -> [2I, ...]."""
    i = gate.shape[0]
    if i % group or up.shape != gate.shape:
        raise ValueError(f'gate/up shapes {tuple(gate.shape)} {tuple(up.shape)} not interleavable by {group}')
    g = gate.reshape(i // group, group, *gate.shape[1:])
    u = up.reshape(i // group, group, *up.shape[1:])
    return torch.cat([g, u], dim=1).reshape(2 * i, *gate.shape[1:]).contiguous()


class FusedMLP(nn.Module):
    """SwiGLU MLP (the reference's fast_runtime._fused_mlp, lib/fast_runtime.py:126-132).

    When gate_proj and up_proj share their input quantisation (no smoothing, or the same
    inv_smooth) it runs as two kernels: [gate|up] GEMM + SwiGLU + requantisation, then the
    down GEMM. When their smoothing differs (per-projection smoothing, as the reference's
    convert produces) it runs gate and up as separate QLinear GEMMs, then one SwiGLU +
    requantisation kernel, then the down GEMM. down_proj's smoothing is applied inside the
    requantisation either way.

    Built from a module with gate_proj / up_proj / down_proj Linears (HF Qwen3MLP) or from
    existing QLinears."""

    def __init__(self, mlp, stats=None, prefix='', alpha=ALPHA):
        super().__init__()
        g, u, d = mlp.gate_proj, mlp.up_proj, mlp.down_proj
        get = (lambda name: stats.get(prefix + name)) if stats is not None else (lambda name: None)
        self.split = None
        if isinstance(g, QLinear):
            qg, sg, qu, su, inv = g.qweight, g.wscale, u.qweight, u.wscale, g.inv_smooth
            bg, bu = g.bias, u.bias
            self.down = d if isinstance(d, QLinear) else QLinear(d)
            self.out_dtype = g.out_dtype
            if not same_smoothing(g.inv_smooth, u.inv_smooth):
                self.split = nn.ModuleList([g, u])      # two quantisations of x: no shared operand
        else:
            amax = get('gate_proj')
            smooth = None
            if amax is not None:
                smooth = smooth_factors(amax, torch.cat([g.weight.detach(), u.weight.detach()]), alpha)
            wg, wu = g.weight.detach().float(), u.weight.detach().float()
            if smooth is not None:
                smooth = smooth.float().to(wg.device)
                wg, wu = wg * smooth[None, :], wu * smooth[None, :]
            qg, sg = quant_weight(wg)
            qu, su = quant_weight(wu)
            inv = None if smooth is None else (1.0 / smooth).contiguous()
            bg = None if g.bias is None else g.bias.detach().float()
            bu = None if u.bias is None else u.bias.detach().float()
            self.down = QLinear(d)
            self.out_dtype = g.weight.dtype
        self.inner = qg.shape[0]
        if self.split is not None:
            self.inv_smooth = self.qweight_gu = self.wscale_gu = self.bias_gu = None
            return
        self.register_buffer('inv_smooth', inv)
        self.register_buffer('qweight_gu', interleave_gate_up(qg, qu))
        self.register_buffer('wscale_gu', interleave_gate_up(sg, su))
        self.register_buffer('bias_gu', None if bg is None and bu is None else interleave_gate_up(
            bg if bg is not None else torch.zeros_like(bu), bu if bu is not None else torch.zeros_like(bg)))

    def quantise_input(self, x2):
        before = dict(aot.STATS['fallback'])
        r = aot.act_quant(x2.contiguous(), self.inv_smooth)
        if r is None:
            raise KernelMiss(f'act_quant miss ({_last_miss(before)})')
        return r

    def forward_quantised(self, qx, sx):
        """Shared-quantisation path: [gate|up] + SwiGLU + requant, then down."""
        before = dict(aot.STATS['fallback'])
        r = aot.mm_i8_swiglu_quant(qx, sx, self.qweight_gu, self.wscale_gu, self.bias_gu, self.down.inv_smooth)
        if r is None:
            raise KernelMiss(f'gate_up miss ({_last_miss(before)})')
        return self._down(r[1], r[2], before)

    def _down(self, qh, sh, before):
        y = aot.mm_i8(qh, sh, self.down.qweight, self.down.wscale, self.down.bias, self.out_dtype)
        if y is None:
            raise KernelMiss(f'down_proj miss ({_last_miss(before)})')
        return y

    def forward(self, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.shape[0] == 0:
            return x.new_zeros(*shape[:-1], self.down.out_features, dtype=self.out_dtype)
        if self.split is not None:
            before = dict(aot.STATS['fallback'])
            g, u = (lin(x2) for lin in self.split)
            r = aot.swiglu_quant(g, u, self.down.inv_smooth)
            if r is None:
                raise KernelMiss(f'swiglu miss ({_last_miss(before)})')
            y = self._down(r[1], r[2], before)
        else:
            qx, sx = self.quantise_input(x2)
            y = self.forward_quantised(qx, sx)
        return y.reshape(*shape[:-1], self.down.out_features)


# ---------------------------------------------------------------------------------------
# INT8 weights file (lib/int8_runtime.py:639-726): a safetensors file whose metadata holds
# format = FILE_FORMAT and `ties` (JSON {alias: source}) for tensors stored once; the keys are
# the model's state dict with every converted projection's QLinear buffers (qweight int8
# [N, K], wscale fp32 [N], and inv_smooth fp32 [K] / bias fp32 [N] when present).
FILE = 'model-int8.safetensors'
FILE_FORMAT = 'int8-w8a8/1'


class InvalidModel(ValueError):
    """The reference's ValueError('invalid_model'), with the reason appended."""

    def __init__(self, why):
        super().__init__(f'invalid_model: {why}')


def read_int8_file(path, device='cpu'):
    """Reads an int8-w8a8/1 file (a folder holding FILE, or the file itself).

    Returns (tensors, ties): every stored tensor by key, with each tied alias resolved to its
    source tensor (the same object), and the ties map. Raises InvalidModel on a wrong format
    tag or a tie whose source is missing (lib/int8_runtime.py:679-688)."""
    import json
    from pathlib import Path
    from safetensors import safe_open
    path = Path(path)
    if path.is_dir():
        path = path / FILE
    with safe_open(str(path), framework='pt', device=str(device)) as f:
        meta = f.metadata() or {}
        if meta.get('format') != FILE_FORMAT:
            raise InvalidModel(f"format {meta.get('format')!r}, expected {FILE_FORMAT!r}")
        ties = json.loads(meta.get('ties') or '{}')
        keys = set(f.keys())
        bad = [a for a, src in ties.items() if src not in keys or a in keys]
        if bad:
            raise InvalidModel(f'ties without a stored source: {sorted(bad)[:4]}')
        tensors = {k: f.get_tensor(k) for k in sorted(keys)}
    for alias, src in ties.items():
        tensors[alias] = tensors[src]
    return tensors, ties


def write_int8_file(path, tensors: dict, ties: dict | None = None):
    """Writes tensors (tied aliases left out: pass them in `ties`) as an int8-w8a8/1 file."""
    import json
    from safetensors.torch import save_file
    ties = dict(ties or {})
    stored = {k: v.contiguous() for k, v in tensors.items() if k not in ties}
    save_file(stored, str(path), metadata={'format': FILE_FORMAT, 'ties': json.dumps(ties, sort_keys=True)})


def target_linears(body, layers=None, modules=None):
    """Every projection Linear of `body.layers` (the reference's int8_quant.target_linears,
    lib/int8_quant.py:99-110): a list of (name 'layers.<i>.<path>', parent module, attribute,
    Linear), layer by layer in module order."""
    names = frozenset(GROUPS['all'] if modules is None else modules)
    picked = range(len(body.layers)) if layers is None else layers
    found = []
    for i in picked:
        layer = body.layers[i]
        for path, mod in layer.named_modules():
            owner, _, leaf = path.rpartition('.')
            if leaf in names and isinstance(mod, nn.Linear):
                found.append((f'layers.{i}.{path}', layer.get_submodule(owner) if owner else layer, leaf, mod))
    return found


def _smoothing(stats, name, linear, alpha):
    """SmoothQuant factors of one projection from its activation statistics, or None."""
    amax = None if stats is None else stats.get(name)
    return None if amax is None else smooth_factors(amax, linear.weight.detach(), alpha)


def convert(body, stats, backend='aot', alpha=ALPHA, keep_bf16=False, fuse_mlp=False):
    """Swaps every projection Linear of the decoder body for a QLinear, smoothed where `stats`
    holds that projection's activation maxima (the reference's int8_runtime.convert,
    lib/int8_runtime.py:195-206). With fuse_mlp each `mlp` holding gate/up/down Linears becomes
    one FusedMLP first. Returns (projections replaced, projections smoothed)."""
    replaced = smoothed = 0
    if fuse_mlp:
        for i, layer in enumerate(body.layers):
            mlp = getattr(layer, 'mlp', None)
            if mlp is None or not all(isinstance(getattr(mlp, n, None), nn.Linear) for n in MLP):
                continue
            layer.mlp = FusedMLP(mlp, stats, f'layers.{i}.mlp.', alpha)
            replaced += len(MLP)
            smoothed += int(layer.mlp.inv_smooth is not None)
    for name, parent, attr, linear in target_linears(body):
        smooth = _smoothing(stats, name, linear, alpha)
        parent.register_module(attr, QLinear(linear, smooth, backend, keep_bf16=keep_bf16))
        replaced += 1
        smoothed += int(smooth is not None)
    return replaced, smoothed


# ---------------------------------------------------------------------------------------
# Start-up self-test (the reference's int8_runtime.selftest, lib/int8_runtime.py:288-443):
# before serving, every projection shape runs through this library's act_quant + mm_i8 on
# seeded data, smoothed and unsmoothed, at several row counts; each result must stay within
# SELFTEST_TOL times the error an exact INT8 emulation makes against the bf16 product, and
# every case must launch the library's two kernels. The seed, the rows and the tolerance are
# the reference's; the data recipe and the code are this library's.
SELFTEST_ROWS = (3, 48, 200, 608, 1500)
SELFTEST_TOL = 1.05
SELFTEST_SEED = 20261022


@dataclass(frozen=True)
class SelfTestCase:
    n: int
    k: int
    bias: bool
    smoothed: bool
    m: int


def selftest_plan(shapes, rows=SELFTEST_ROWS):
    """The cases for these (N, K, has_bias) shapes: each shape smoothed and plain, at each row count."""
    return [SelfTestCase(int(n), int(k), bool(b), sm, int(m)) for n, k, b in shapes for sm in (True, False)
            for m in rows]


def _worst_row_error(y, ref):
    """Largest per-row relative L2 error of y against ref."""
    err = (y - ref).norm(dim=-1) / ref.norm(dim=-1).clamp_min(1e-30)
    return float(err.max())


class _ShapeData:
    """Seeded weights, channel ranges and bias of one (N, K, has_bias) shape, on the device:
    weights N(0, 0.05) in bf16; per-channel activation ranges log-normal around 1 with one
    channel in 50 twenty times wider (outlier channels, what smoothing is for)."""

    def __init__(self, n, k, bias, gen, dev):
        self.w = (torch.randn(n, k, generator=gen, device=dev) * 0.05).to(torch.bfloat16)
        spread = torch.exp(0.5 * torch.randn(k, generator=gen, device=dev))
        spread[torch.arange(0, k, 50, device=dev)] *= 20.0
        self.spread = spread
        self.bias = (torch.randn(n, generator=gen, device=dev) * 0.1).float() if bias else None
        self.prepared = {}

    def weights(self, smoothed):
        """(qweight, wscale, inv_smooth or None, dequantised weight) of the projection."""
        if smoothed not in self.prepared:
            wf = self.w.float()
            inv = None
            if smoothed:
                f = smooth_factors(self.spread, self.w, ALPHA)
                wf = wf * f[None, :]
                inv = (1.0 / f).contiguous()
            qw, sw = quant_weight(wf)
            w_eff = qw.float() * sw[:, None]
            self.prepared[smoothed] = (qw, sw, inv, w_eff if inv is None else w_eff * inv[None, :])
        return self.prepared[smoothed]


def _emulated_linear(x, inv, qw, sw, bias):
    """An exact W8A8 linear: per-token codes (round half even), exact integer products
    (float64 on the device), fp32 dequant, cast to bf16."""
    xf = x.float() if inv is None else x.float() * inv
    amax = xf.abs().amax(-1).clamp_min(EPS)
    s = amax / torch.full_like(amax, 127.0)
    codes = torch.round(xf / s[:, None]).clamp(-127, 127)
    y = (codes.double() @ qw.double().t()).float() * s[:, None] * sw[None, :]
    return (y if bias is None else y + bias).to(torch.bfloat16).float()


def selftest(shapes, device, rows=SELFTEST_ROWS):
    """Runs selftest_plan(shapes, rows) on `device`; returns the reference's report
    {'ok', 'reason', 'checked', 'worst_ratio', 'launches', 'seconds'}. Never raises."""
    import time

    started = time.perf_counter()
    report = {'ok': False, 'reason': '', 'checked': 0, 'worst_ratio': 0.0}
    try:
        dev = torch.device(device)
        usable, why = aot.available(dev)
        if not usable:
            report['reason'] = why
            return report
        gen = torch.Generator(device=dev).manual_seed(SELFTEST_SEED)
        first_launch = aot.STATS['launch']
        data = {}
        for case in selftest_plan(shapes, rows):
            shape = (case.n, case.k, case.bias)
            if shape not in data:
                data[shape] = _ShapeData(*shape, gen, dev)
            d = data[shape]
            qw, sw, inv, w_eff = d.weights(case.smoothed)
            x = (torch.randn(case.m, case.k, generator=gen, device=dev) * d.spread / 3).to(torch.bfloat16)
            where = 'N %d K %d M %d%s' % (case.n, case.k, case.m, ' smoothed' if case.smoothed else '')
            before = aot.STATS['launch']
            qx = aot.act_quant(x, inv)
            y = None if qx is None else aot.mm_i8(qx[0], qx[1], qw, sw, d.bias, torch.bfloat16)
            if y is None or aot.STATS['launch'] - before != 2:
                report['reason'] = f'{where}: the kernels did not serve the call ({aot.STATS["fallback"]})'
                return report
            y = y.float()
            if not bool(torch.isfinite(y).all()):
                report['reason'] = f'{where}: non-finite output'
                return report
            exact = x.float() @ w_eff.t() + (d.bias if d.bias is not None else 0.0)
            noise = _worst_row_error(_emulated_linear(x, inv, qw, sw, d.bias), exact)
            err = _worst_row_error(y, exact)
            if err > SELFTEST_TOL * noise:
                report['reason'] = f'{where}: error {err:.4g} > {SELFTEST_TOL:.2f} x INT8 noise {noise:.4g}'
                return report
            report['worst_ratio'] = max(report['worst_ratio'], err / max(noise, 1e-30))
            report['checked'] += 1
        torch.cuda.synchronize(dev)
        report.update(ok=True, reason='ok', launches=aot.STATS['launch'] - first_launch,
                      worst_ratio=round(report['worst_ratio'], 5))
    except Exception as exc:  # a start-up check reports; it never takes the server down
        report['reason'] = f'{type(exc).__name__}: {exc}'[:300]
    finally:
        report['seconds'] = round(time.perf_counter() - started, 2)
    return report
