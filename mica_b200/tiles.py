"""GEMM tile table: the `--kernel-tune pinned|full` mechanism for the W8A8 GEMM.

The reference pins one Triton specialisation per (N, K, bias, dtype, M%16, M-class) in
v0.5/serving/kernel_src/specs/sm100.json, picked at launch by the M-class table
GEMM_CLASSES (v0.5/serving/lib/int8_kernels.py:356, :381-385); its FLA autotune caches are
pinned or re-tuned on the device and persisted in --state-dir (lib/kernel_state.py:111-256,
lib/release_runtime.py:1260-1333).

Here a key is (N, K, M-class) and the value a tile code for the GEMM:
    splits * 10**6 + block_m * 1000 + block_n
  0                       the library's own choice for the call's exact M (its 128 x 320 tiles
                          for grids just past one wave, stream-K where a second wave would be
                          long and mostly empty, a cluster K split for grids that leave SMs idle);
  128064 / 128128 / 128256 / 128320
                          one CTA per 128-row tile (the library may still split K or run
                          stream-K for 64/128/256; 320 runs only where the grid fits one wave);
  256128 / 256256         CTA pairs sharing each MMA (256-row tiles);
  1128xxx                 one CTA per tile, never split;
  S128xxx, S = 2..8       K split across a cluster of S CTAs (forced);
  9128128 / 9128256       stream-K (forced).
`pinned` ships with the package (tiles_sm100a.json); `full` times every candidate on the
device for the shapes in use, each launch from a cold L2 inside a CUDA graph (as the bench
times them), and writes the winners to <state_dir>/tiles_sm100a.json, which later runs load
on top of the pinned table.
"""
from __future__ import annotations

import json
import os
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
PINNED = HERE / 'tiles_sm100a.json'
STATE_NAME = 'tiles_sm100a.json'
CLASSES = ((128, 's'), (384, 'm'), (1024, 'n'))
CHOICES = ((0, 128064, 128128, 128256, 128320, 256128, 256256, 1128064, 1128128, 1128256)
           + tuple(s * 1000000 + 128000 + bn for s in range(2, 9) for bn in (128, 256))
           + (9128128, 9128256))


def valid(code: int) -> bool:
    """A tile code the library accepts (it may still decline it for a shape: a 320-wide grid
    past one wave, a split that leaves a rank without k-blocks)."""
    if code == 0:
        return True
    if code < 0:
        return False
    s, bm, bn = code // 1000000, (code // 1000) % 1000, code % 1000
    if bm == 256:
        return s == 0 and bn in (128, 256)
    if bm != 128 or bn not in (64, 128, 256, 320):
        return False
    if bn == 320:
        return s in (0, 1)
    if s == 9:
        return bn in (128, 256)
    return s <= 8


def effective(code: int, n: int, m: int, sms: int) -> int:
    """The code a call of this M runs: a 128 x 320 entry applies only where its grid fits one
    wave (one CTA per tile); elsewhere the call takes the library's own choice (0)."""
    if code % 1000 == 320 and ((m + 127) // 128) * ((n + 319) // 320) > sms:
        return 0
    return code


_TABLE = None
_LOCK = threading.Lock()
_STATE = {'dir': os.environ.get('MICA_STATE_DIR')}


def m_class(m: int) -> str:
    return next((c for hi, c in CLASSES if m <= hi), 'l')


def key(n: int, k: int, m: int) -> str:
    return f'mm|N{n}|K{k}|c{m_class(m)}'


def _load(path: Path) -> dict:
    try:
        data = json.loads(path.read_text(encoding='utf-8'))
    except (OSError, ValueError):
        return {}
    entries = data.get('entries', {}) if isinstance(data, dict) else {}
    out = {}
    for k, v in entries.items():
        try:
            code = int(v)
        except (TypeError, ValueError):
            continue
        if valid(code):
            out[k] = code
    return out


def table() -> dict:
    global _TABLE
    if _TABLE is None:
        with _LOCK:
            if _TABLE is None:
                t = _load(PINNED)
                if _STATE['dir']:
                    t.update(_load(Path(_STATE['dir']) / STATE_NAME))
                _TABLE = t
    return _TABLE


def set_state_dir(path) -> None:
    """Use <path>/tiles_sm100a.json (tuned entries) on top of the pinned table."""
    global _TABLE
    with _LOCK:
        _STATE['dir'] = str(path) if path else None
        _TABLE = None


def tile(n: int, k: int, m: int, sms: int = None) -> int:
    """Tile code for a GEMM of N x K weights over M rows (sms: the device's SM count, which
    decides whether a 320-wide entry applies to this M)."""
    code = table().get(key(n, k, m), 0)
    return code if sms is None else effective(code, n, m, sms)


def tune(shapes, device='cuda', reps: int = 10, state_dir=None, choices=CHOICES) -> dict:
    """Times every tile code in `choices` for each (N, K, M) on the device and returns
    {key: best}; with a state dir the winners are merged into <state_dir>/tiles_sm100a.json
    and used from then on. Each candidate runs `reps` times inside one CUDA graph, every
    launch after an L2 flush and bracketed by events (timing.graph_time). Shapes that share a
    key (several M of one M-class) are weighed together: the winner minimises the sum over
    those M of its time relative to the fastest code at that M. A code the library declines
    for one of them (MICA_ERR_UNSUPPORTED, e.g. a K split that leaves a rank empty) is out;
    a 320-wide code is timed as what it runs at each M (effective())."""
    import torch

    from . import _native as N
    from . import ops  # noqa: F401  (registers torch.ops.mica.*)
    from .timing import graph_time

    dev = torch.device(device)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    groups = {}
    for n, k, m in shapes:
        groups.setdefault(key(n, k, m), []).append((n, k, m))
    out = {}
    for kk, items in groups.items():
        rel = {code: 0.0 for code in choices}
        for n, k, m in items:
            g = torch.Generator(device=dev).manual_seed(n * 7 + k * 13 + m)
            qx = torch.randint(-127, 128, (m, k), generator=g, device=dev, dtype=torch.int8)
            qw = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
            sx = torch.rand(m, generator=g, device=dev) * 1e-2 + 1e-3
            sw = torch.rand(n, generator=g, device=dev) * 1e-2 + 1e-3
            times = {}
            for code in choices:
                eff = effective(code, n, m, sms)
                if eff not in times:
                    try:
                        torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, eff)
                    except N.NativeError as exc:
                        if exc.rc != 8:            # anything but MICA_ERR_UNSUPPORTED is a real failure
                            raise
                        times[eff] = None
                    else:
                        times[eff] = graph_time(
                            dev, lambda c=eff: torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, c), reps)
            fastest = min(t for t in times.values() if t is not None)
            for code in choices:
                t = times[effective(code, n, m, sms)]
                rel[code] = None if (t is None or rel[code] is None) else rel[code] + t / fastest
            del qx, qw
        out[kk] = min((code for code in choices if rel[code] is not None), key=lambda c: (rel[c], c != 0))
    if state_dir:
        p = Path(state_dir)
        p.mkdir(parents=True, exist_ok=True)
        old = _load(p / STATE_NAME)
        old.update(out)
        (p / STATE_NAME).write_text(json.dumps({'format': 'mica-tiles/1', 'entries': old}, indent=1, sort_keys=True))
        set_state_dir(p)
    return out


MODEL_SHAPES = ((6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728), (2048, 2560), (4096, 2560),
                # the Qwen3.5-4B hybrid's shapes (GDN a/b 32, k/v 1024, qkv 8192, FFN 9216)
                (32, 2560), (1024, 2560), (8192, 2560), (9216, 2560), (2560, 9216))
CLASS_M = (64, 256, 1024, 2048, 8192)     # one M per class s / m / n, two for l (a wave or two, many waves)


def main(argv=None):
    """python -m mica_b200.tiles --tune --state-dir DIR  (the `--kernel-tune full` step):
    sweeps the tile choices on this GPU for the 4B model's projections and M-classes and
    writes DIR/tiles_sm100a.json."""
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument('--tune', action='store_true')
    ap.add_argument('--state-dir', required=True)
    ap.add_argument('--reps', type=int, default=10)
    a = ap.parse_args(argv)
    if a.tune:
        shapes = [(n, k, m) for n, k in MODEL_SHAPES for m in CLASS_M]
        res = tune(shapes, reps=a.reps, state_dir=a.state_dir)
        print(json.dumps(res, indent=1, sort_keys=True))


if __name__ == '__main__':
    main()
