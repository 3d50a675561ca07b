"""GEMM tile table: the `--kernel-tune pinned|full` mechanism for the W8A8 GEMM.

The reference pins one Triton specialisation per (N, K, bias, dtype, M%16, M-class) in
v0.5/serving/kernel_src/specs/sm100.json, picked at launch by the M-class table
GEMM_CLASSES (v0.5/serving/lib/int8_kernels.py:356, :381-385); its FLA autotune caches are
pinned or re-tuned on the device and persisted in --state-dir (lib/kernel_state.py:111-256,
lib/release_runtime.py:1260-1333).

Here a key is (N, K, M-class) and the value the GEMM's output tile, coded
block_m * 1000 + block_n: 128064 / 128128 / 128256 for one CTA per tile, 256128 / 256256
for a CTA pair sharing each MMA (0 = let the library choose). `pinned` ships with the package
(tiles_sm100a.json); `full` sweeps block_n on the device for the shapes in use and writes
the winners to <state_dir>/tiles_sm100a.json, which later runs load first.
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
# tile = splits * 10**6 + block_m * 1000 + block_n: 128-row tiles split K across a cluster when
# few tiles would leave SMs idle (the library's choice), or never (the 1xxxxxx codes); 256-row
# tiles run on CTA pairs.
CHOICES = (128064, 128128, 128256, 256128, 256256, 1128064, 1128128, 1128256)

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
    return {k: int(v) for k, v in entries.items() if int(v) in (0,) + CHOICES}


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


def tile(n: int, k: int, m: int) -> int:
    return table().get(key(n, k, m), 0)


def tune(shapes, device='cuda', reps: int = 20, state_dir=None) -> dict:
    """Sweeps the tile choices for each (N, K, M) on the device; returns {key: best} and,
    with a state dir, persists it there. Times with CUDA events on the current stream."""
    import torch

    from . import ops

    out = {}
    dev = torch.device(device)
    for n, k, m in shapes:
        g = torch.Generator(device=dev).manual_seed(n * 7 + k * 13 + m)
        qx = torch.randint(-127, 128, (m, k), generator=g, device=dev, dtype=torch.int8)
        qw = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
        sx = torch.rand(m, generator=g, device=dev) * 1e-2 + 1e-3
        sw = torch.rand(n, generator=g, device=dev) * 1e-2 + 1e-3
        best, best_t = 0, float('inf')
        for tile_code in CHOICES:
            # time `reps` back-to-back launches replayed from a CUDA graph: device time only,
            # no per-launch Python overhead (which would swamp small shapes)
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(3):
                    torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, tile_code)
            torch.cuda.current_stream(dev).wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    torch.ops.mica.w8a8_gemm(qx, sx, qw, sw, None, 0, tile_code)
            graph.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            b.synchronize()
            t = a.elapsed_time(b) / reps
            del graph
            if t < best_t:
                best, best_t = tile_code, t
        out[key(n, k, m)] = best
    if state_dir:
        p = Path(state_dir)
        p.mkdir(parents=True, exist_ok=True)
        old = _load(p / STATE_NAME)
        old.update(out)
        (p / STATE_NAME).write_text(json.dumps({'format': 'mica-tiles/1', 'entries': old}, indent=1, sort_keys=True))
        set_state_dir(p)
    del ops
    return out


MODEL_SHAPES = ((6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728), (2048, 2560), (4096, 2560),
                # the Qwen3.5-4B hybrid's shapes (GDN a/b 32, k/v 1024, qkv 8192, FFN 9216)
                (32, 2560), (1024, 2560), (8192, 2560), (9216, 2560), (2560, 9216))
CLASS_M = (64, 256, 1024, 8192)     # one M per class s / m / n / l


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
