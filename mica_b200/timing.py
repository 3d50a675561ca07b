"""Device timing of short launch sequences, shared by the tile tuner and the benchmark.

graph_time() replays one CUDA graph holding, per repetition, [L2 flush, event, fn(), event]:
the events bracket fn() exactly, so its launches are timed on the device without host
launch overhead, and the flush (a write larger than the 126 MB L2) makes every repetition
start from a cold L2, as a layer's GEMM does when the previous layer's activations have
passed through."""
from __future__ import annotations

FLUSH_BYTES = 256 << 20


def graph_time(dev, fn, reps: int, flush_bytes: int = FLUSH_BYTES, warmup: int = 3) -> float:
    """Mean device time of fn() in microseconds over `reps` flushed repetitions."""
    import torch
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=dev) if flush_bytes else None
    ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
          for _ in range(reps)]
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for a, b in ev:
            if flush is not None:
                flush.fill_(1)
            a.record()
            fn()
            b.record()
    graph.replay()
    graph.replay()
    torch.cuda.synchronize(dev)
    t = sum(a.elapsed_time(b) for a, b in ev) / reps * 1e3
    del graph
    return t
