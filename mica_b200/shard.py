"""Spreading independent scoring requests over GPUs: one process per GPU, no data-path collective.

The reference serves one worker per GPU and lets each score whole requests (weights are
replicated, requests share nothing). Here every rank computes the same deterministic plan from
the request lengths, scores its share, and the host side joins the results:

    mine = lpt_shard(lengths, world, rank)         # the same split on every rank
    batches = plan_batches([lengths[i] for i in mine], batch_tokens)
    ...score...
    results = gather_to_rank0({i: result_i for i in mine}, world)     # rank 0: all, ordered
    t = max_over_ranks([elapsed_ms], device)                          # the box's time

Only the timing reduction and the final gather cross processes (torch.distributed, NCCL on GPUs
or gloo on CPU); the kernels themselves are single-GPU.
"""
from __future__ import annotations


def request_cost(length: int) -> float:
    """Relative prefill cost of one request: linears ~ L, causal attention ~ L^2 (the 4B
    model's two terms cross near L = 8192)."""
    return float(length) + float(length) * float(length) / 8192.0


def lpt_shard(lengths, world: int, rank: int) -> list:
    """Greedy longest-processing-time assignment: requests in falling cost order, each to the
    least-loaded rank (ties to the lowest rank). Deterministic, so every rank derives the same
    plan without communicating. Returns this rank's request indices, ascending."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} of world {world}')
    cost = [request_cost(int(L)) for L in lengths]
    order = sorted(range(len(cost)), key=lambda i: (-cost[i], i))
    load = [0.0] * world
    mine = []
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        load[r] += cost[i]
        if r == rank:
            mine.append(i)
    return sorted(mine)


# Fixed cost of one more batch (36 layers of launches, ramp-ups and tails), in tokens of work.
# Fitted on B200 from two plans of the 256-request set: 34 batches with 6.0 % padding ran at
# 178.6 K tokens/s and 52 batches with 2.1 % padding at 180.9 K, which puts one batch at ~625 tokens.
BATCH_COST_TOKENS = 640


def plan_batches(lengths, batch_tokens: int, bucket: int = 64, batch_cost: int = BATCH_COST_TOKENS) -> list:
    """Groups request indices (into `lengths`) into padded [B, L] batches: contiguous runs of
    the length-sorted requests, L = the longest rounded up to `bucket`, B x L <= batch_tokens
    (a longer request goes alone). Among all such partitions it returns one that minimises the
    rows computed (sum of B x L, padding included) plus `batch_cost` per batch: an exact
    dynamic program over the sorted order, O(n^2) for n requests."""
    order = sorted(range(len(lengths)), key=lambda i: (lengths[i], i))
    n = len(order)
    pad = [-(-int(lengths[i]) // bucket) * bucket for i in order]
    inf = float('inf')
    best = [0.0] + [inf] * n
    cut = [0] * (n + 1)
    for j in range(1, n + 1):
        L = pad[j - 1]                   # the run [i, j) is padded to its longest, the last
        for i in range(j - 1, -1, -1):
            if j - i > 1 and (j - i) * L > batch_tokens:
                break
            c = best[i] + (j - i) * L + batch_cost
            if c < best[j]:
                best[j], cut[j] = c, i
    out, j = [], n
    while j > 0:
        out.append([order[k] for k in range(cut[j], j)])
        j = cut[j]
    return out[::-1]


def max_over_ranks(values, device='cpu'):
    """Element-wise maximum of `values` over all ranks (every rank gets it): the device time of
    a multi-GPU step is the slowest rank's. Works on one process without a process group."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.cpu().tolist()


def per_rank(values, device='cpu') -> list:
    """Every rank's `values` (a list of floats of the same length on each rank), indexed by
    rank, on every rank: for reports of per-rank busy time, clocks and link rates."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
        return [t.cpu().tolist()]
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.cpu().tolist() for o in out]


def gather_to_rank0(local: dict, world: int):
    """Joins per-rank {request index: result} maps: rank 0 returns the union ordered by request
    index, other ranks None. Raises if two ranks report the same request."""
    import torch.distributed as dist
    if world == 1 or not (dist.is_available() and dist.is_initialized()):
        return [local[i] for i in sorted(local)]
    parts = [None] * world if dist.get_rank() == 0 else None
    dist.gather_object(local, parts, dst=0)
    if dist.get_rank() != 0:
        return None
    merged = {}
    for part in parts:
        dup = set(merged) & set(part)
        if dup:
            raise ValueError(f'requests scored twice: {sorted(dup)[:4]}')
        merged.update(part)
    return [merged[i] for i in sorted(merged)]
