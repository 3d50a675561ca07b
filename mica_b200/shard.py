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

import functools


def request_cost(length: int) -> float:
    """Relative prefill cost of one request: linears ~ L, causal attention ~ L^2 (the 4B
    model's two terms cross near L = ATT_CROSS)."""
    return float(length) + float(length) * float(length) / ATT_CROSS


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


# Cost of one padded [B, L] batch of the 4B model in "tokens of linear work":
#   B * L                      the projections and MLP (per token),
#   B * L * L / ATT_CROSS      causal attention (per token, growing with L),
#   BATCH_COST_TOKENS          a fixed cost per batch (36 layers of small-M GEMM floors, launches).
# Fitted on B200 (least squares on relative error) to 15 batch shapes from [1, 256] to [1, 32768]
# and [64, 256], timed through the captured batch graphs config 4 replays: 3.63 us per token,
# 0.218 ns per token per key, 4.37 ms per batch; every shape within 5 % of the fit.
ATT_CROSS = 16600.0
BATCH_COST_TOKENS = 1200


def batch_cost(B: int, L: int, att_cross: float = ATT_CROSS, fixed: float = BATCH_COST_TOKENS) -> float:
    """Modelled cost of one padded [B, L] batch (see above)."""
    return float(B) * float(L) * (1.0 + float(L) / att_cross) + float(fixed)


def plan_batches(lengths, batch_tokens: int, bucket: int = 64, batch_cost_tokens: float = BATCH_COST_TOKENS,
                 att_cross: float = ATT_CROSS) -> list:
    """Groups request indices (into `lengths`) into padded [B, L] batches: contiguous runs of
    the length-sorted requests, L = the longest rounded up to `bucket`, B x L <= batch_tokens
    (a longer request goes alone). Among all such partitions it returns one of least total
    batch_cost (padding included): an exact dynamic program over the sorted order, O(n^2)."""
    return _plan(lengths, batch_tokens, bucket, batch_cost_tokens, att_cross)[0]


def _plan(lengths, batch_tokens, bucket, fixed, att_cross):
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
            c = best[i] + batch_cost(j - i, L, att_cross, fixed)
            if c < best[j]:
                best[j], cut[j] = c, i
    out, j = [], n
    while j > 0:
        out.append([order[k] for k in range(cut[j], j)])
        j = cut[j]
    return out[::-1], best[n]


def plan_cost(lengths, batch_tokens: int, bucket: int = 64) -> float:
    """Modelled cost of scoring `lengths` as plan_batches would batch them."""
    return _plan_cost_sorted(tuple(sorted(int(x) for x in lengths)), batch_tokens, bucket)


@functools.lru_cache(maxsize=65536)
def _plan_cost_sorted(lengths: tuple, batch_tokens: int, bucket: int) -> float:
    return _plan(list(lengths), batch_tokens, bucket, BATCH_COST_TOKENS, ATT_CROSS)[1] if lengths else 0.0


def balanced_shard(lengths, world: int, rank: int, batch_tokens: int, max_rounds: int = 64) -> list:
    """Shares refined against each rank's batch plan: LPT balances per-request costs, but a
    rank's time is its batches' (padding to each batch's longest, one fixed cost per batch).
    Starting from the better (by that model) of lpt_shard and batch_first_shards, it repeatedly
    moves one request from the rank of largest plan_cost to the
    rank of least, or swaps one pair between them, taking the change that lowers the larger of
    the two the most among the 48 that move nearest half the gap (by request_cost); it stops
    when none lowers it (or after max_rounds). Deterministic,
    so every rank derives the same plan. Returns this rank's request indices, ascending."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} of world {world}')
    return list(_balanced(tuple(int(x) for x in lengths), world, batch_tokens, max_rounds)[rank])


def batch_first_shards(lengths, world: int, batch_tokens: int) -> list:
    """All ranks' shares when the batches are planned over the whole request set (the plan one
    GPU would run) and whole batches are dealt out by LPT on their modelled cost. Splitting a
    length class across ranks costs extra batches, each a fixed cost; this keeps the batch
    count of the single-GPU plan. Deterministic."""
    L = [int(x) for x in lengths]
    plan = plan_batches(L, batch_tokens)
    costs = [batch_cost(len(b), -(-max(L[i] for i in b) // 64) * 64) for b in plan]
    order = sorted(range(len(plan)), key=lambda k: (-costs[k], k))
    load = [0.0] * world
    shards = [[] for _ in range(world)]
    for k in order:
        r = min(range(world), key=lambda j: (load[j], j))
        load[r] += costs[k]
        shards[r].extend(plan[k])
    return [sorted(sh) for sh in shards]


@functools.lru_cache(maxsize=16)
def _balanced(L: tuple, world: int, batch_tokens: int, max_rounds: int) -> tuple:
    # start from whichever of request-level LPT and batch-first LPT leaves the slowest rank
    # cheaper under the batch-plan model
    starts = [[lpt_shard(L, world, r) for r in range(world)], batch_first_shards(L, world, batch_tokens)]
    worst = [max(plan_cost([L[i] for i in sh], batch_tokens) for sh in st) for st in starts]
    shards = [list(sh) for sh in starts[0 if worst[0] <= worst[1] else 1]]
    if world > 1:
        cost = [plan_cost([L[i] for i in sh], batch_tokens) for sh in shards]
        for _ in range(max_rounds):
            hi = max(range(world), key=lambda r: (cost[r], -r))
            lo = min(range(world), key=lambda r: (cost[r], r))
            if hi == lo:
                break
            gap = cost[hi] - cost[lo]
            best = (cost[hi], None)
            a, b = shards[hi], shards[lo]
            # a change helps when it moves between 0 and `gap` of work; try the 48 whose per-request
            # cost moved is nearest half the gap (each try costs two plan evaluations)
            cands = [(abs(request_cost(L[i]) - gap / 2), i, -1) for i in a if request_cost(L[i]) < gap]
            cands += [(abs(request_cost(L[i]) - request_cost(L[j]) - gap / 2), i, j) for i in a for j in b
                      if 0.0 < request_cost(L[i]) - request_cost(L[j]) < gap]
            cands.sort()
            for _, i, j in cands[:48]:
                out_, in_ = [i], ([j] if j >= 0 else [])
                na = [i for i in a if i not in out_] + in_
                nb = [j for j in b if j not in in_] + out_
                ca = plan_cost([L[i] for i in na], batch_tokens)
                cb = plan_cost([L[j] for j in nb], batch_tokens)
                if max(ca, cb) < best[0] - 1e-9:
                    best = (max(ca, cb), (sorted(na), sorted(nb), ca, cb))
            if best[1] is None:
                break
            shards[hi], shards[lo], cost[hi], cost[lo] = best[1]
    return tuple(tuple(sorted(sh)) for sh in shards)


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
