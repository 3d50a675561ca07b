"""The multi-GPU host logic (mica_b200.shard) with world_size 2 gloo ranks on CPU: both ranks
derive the same request plan, their shares partition the requests, the timing reduction is the
maximum over ranks, results gather on rank 0 in request order, and a rank that leaves before a
collective makes its peer fail within the group timeout instead of hanging."""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from mica_b200 import shard as SH  # noqa: E402

WORLD = 2


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _lengths(n=256, seed=4):
    g = torch.Generator().manual_seed(seed)
    x = torch.exp(torch.randn(n, generator=g, dtype=torch.float64) + torch.log(torch.tensor(1024.0)))
    return [int(v) for v in x.round().clamp(256, 32768)]


def _init(rank, port, timeout_s=30):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=timeout_s))


def _fake_score(i, length):
    """Stands in for a request's option probabilities: deterministic per request."""
    return [round((i * 7919 + length) % 1000 / 1000.0, 6), length]


def _worker(rank, port, out_dir):
    _init(rank, port)
    try:
        lengths = _lengths()
        mine = SH.lpt_shard(lengths, WORLD, rank)
        # every rank's share, seen from every rank: a partition of all requests
        shares = [None] * WORLD
        dist.all_gather_object(shares, mine)
        # timing: the box's time is the slowest rank's
        t = SH.max_over_ranks([10.0 + rank, 5.0 - rank])
        every = SH.per_rank([10.0 + rank, 5.0 - rank])
        # results: scored here, gathered on rank 0 in request order
        batches = SH.plan_batches([lengths[i] for i in mine], 16384)
        local = {}
        for b in batches:
            for j in b:
                i = mine[j]
                local[i] = _fake_score(i, lengths[i])
        res = SH.gather_to_rank0(local, WORLD)
        torch.save({'mine': mine, 'shares': shares, 't': t, 'every': every, 'res': res, 'batches': batches},
                   Path(out_dir) / f'rank{rank}.pt')
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_reduce_and_gather(tmp_path):
    mp.spawn(_worker, args=(_port(), str(tmp_path)), nprocs=WORLD, join=True)
    r0 = torch.load(tmp_path / 'rank0.pt', weights_only=False)
    r1 = torch.load(tmp_path / 'rank1.pt', weights_only=False)
    lengths = _lengths()
    assert r0['shares'] == r1['shares'] == [r0['mine'], r1['mine']]
    assert sorted(r0['mine'] + r1['mine']) == list(range(len(lengths)))
    assert not set(r0['mine']) & set(r1['mine'])
    # LPT balance: the two loads differ by at most the costliest request
    loads = [sum(SH.request_cost(lengths[i]) for i in m) for m in (r0['mine'], r1['mine'])]
    assert abs(loads[0] - loads[1]) <= max(SH.request_cost(L) for L in lengths)
    assert r0['t'] == r1['t'] == [11.0, 5.0]
    assert r0['every'] == r1['every'] == [[10.0, 5.0], [11.0, 4.0]]
    assert r0['res'] == [_fake_score(i, L) for i, L in enumerate(lengths)]
    assert r1['res'] is None
    # each rank's batches cover its requests once, within the token budget
    for r in (r0, r1):
        flat = sorted(j for b in r['batches'] for j in b)
        assert flat == list(range(len(r['mine'])))
        for b in r['batches']:
            pad = max(-(-lengths[r['mine'][j]] // 64) * 64 for j in b)
            assert len(b) == 1 or len(b) * pad <= 16384


def test_batch_plan_minimises_modelled_batch_cost():
    """The planner's partition is never worse, on its own objective (padded rows, their
    attention term and a fixed cost per batch), than the greedy fill of each batch up to the
    token budget, and respects the budget."""
    lengths = _lengths(n=200, seed=11)
    plan = SH.plan_batches(lengths, 16384)
    assert sorted(i for b in plan for i in b) == list(range(len(lengths)))

    def cost(batches):
        return sum(SH.batch_cost(len(b), -(-max(lengths[i] for i in b) // 64) * 64) for b in batches)

    assert abs(cost(plan) - SH.plan_cost(lengths, 16384)) < 1e-6 * cost(plan)

    order = sorted(range(len(lengths)), key=lambda i: (lengths[i], i))
    greedy, cur = [], []
    for i in order:
        pad = -(-lengths[i] // 64) * 64
        if cur and (len(cur) + 1) * pad > 16384:
            greedy.append(cur)
            cur = []
        cur.append(i)
    greedy.append(cur)
    assert cost(plan) <= cost(greedy)
    for b in plan:
        assert len(b) == 1 or len(b) * (-(-max(lengths[i] for i in b) // 64) * 64) <= 16384


def test_plan_is_the_single_process_plan():
    lengths = _lengths()
    assert SH.lpt_shard(lengths, 1, 0) == list(range(len(lengths)))
    assert SH.max_over_ranks([3.0, 4.0]) == [3.0, 4.0]
    assert SH.per_rank([3.0, 4.0]) == [[3.0, 4.0]]
    assert SH.gather_to_rank0({2: 'b', 0: 'a'}, 1) == ['a', 'b']
    with pytest.raises(ValueError):
        SH.lpt_shard(lengths, 2, 2)


def _leaver(rank, port, out_dir):
    _init(rank, port, timeout_s=5)
    if rank == 1:
        return                      # leaves between steps, joins no collective
    err = None
    try:
        SH.max_over_ranks([1.0])
    except Exception as e:          # gloo reports the lost peer (or the timeout)
        err = type(e).__name__
    Path(out_dir, 'rank0.txt').write_text(str(err))


def test_a_rank_that_leaves_makes_its_peer_fail_not_hang(tmp_path):
    ctx = mp.start_processes(_leaver, args=(_port(), str(tmp_path)), nprocs=WORLD, join=False, start_method='spawn')
    ctx.join(timeout=60)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert (tmp_path / 'rank0.txt').read_text() != 'None'


def test_plan_edge_cases():
    """No requests, one request past the token budget (it goes alone), more ranks than requests."""
    assert SH.plan_batches([], 16384) == []
    assert SH.lpt_shard([], 4, 3) == []
    assert SH.plan_batches([40000], 16384) == [[0]]
    plan = SH.plan_batches([40000, 100, 120], 16384)
    assert sorted(i for b in plan for i in b) == [0, 1, 2] and [0] in plan
    shares = [SH.lpt_shard([300, 5000], 4, r) for r in range(4)]
    assert sorted(i for s in shares for i in s) == [0, 1] and sum(1 for s in shares if not s) == 2


def test_balanced_shard_refines_lpt_against_the_batch_plans():
    """Every request lands on exactly one rank, every rank derives the same split, and the
    slowest rank's modelled plan cost is never above LPT's (the BASELINE config-4 set: 256
    lognormal requests, 8 ranks)."""
    lengths = _lengths(n=256, seed=3)
    for world in (2, 4, 8):
        bal = [SH.balanced_shard(lengths, world, r, 16384) for r in range(world)]
        assert sorted(i for sh in bal for i in sh) == list(range(len(lengths)))
        assert bal == [SH.balanced_shard(lengths, world, r, 16384) for r in range(world)]
        lpt = [SH.lpt_shard(lengths, world, r) for r in range(world)]
        worst = lambda shards: max(SH.plan_cost([lengths[i] for i in sh], 16384) for sh in shards)  # noqa: E731
        assert worst(bal) <= worst(lpt) + 1e-6
    assert SH.balanced_shard(lengths, 1, 0, 16384) == list(range(len(lengths)))
    assert SH.balanced_shard([], 4, 2, 16384) == []
    shares = [SH.balanced_shard([300, 5000], 4, r, 16384) for r in range(4)]
    assert sorted(i for s in shares for i in s) == [0, 1]
    with pytest.raises(ValueError):
        SH.balanced_shard(lengths, 2, 2, 16384)
