"""The ragged-batch partition across ranks (dropkv_b200.sharding): host logic only.

Every rank derives the same plan without communicating; the two-rank test runs
real gloo processes on CPU and checks that their plans cover the batch exactly
once, as the multi-GPU bench relies on.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dropkv_b200.sharding import (Unit, contiguous_partition, load_imbalance, lpt_partition, make_units,
                                  ragged_lengths, rank_plan)


def test_ragged_lengths_seeded_and_in_range():
    a = ragged_lengths(16, 4096, 65536, seed=5)
    assert a == ragged_lengths(16, 4096, 65536, seed=5)
    assert a != ragged_lengths(16, 4096, 65536, seed=6)
    assert len(a) == 16 and all(4096 <= x <= 65536 for x in a)


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_lpt_covers_every_unit_once_and_balances(n):
    units = make_units(ragged_lengths(16, 4096, 65536, seed=5), 32)
    parts = lpt_partition(units, n)
    flat = [u for p in parts for u in p]
    assert sorted(flat) == sorted(units) and len(set(flat)) == len(units)
    # longest-first greedy: the heaviest rank exceeds the mean by less than one unit
    loads = [sum(u.lk for u in p) for p in parts]
    assert max(loads) - sum(loads) / n <= max(u.lk for u in units)
    assert load_imbalance(parts) < 1.02
    assert parts == lpt_partition(list(reversed(units)), n)  # order of the input does not matter


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_contiguous_covers_every_unit_once_in_few_runs(n):
    units = make_units(ragged_lengths(16, 4096, 65536, seed=5), 32)
    parts = contiguous_partition(units, n)
    flat = [u for p in parts for u in p]
    assert flat == sorted(units, key=lambda u: (u.seq, u.layer))  # consecutive runs, in order
    loads = [sum(u.lk for u in p) for p in parts]
    assert max(loads) - sum(loads) / n <= max(u.lk for u in units)
    assert load_imbalance(parts) < 1.05
    # a rank holds whole layer ranges of few sequences (one call per sequence)
    assert max(len({u.seq for u in p}) for p in parts) <= -(-16 // n) + 2
    assert parts == contiguous_partition(list(reversed(units)), n)


def test_contiguous_small_cases():
    units = [Unit(0, 0, 10), Unit(0, 1, 10), Unit(1, 0, 10), Unit(1, 1, 10)]
    assert [[u.seq for u in p] for p in contiguous_partition(units, 2)] == [[0, 0], [1, 1]]
    assert contiguous_partition(units, 8)[0] == [Unit(0, 0, 10)]
    assert sum(len(p) for p in contiguous_partition(units, 8)) == 4
    with pytest.raises(ValueError):
        contiguous_partition(units, 0)


def test_lpt_uneven_units():
    units = [Unit(0, 0, 100), Unit(1, 0, 60), Unit(2, 0, 50), Unit(3, 0, 40)]
    parts = lpt_partition(units, 2)
    assert [sum(u.lk for u in p) for p in parts] == [140, 110]
    with pytest.raises(ValueError):
        lpt_partition(units, 0)
    with pytest.raises(ValueError):
        rank_plan(2, 2, [10, 20], 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out, method="lpt"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = ragged_lengths(16, 4096, 65536, seed=5)
        mine = rank_plan(rank, world, lengths, 32, method)
        gathered = [None] * world
        dist.all_gather_object(gathered, [(u.seq, u.layer, u.lk) for u in mine])
        # the bench's max-over-ranks reduction of device times
        t = torch.tensor([float(10 + rank)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out.put((gathered, float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("method", ["lpt", "contiguous"])
def test_two_gloo_ranks_plan_the_batch_exactly_once(method):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, method)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    all_units = set(make_units(ragged_lengths(16, 4096, 65536, seed=5), 32))
    got = [set(Unit(*t) for t in g) for g in gathered]
    assert got[0].isdisjoint(got[1]) and got[0] | got[1] == all_units
    assert tmax == 11.0
