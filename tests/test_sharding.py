"""Request sharding across ranks (CPU, gloo): every request drafted by exactly
one rank, loads balanced to within one request, the same assignment derived
independently on every rank, and a rank that fails is reported to the others
on the host instead of hanging them."""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashmap_b200.sharding import chunks, lpt_assign, request_costs, shard_loads, shard_requests


def _lengths(n=512, seed=5):
    rng = random.Random(seed)
    return [rng.randint(1024, 8192) for _ in range(n)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_every_request_once_and_balanced(world):
    lengths = _lengths()
    shares = lpt_assign(request_costs(lengths), world)
    flat = sorted(i for s in shares for i in s)
    assert flat == list(range(len(lengths)))
    loads = shard_loads(lengths, world)
    biggest = max(request_costs(lengths))
    assert max(loads) - min(loads) <= biggest
    # LPT bound: the slowest rank within 4/3 of the optimum (mean is a lower bound)
    assert max(loads) <= 4.0 / 3.0 * (sum(loads) / world) + biggest


def test_deterministic_and_rank_local():
    lengths = _lengths(300, seed=9)
    a = [shard_requests(lengths, 4, r) for r in range(4)]
    b = [shard_requests(list(lengths), 4, r) for r in range(4)]
    assert a == b
    with pytest.raises(ValueError):
        shard_requests(lengths, 4, 4)
    assert chunks(list(range(130)), 64) == [list(range(64)), list(range(64, 128)), [128, 129]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lengths, out, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        mine = shard_requests(lengths, world, rank)
        # a rank's "drafting" step: here the per-request result is a pure function of the request
        ok = torch.tensor([0 if rank == fail_rank else 1], dtype=torch.int32)
        results = {i: lengths[i] * 3 + 1 for i in mine} if rank != fail_rank else {}
        # ranks learn of a failed rank on the host, between steps, before any further work
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        gathered = [None] * world
        dist.all_gather_object(gathered, (mine, results, int(ok.item())))
        if rank == 0:
            out.put(gathered)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_two_ranks_gloo(fail_rank):
    lengths = _lengths(200, seed=11)
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, out, fail_rank)) for r in range(2)]
    for p in procs:
        p.start()
    gathered = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shares = [g[0] for g in gathered]
    assert sorted(i for s in shares for i in s) == list(range(len(lengths)))
    assert not set(shares[0]) & set(shares[1])
    flags = {g[2] for g in gathered}
    if fail_rank < 0:
        assert flags == {1}
        merged = {}
        for g in gathered:
            merged.update(g[1])
        assert merged == {i: c * 3 + 1 for i, c in enumerate(lengths)}
    else:
        assert flags == {0}  # every rank saw the failure
