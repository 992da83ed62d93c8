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


# a tiny drafter (CPU oracle) that stands in for the GPU draft of each request
_TINY = dict(target_hidden_size=64, vocab_size=512, target_layer_ids=[0], block_size=16, hidden_size=64,
             num_hidden_layers=1, num_attention_heads=2, intermediate_size=128, mlp_type="gelu")


def _tiny_drafter():
    from flashmap_b200 import FlashMapConfig
    from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
    from oracle.flashmap_oracle import Oracle

    config = FlashMapConfig(**_TINY)
    sd = synthetic_state_dict(config, seed=3, dtype=torch.float32)
    emb, head = synthetic_target_head(config, seed=3, dtype=torch.float32)
    return config, Oracle(config, sd, torch.float32), emb, head


def _draft_request(drafter, i, length):
    """Request i: its own seeded context of `length` positions, anchor and noise; one jump."""
    from oracle.flashmap_oracle import OracleCache

    config, oracle, emb, head = drafter
    g = torch.Generator().manual_seed(100 + i)
    K = config.block_size
    cache = OracleCache(config, 1, length + K + 2, torch.float32)
    oracle.extend_context(cache, torch.randn(1, length, config.target_hidden_size, generator=g))
    anchor = torch.randint(0, config.vocab_size, (1,), generator=g)
    z = torch.randn(1, K, config.target_hidden_size, generator=g)
    logits = oracle.draft(anchor, cache, emb, head, num_steps=1, z=z)
    return logits.float().argmax(-1).reshape(-1).tolist()


def _worker(rank, world, port, lengths, out, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from flashmap_b200.sharding import balanced_capacity

        mine = shard_requests(lengths, world, rank, capacity=balanced_capacity(len(lengths), world))
        ok = torch.tensor([0 if rank == fail_rank else 1], dtype=torch.int32)
        results = {}
        if rank != fail_rank:
            drafter = _tiny_drafter()
            for idx in chunks(mine, 4):
                for i in idx:
                    results[i] = _draft_request(drafter, i, lengths[i])
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
    """Two gloo ranks draft their LPT shares of 12 requests with the CPU oracle
    standing in for the GPU draft; together they reproduce, request by request,
    the tokens of drafting every request in one process."""
    lengths = [random.Random(11).randint(4, 40) for _ in range(12)]
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
        assert sorted(merged) == list(range(len(lengths)))
        assert {len(s) for s in shares} == {len(lengths) // 2}
        drafter = _tiny_drafter()
        for i, length in enumerate(lengths):
            assert merged[i] == _draft_request(drafter, i, length), f"request {i}"
    else:
        assert flags == {0}  # every rank saw the failure
