"""Sequence sharding host logic on two gloo ranks (CPU): each rank decodes its
own prompts, and the job's rate is taken against the slowest rank."""

from __future__ import annotations

import socket

import torch.multiprocessing as mp

from breezetoken_b200.shard import aggregate_rate, max_over_ranks, rank_prompts


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        prompts = rank_prompts(rank, 2, 151936, 16)
        # rank r "took" 1 + r seconds and 10 + r seconds end to end
        slowest = max_over_ranks([1.0 + rank, 10.0 + rank])
        q.put((rank, prompts, slowest))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_sequences_and_take_the_slowest_time() -> None:
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (pr, sl)) for r, pr, sl in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (p0, s0), (p1, s1) = results[0], results[1]
    # every sequence of the job has its own prompt, reproducible by rank alone
    flat = [tuple(x) for x in p0 + p1]
    assert len(set(flat)) == 4
    assert p1 == rank_prompts(1, 2, 151936, 16)
    # both ranks see the slowest rank's times
    assert s0 == s1 == [2.0, 11.0]
    assert aggregate_rate(100, world, s0[0]) == 100.0


def test_single_process_needs_no_group() -> None:
    assert max_over_ranks([3.0, 4.0]) == [3.0, 4.0]
