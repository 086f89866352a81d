"""The N>1 host logic of bench.py on CPU: two gloo ranks (one process per
rank, rendezvous on 127.0.0.1), max- and sum-over-ranks reductions, each
rank's shard of the job, and the reference arm running on rank 0 only."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    from datetime import timedelta
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        w, r, l = bench.dist_env()
        got = bench.reduce([1.0 + rank, 10.0 - rank, 0.5 * rank], w)
        tot = bench.reduce([1.0 + rank, 2.0], w, op="sum")
        units = {name: bench.rank_units(name, r, w, bench.SHARD[name]) for name in ("c2", "c3", "c4", "c1")}
        ref = None
        if r != 0:
            # The reference arm: non-zero ranks exit without work.
            class A:
                workload, steps, warmup = "c2", 1, 1
            ref = bench.run_reference(A())
        q.put((rank, (w, r, l), got, tot, units, ref))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_shard_and_rank0_reference():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import bench
    for rank, env, got, tot, units, ref in results:
        assert env == (2, rank, rank)
        assert got == [2.0, 10.0, 0.5]
        assert tot == [3.0, 4.0]
        assert units["c2"] == ([0, 1, 2, 3] if rank == 0 else [4, 5, 6, 7])
        assert units["c3"] == ([0, 1, 2, 3] if rank == 0 else [4, 5, 6, 7])
        assert units["c4"] == bench.balance(bench.c4_lengths(), 2)[rank]
        assert units["c1"] is None  # replicas
        if rank == 1:
            assert ref is None
    # The two ranks' shards cover every unit exactly once.
    c4 = sorted(u for r in results for u in r[4]["c4"])
    assert c4 == list(range(64))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_partition_the_job(world):
    import bench
    for n in (8, 30, 64):
        parts = [bench.shard_range(n, r, world) for r in range(world)]
        assert sorted(u for p in parts for u in p) == list(range(n))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1
    lens = bench.c4_lengths()
    parts = bench.balance(lens, world)
    assert sorted(u for p in parts for u in p) == list(range(64))
    loads = [sum(lens[i] for i in p) for p in parts]
    # Longest-first greedy stays within one sequence of the mean load.
    assert max(loads) - sum(loads) / world <= max(lens)
    if world == 8:
        assert max(loads) / (sum(loads) / world) < 1.03


def test_line_config_is_the_same_in_both_arms():
    import bench
    for name in ("c1", "c2", "c2fp16", "c3", "c4"):
        for world in (1, 2, 8):
            a = bench.line_config(name, world, bench.SHARD[name])
            b = bench.line_config(name, world, bench.SHARD[name])
            assert a == b and a["bytes_per_step"] > 0
    assert bench.job_bytes("c2") == 32 * 8 * (32768 * 128 * 2 + 5462 * 22 * 20) + 32 * 32 * 128 * 2 + 32 * 4
