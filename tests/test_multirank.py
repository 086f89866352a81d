"""The N>1 host logic of bench.py on CPU: two gloo ranks (one process per
rank, rendezvous on 127.0.0.1), max-over-ranks timing reduction, and the
reference arm running on rank 0 only."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


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
        got = bench.reduce_max([1.0 + rank, 10.0 - rank, 0.5 * rank], w)
        ref = None
        if r != 0:
            # The reference arm: non-zero ranks exit without work.
            class A:
                workload, steps, warmup = "c2", 1, 1
            ref = bench.run_reference(A())
        q.put((rank, (w, r, l), got, ref))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_max_and_rank0_reference():
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
    for rank, env, got, ref in results:
        assert env == (2, rank, rank)
        assert got == [2.0, 10.0, 0.5]
        if rank == 1:
            assert ref is None
