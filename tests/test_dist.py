"""Multi-process host logic of the data-parallel bench on CPU (gloo,
world_size 2): the rank reduction (max device time, summed tokens) and
the per-rank sequence partition."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms, tok, e2e = bench.reduce_over_ranks(10.0 + rank, 100.0 * (rank + 1), 5.0 + rank, world, "cpu")
        ms1, tok1, e2e1 = bench.reduce_over_ranks(1.0, 2.0, None, world, "cpu")
        first = [int(p[0]) for p in bench.prompts(2, rank)]
        out.put((rank, ms, tok, e2e, ms1, tok1, e2e1, first))
    finally:
        dist.destroy_process_group()


def test_reduce_and_partition_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    for r in res:
        assert r[1] == 11.0 and r[2] == 300.0 and r[3] == 11.0
        assert r[4] == 1.0 and r[5] == 4.0 and r[6] is None
    # each rank prefills its own sequences: different prompts per rank
    assert res[0][7] != res[1][7]


def test_single_rank_passthrough():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.reduce_over_ranks(3.0, 7.0, None, 1, "cpu") == (3.0, 7.0, None)
    p0 = bench.prompts(3, 0)
    assert len(p0) == 3 and all(len(p) == bench.PROMPT for p in p0)
    assert all(np.array_equal(a, b) for a, b in zip(p0, bench.prompts(3, 0)))
