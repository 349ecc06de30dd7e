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


# ------------------------------------------------- expert-parallel bookkeeping
#
# The dispatch plan of the expert-parallel MoE layer (llama98-zh_b200/csrc/
# lz98_ep.cuh), restated on host arrays: each rank packs its (token,
# expert) pairs into its experts' owners' slot buffers in pair order, the
# buffers are exchanged, every owner runs its experts over the received
# pairs source by source, the answers go back to the slots they came from,
# and each token row combines its pairs in selection order.  Checked on two
# gloo ranks against the same layer computed on one process.

E_TOT, TOPK, LAT, WORLD = 8, 2, 4, 2


def _expert(e, x):
    """A stand-in expert: a fixed float32 map of the latent row per expert."""
    w = np.float32(0.5 + 0.125 * e)
    return (x * w + np.float32(e)).astype(np.float32)


def _pairs(rank):
    rng = np.random.default_rng(40 + rank)
    R = 5
    pe = np.stack([rng.choice(E_TOT, TOPK, replace=False) for _ in range(R)]).reshape(-1).astype(np.int32)
    pe[3] = -1                                     # an unrouted pair
    pw = rng.random(R * TOPK).astype(np.float32)
    lat = rng.standard_normal((R, LAT)).astype(np.float32)
    return pe, pw, lat


def _combine(pe, pw, rows):
    R = len(pe) // TOPK
    y = np.zeros((R, LAT), np.float32)
    for r in range(R):
        acc = np.zeros(LAT, np.float32)
        for t in range(TOPK):
            p = r * TOPK + t
            if pe[p] < 0:
                continue
            acc = (acc + (np.float32(pw[p]) * rows[p]).astype(np.float32)).astype(np.float32)
        y[r] = acc
    return y


def _ep_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        epr = E_TOT // world
        pe, pw, lat = _pairs(rank)
        P = len(pe)
        cap = P
        # pack: the stable slot of each pair at its owner, in pair order
        send = np.zeros((world, cap, LAT + 2), np.float32)   # latent | local expert | pair
        cnt = np.zeros(world, np.int64)
        dest = np.full(P, -1)
        slot = np.full(P, -1)
        for p in range(P):
            if pe[p] < 0:
                continue
            d = pe[p] // epr
            dest[p], slot[p] = d, cnt[d]
            send[d, cnt[d]] = np.concatenate([lat[p // TOPK], [pe[p] - d * epr, p]])
            cnt[d] += 1
        # exchange counts and slot buffers
        recv = np.zeros_like(send)
        rcnt = np.zeros(world, np.int64)
        for peer in range(world):
            if peer == rank:
                recv[peer], rcnt[peer] = send[peer], cnt[peer]
                continue
            c_out, c_in = torch.tensor([cnt[peer]]), torch.zeros(1, dtype=torch.int64)
            b_out, b_in = torch.from_numpy(send[peer].copy()), torch.zeros(cap, LAT + 2)
            ops = [dist.P2POp(dist.isend, c_out, peer), dist.P2POp(dist.irecv, c_in, peer),
                   dist.P2POp(dist.isend, b_out, peer), dist.P2POp(dist.irecv, b_in, peer)]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            recv[peer], rcnt[peer] = b_in.numpy(), int(c_in[0])
        # the owned experts over the received pairs, source by source; the
        # answers back to their slots
        back = np.zeros((world, cap, LAT), np.float32)
        for src in range(world):
            for i in range(rcnt[src]):
                e = rank * epr + int(recv[src, i, LAT])
                back[src, i] = _expert(e, recv[src, i, :LAT])
        ret = np.zeros_like(back)
        for peer in range(world):
            if peer == rank:
                ret[peer] = back[peer]
                continue
            b_out, b_in = torch.from_numpy(back[peer].copy()), torch.zeros(cap, LAT)
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, b_out, peer), dist.P2POp(dist.irecv, b_in, peer)]):
                w.wait()
            ret[peer] = b_in.numpy()
        rows = np.zeros((P, LAT), np.float32)
        for p in range(P):
            if dest[p] >= 0:
                rows[p] = ret[dest[p], slot[p]]
        out.put((rank, _combine(pe, pw, rows)))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_dispatch_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(WORLD):
        pe, pw, lat = _pairs(rank)
        rows = np.stack([_expert(e, lat[p // TOPK]) if e >= 0 else np.zeros(LAT, np.float32)
                         for p, e in enumerate(pe)])
        assert np.array_equal(res[rank].view(np.uint32), _combine(pe, pw, rows).view(np.uint32)), rank
