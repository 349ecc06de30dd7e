"""GPU tests of expert parallelism (lz_ep_init): the routed experts of
every layer split over ranks, pairs exchanged with NCCL, the combine in
selection order - the streams must be the single-GPU reference streams.

* one rank: the whole pack / exchange / unpack / grouped experts / reply /
  combine path runs (an exchange with no peers) and must reproduce the
  reference's generations and prompt capture bit for bit;
* two ranks (two GPUs, skipped with fewer): each rank in its own process
  with its own sequences; every pair whose expert the other rank owns
  crosses NVLink both ways."""
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch  # noqa: F401  (its NCCL is loaded before the library binds one)

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", ["tiny", "midi"])
def test_ep_single_rank_matches_reference(name):
    import lz98
    from conftest import model_dir
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    m = lz98.Model(model_dir(name))
    uid = lz98.ep_unique_id()
    s = lz98.State(m, 512, 4)
    s.ep_init(uid, 0, 1)
    h = s.batch_capture(g["prompt"][:-1], 0)
    assert np.array_equal(bits(h), bits(g["prefill_hidden"]))
    for k, temp in ((2, 0.0), (3, 0.8)):
        toks, rounds = s.generate(g["prompt"], 48 if name == "midi" else 40, k, temp=temp, topp=0.95, seed=1234)
        tag = f"gen_t{int(temp * 10)}_k{k}"
        assert np.array_equal(toks, g[tag + "_tokens"]) and np.array_equal(rounds, g[tag + "_rounds"]), tag
    s.close()
    m.close()


def _ep_rank(rank, world, uid, name, out):
    """One rank: its own 3 sequences (prompts of equal lengths on every
    rank, so both take the same forwards), temperature rounds."""
    try:
        import torch
        torch.cuda.set_device(rank)
        import sys
        here = os.path.dirname(os.path.abspath(__file__))
        sys.path.insert(0, here)
        sys.path.insert(0, os.path.join(os.path.dirname(here), "llama98-zh_b200"))
        import lz98
        from conftest import model_dir
        m = lz98.Model(model_dir(name))
        s = lz98.State(m, 256, 4, n_seq=3)
        s.ep_init(uid, rank, world)
        rng = np.random.default_rng(100 + rank)
        prompts = [rng.integers(0, m.vocab, n).astype(np.int32) for n in (11, 7, 15)]
        emitted = [[] for _ in range(3)]
        for b in range(3):
            s.set_sampler(b, 0.8, 0.95, 2000 + 10 * rank + b)
            emitted[b].append(s.seq_prefill(b, prompts[b]))
        for _ in range(5):
            toks, cnt = s.round_batch(3)
            for b in range(3):
                emitted[b].extend(toks[b, :cnt[b]].tolist())
        s.close()
        m.close()
        out.put((rank, [p.tolist() for p in prompts], emitted))
    except Exception as e:   # reported to the parent
        out.put((rank, None, repr(e)))


def test_ep_two_ranks_match_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import lz98
    from conftest import model_dir
    from oracles import Oracle
    name = "midi"
    d = model_dir(name)
    uid = lz98.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, uid, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, prompts, emitted = q.get(timeout=600)
            res[rank] = (prompts, emitted)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    O = Oracle(d, 256, 4)
    for rank in range(2):
        prompts, emitted = res[rank]
        assert prompts is not None, emitted
        for b in range(3):
            n = len(emitted[b])
            want, _ = O.generate(np.array(prompts[b], np.int32), n + 8, 3, temp=0.8, topp=0.95,
                                 seed=2000 + 10 * rank + b)
            assert emitted[b] == want[:n].tolist(), (rank, b)
    O.close()
