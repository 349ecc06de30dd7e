"""CPU tests: the C restatement (oracle) against the golden vectors made by
the reference engine, and op by op against the reference itself when its
compiled library is present."""
import os

import numpy as np
import pytest

from oracles import Oracle, Reference, oracle_available, reference_available

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

pytestmark = pytest.mark.skipif(not oracle_available(), reason="oracle library not built")


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.fixture(scope="module", params=["tiny", "mini", "midi", "midi_f16", "tiny_u8"])
def case(request):
    from conftest import model_dir
    import lz98_synth
    name = request.param
    d = model_dir(name)
    g = load_golden(name)
    sha = lz98_synth.write_model(lz98_synth.CONFIGS[name], d)
    assert bytes(g["sha256"]).hex() == sha, "model writer drifted from the golden vectors"
    return name, d, g


def test_oracle_forward_matches_golden(case):
    name, d, g = case
    O = Oracle(d, 512, 4)
    p = g["prompt"]
    h, _ = O.forward(p[:-1], 0, 0, want_logits=False)
    assert bits_equal(h, g["prefill_hidden"])
    hv, lv = O.forward(g["verify_tokens"], len(p) - 1, 1)
    assert bits_equal(hv, g["verify_hidden"])
    assert bits_equal(lv, g["verify_logits"])
    assert O.positions()[1] == int(g["ring_slot_after_verify"][0])
    O.close()


def test_oracle_draft_matches_golden(case):
    name, d, g = case
    O = Oracle(d, 512, 4)
    p = g["prompt"]
    hb, _ = O.forward(p[:-1], 0, 0, want_logits=False)
    O.mtp_prefill(hb, p[1:], 0)
    hc, lc = O.forward(p[-1:], len(p) - 1, 0)
    assert bits_equal(hc[0], g["capture_chain"])
    assert bits_equal(lc[0], g["capture_logits"])
    O.set_chain(hc[0])
    for i, t in enumerate(g["draft_tokens"]):
        lg = O.mtp_draft(int(t), len(p) - 1 + i)
        # bit-exact: the MTP RoPE table is built with the reference's own
        # all-float pow / cos / sin (lz98_rope_table.h)
        assert bits_equal(lg, g["draft_logits"][i]), f"draft step {i}"
    O.close()


@pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")
def test_rope_table_matches_reference():
    """The restated RoPE table (llama98-zh_b200/csrc/lz98_rope_table.h, used
    by the library and the oracle) equals the reference's own rope_cs bit for
    bit over 4096 positions, including the angles above 120 radians that take
    the 192-bit reduction."""
    import ctypes
    from conftest import model_dir
    d = model_dir("midi")
    R = Reference(d, 4096, 4)
    R.L.rd_rope_table.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    O = Oracle(d, 16, 4)
    O.L.lzo_rope_table.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    n = 4096 * 64
    ref = np.zeros(n, np.float32)
    got = R.L.rd_rope_table(ctypes.c_void_p(R.h), ref.ctypes.data_as(ctypes.c_void_p), n)
    assert got > 0
    rot = got // 4096
    import lz98_synth
    theta = lz98_synth.CONFIGS["midi"].rope_theta
    ours = np.zeros(got, np.float32)
    O.L.lzo_rope_table(theta, rot, 4096, ours.ctypes.data_as(ctypes.c_void_p))
    assert bits_equal(ours, ref[:got])
    R.close()
    O.close()


@pytest.mark.parametrize("temp", [0.0, 0.8])
@pytest.mark.parametrize("k", [0, 1, 2, 3])
def test_oracle_generation_matches_golden(case, temp, k):
    name, d, g = case
    O = Oracle(d, 512, 4)
    tag = f"gen_t{int(temp * 10)}_k{k}"
    toks, rounds = O.generate(g["prompt"], 40 if name.startswith("tiny") else 48, k, temp=temp, seed=1234)
    assert np.array_equal(toks, g[tag + "_tokens"])
    assert np.array_equal(rounds, g[tag + "_rounds"])
    O.close()


# ------------------------------------------------- op level, against the reference

needs_ref = pytest.mark.skipif(not reference_available(), reason="reference library not built here")


@pytest.fixture(scope="module")
def pair(tiny_dir):
    O = Oracle(tiny_dir, 256, 4)
    R = Reference(tiny_dir, 256, 4)
    yield O, R
    O.close()
    R.close()


@needs_ref
@pytest.mark.parametrize("fn", ["exp", "rsqrt", "sigmoid"])
def test_scalar_math_bit_exact(pair, fn):
    O, R = pair
    rng = np.random.default_rng(5)
    xs = np.concatenate([rng.standard_normal(3000) * 30, rng.uniform(-90, 90, 2000),
                         [0.0, -0.0, 88.0, 88.5, -87.3, -87.4, 1e-30, 1e30]]).astype(np.float32)
    if fn == "rsqrt":
        xs = np.abs(xs) + np.float32(1e-30)
    fo, fr = getattr(O.L, "lzo_" + fn), getattr(R.L, "rd_" + fn)
    bad = [float(x) for x in xs if np.float32(fo(float(x))).tobytes() != np.float32(fr(float(x))).tobytes()]
    assert not bad, bad[:5]


@needs_ref
@pytest.mark.parametrize("gs_mode", ["32", "row"])
@pytest.mark.parametrize("in_dim,out_dim,nt", [(64, 48, 1), (512, 33, 3), (1024, 40, 5), (2048, 16, 2)])
def test_matmul_q8_bit_exact(pair, gs_mode, in_dim, out_dim, nt):
    O, R = pair
    import ctypes
    rng = np.random.default_rng(in_dim + out_dim)
    gs = 32 if gs_mode == "32" else in_dim
    x = (rng.standard_normal((nt, in_dim)) * rng.uniform(0.01, 3)).astype(np.float32)
    wq = rng.integers(-127, 128, (out_dim, in_dim)).astype(np.int8)
    ws = (rng.random((out_dim, in_dim // gs)) * 0.01).astype(np.float32)
    xq = np.zeros((nt, in_dim), np.int8)
    xs = np.zeros((nt, in_dim // 32), np.float32)
    xq2, xs2 = xq.copy(), xs.copy()
    V = ctypes.c_void_p
    for t in range(nt):
        O.L.lzo_quantize_q8(V(x[t].ctypes.data), in_dim, 32, V(xq[t].ctypes.data), V(xs[t].ctypes.data))
        R.L.rd_quantize_q8(V(x[t].ctypes.data), in_dim, 32, V(xq2[t].ctypes.data), V(xs2[t].ctypes.data))
    assert np.array_equal(xq, xq2) and bits_equal(xs, xs2)
    o1 = np.zeros((nt, out_dim), np.float32)
    o2 = np.zeros((nt, out_dim), np.float32)
    O.L.lzo_matmul_q8(V(o1.ctypes.data), V(xq.ctypes.data), V(xs.ctypes.data), V(wq.ctypes.data),
                      V(ws.ctypes.data), gs, in_dim, out_dim, nt)
    R.L.rd_matmul_q8(V(o2.ctypes.data), V(xq.ctypes.data), V(xs.ctypes.data), V(wq.ctypes.data),
                     V(ws.ctypes.data), gs, in_dim, out_dim, nt)
    assert bits_equal(o1, o2)


@needs_ref
def test_kda_recurrence_bit_exact(pair):
    O, R = pair
    import ctypes
    V = ctypes.c_void_p
    rng = np.random.default_rng(9)
    kd = vd = 64
    hi = rng.integers(-127, 128, (kd, vd)).astype(np.int8)
    lo = rng.integers(-127, 128, (kd, vd)).astype(np.int8)
    ss = (rng.random((kd, vd // 32)) * 0.01).astype(np.float32)
    q = rng.standard_normal(kd).astype(np.float32); q /= np.linalg.norm(q)
    k = rng.standard_normal(kd).astype(np.float32); k /= np.linalg.norm(k)
    v = rng.standard_normal(vd).astype(np.float32)
    g = rng.uniform(0.01, 1.0, kd).astype(np.float32)
    outs = []
    for L, fn in ((O.L, "lzo_recur_step"), (R.L, "rd_recur_step")):
        out = np.zeros(vd, np.float32)
        h2, l2, s2 = np.zeros_like(hi), np.zeros_like(lo), np.zeros_like(ss)
        getattr(L, fn)(V(out.ctypes.data), V(hi.ctypes.data), V(h2.ctypes.data), V(lo.ctypes.data),
                       V(l2.ctypes.data), V(ss.ctypes.data), V(s2.ctypes.data), V(q.ctypes.data),
                       V(k.ctypes.data), V(v.ctypes.data), V(g.ctypes.data), ctypes.c_float(0.37), kd, vd)
        outs.append((out, h2, l2, s2))
    (o1, a1, b1, c1), (o2, a2, b2, c2) = outs
    assert bits_equal(o1, o2) and np.array_equal(a1, a2) and np.array_equal(b1, b2) and bits_equal(c1, c2)


@needs_ref
@pytest.mark.parametrize("E,topk", [(8, 2), (64, 4), (128, 8)])
def test_moe_route_matches(pair, E, topk):
    O, R = pair
    import ctypes
    V = ctypes.c_void_p
    rng = np.random.default_rng(E)
    for trial in range(20):
        lg = (rng.standard_normal(E) * 2).astype(np.float32)
        if trial % 5 == 0:
            lg[3] = lg[5]          # ties must keep the first index
        bias = (rng.standard_normal(E) * 0.02).astype(np.float32)
        res = []
        for L, fn in ((O.L, "lzo_moe_route"), (R.L, "rd_moe_route")):
            idx = np.zeros(topk, np.int32)
            w = np.zeros(topk, np.float32)
            getattr(L, fn)(V(lg.ctypes.data), V(bias.ctypes.data), E, topk, 1, 1, V(idx.ctypes.data), V(w.ctypes.data))
            res.append((idx, w))
        assert np.array_equal(res[0][0], res[1][0]) and bits_equal(res[0][1], res[1][1])


@needs_ref
def test_target_dist_matches(pair):
    O, R = pair
    import ctypes
    V = ctypes.c_void_p
    rng = np.random.default_rng(2)
    for n in (100, 8192):
        lg = (rng.standard_normal(n) * 1.5).astype(np.float32)
        p1, p2 = np.zeros(n, np.float32), np.zeros(n, np.float32)
        a, b = lg.copy(), lg.copy()
        O.L.lzo_target_dist(ctypes.c_float(0.8), ctypes.c_float(0.95), V(a.ctypes.data), n, V(p1.ctypes.data))
        R.L.rd_target_dist(ctypes.c_float(0.8), ctypes.c_float(0.95), V(b.ctypes.data), n, V(p2.ctypes.data))
        assert bits_equal(p1, p2)


@needs_ref
def test_argmax_p1_matches(pair):
    """lz_argmax_p1 (src/sampler.c:279-295): the oracle's index and
    online-softmax probability equal the reference's bit for bit."""
    import ctypes
    from argmax_rows import argmax_rows
    O, R = pair
    V, P = ctypes.c_void_p, ctypes.POINTER
    O.L.lzo_argmax_p1.argtypes = [V, ctypes.c_int, P(ctypes.c_float)]
    R.L.rd_argmax_p1.argtypes = [V, ctypes.c_int, P(ctypes.c_float)]
    for row in argmax_rows():
        a, b = ctypes.c_float(), ctypes.c_float()
        i1 = O.L.lzo_argmax_p1(V(row.ctypes.data), len(row), ctypes.byref(a))
        i2 = R.L.rd_argmax_p1(V(row.ctypes.data), len(row), ctypes.byref(b))
        assert i1 == i2
        assert np.float32(a.value).view(np.uint32) == np.float32(b.value).view(np.uint32)



@needs_ref
def test_reference_stock_tier_and_back(tiny_dir):
    """The reference's default arithmetic (--fixed all, --fastfp on), which
    the bench times beside the parity tier, runs on the same model; the
    tier is process-global, and selecting the parity tier again brings back
    the golden greedy stream exactly."""
    g = load_golden("tiny")
    R = Reference(tiny_dir, 512, 4)
    try:
        R.stock_tier()
        toks, _ = R.generate(g["prompt"], 40, 1)
        assert len(toks) == 40 and int(toks.min()) >= 0 and int(toks.max()) < R.vocab
        R.L.rd_set_tier(7)
        toks, rounds = R.generate(g["prompt"], 40, 1)
        assert np.array_equal(toks, g["gen_t0_k1_tokens"])
        assert np.array_equal(rounds, g["gen_t0_k1_rounds"])
    finally:
        R.L.rd_set_tier(7)
        R.close()


@needs_ref
@pytest.mark.parametrize("name,plen", [("tiny", 1), ("tiny", 2), ("tiny", 3), ("tiny", 5),
                                       ("mini", 1), ("mini", 5), ("midi", 1), ("midi", 5),
                                       ("midi_f16", 1), ("midi_f16", 5), ("tiny_u8", 1), ("tiny_u8", 5)])
def test_oracle_generation_edge_cases_match_reference(name, plen):
    """Short prompts (down to one token, where the capture prefill is empty)
    and short generations (max_new below k + 1, so the last round is cut)
    for every draft depth 0..3, greedy and temperature, on every parity
    config (per-32 and per-row scales, binary16 and u8-code scale planes):
    the restatement and the live reference emit the same tokens and the
    same round records."""
    from conftest import model_dir
    d = model_dir(name)
    O = Oracle(d, 512, 4)
    R = Reference(d, 512, 4)
    try:
        rng = np.random.default_rng([7, plen])
        prompt = rng.integers(0, O.vocab, plen).astype(np.int32)
        for max_new in (1, 2, 3, 7):
            for k in (0, 1, 2, 3):
                for temp in (0.0, 0.8):
                    to, ro = O.generate(prompt, max_new, k, temp=temp, seed=99)
                    tr, rr = R.generate(prompt, max_new, k, temp=temp, seed=99)
                    ctx = (plen, max_new, k, temp)
                    assert np.array_equal(to, tr), ctx
                    assert np.array_equal(ro, rr), ctx
    finally:
        O.close()
        R.close()


def test_oracle_pmin_nmin_matches_golden():
    """Rounds with p_min / n_min (drafting stopped at a low-confidence
    step, short drafts discarded before the verify) reproduce the
    reference's golden generations, greedy and temperature."""
    from conftest import model_dir
    for name in ("tiny", "midi"):
        g = load_golden(name)
        O = Oracle(model_dir(name), 512, 4)
        try:
            max_new = 40 if name.startswith("tiny") else 48
            for j, (pm, nm, temp) in enumerate(g["pm_cases"]):
                toks, rounds = O.generate(g["prompt"], max_new, 3, temp=float(temp), seed=1234,
                                          p_min=float(pm), n_min=int(nm))
                assert np.array_equal(toks, g[f"pm{j}_tokens"]), (name, j)
                assert np.array_equal(rounds, g[f"pm{j}_rounds"]), (name, j)
        finally:
            O.close()


@needs_ref
@pytest.mark.parametrize("name", ["tiny", "mini", "midi", "midi_f16", "tiny_u8"])
def test_oracle_pmin_nmin_matches_reference(name):
    """A sweep of p_min thresholds (from never stopping to stopping at the
    first step) and n_min 0..3, greedy and temperature, against the live
    reference: same tokens and the same (k_eff, n_accept) round records,
    discarded rounds included."""
    from conftest import model_dir
    d = model_dir(name)
    g = load_golden(name)
    O = Oracle(d, 512, 4)
    R = Reference(d, 512, 4)
    try:
        for pm in (0.0, 1e-4, 3.5e-4, 1.2e-3, 0.5):
            for nm in (0, 2, 3):
                for temp in (0.0, 0.8):
                    to, ro = O.generate(g["prompt"], 24, 3, temp=temp, seed=1234, p_min=pm, n_min=nm)
                    tr, rr = R.generate(g["prompt"], 24, 3, temp=temp, seed=1234, p_min=pm, n_min=nm)
                    assert np.array_equal(to, tr), (pm, nm, temp)
                    assert np.array_equal(ro, rr), (pm, nm, temp)
    finally:
        O.close()
        R.close()


def test_oracle_headline_config_matches_golden():
    """The ~0.5B bench config itself (d 1024, 24 layers, 64 experts top-4,
    vocabulary 64000, MTP depth 2): the restatement reproduces the
    reference's token streams and round records, greedy and temperature,
    plain decode and k = 2, 3."""
    from conftest import model_dir
    import lz98_synth
    d = model_dir("0p5b")
    g = load_golden("0p5b")
    sha = lz98_synth.write_model(lz98_synth.CONFIGS["0p5b"], d)
    assert bytes(g["sha256"]).hex() == sha, "model writer drifted from the golden vectors"
    O = Oracle(d, 512, 4)
    try:
        for j, (k, temp) in enumerate(g["runs"]):
            toks, rounds = O.generate(g["prompt"], int(g["max_new"][0]), int(k), temp=float(temp), seed=1234)
            assert np.array_equal(toks, g[f"run{j}_tokens"]), (j, k, temp)
            assert np.array_equal(rounds, g[f"run{j}_rounds"]), (j, k, temp)
    finally:
        O.close()


def test_bench_golden_inputs_regenerate():
    """The pinned bench workloads (tests/golden/0p5b_bench.npz) are the ones
    bench.py runs: the batch-1 prompt is bench.prompts(1, 0)[0], the batch-32
    prompts are workload_prompts(cfg, 32, 256, 1024, 1.1, seed=0) with the
    shortest and the longest among the pinned four."""
    import bench
    import lz98_synth
    from golden.make_golden import b32_pick
    g = np.load(os.path.join(GOLDEN, "0p5b_bench.npz"))
    assert np.array_equal(bench.prompts(1, 0)[0], g["b1_prompt"])
    prompts = lz98_synth.workload_prompts(lz98_synth.CONFIGS["0p5b"], 32, 256, 1024, 1.1, seed=0)
    assert b32_pick(prompts) == g["b32_pick"].tolist()
    lens = [len(p) for p in prompts]
    assert min(lens) in [len(g[f"b32_{b}_prompt"]) for b in g["b32_pick"]]
    assert max(lens) in [len(g[f"b32_{b}_prompt"]) for b in g["b32_pick"]]
    for b in g["b32_pick"]:
        assert np.array_equal(np.array(prompts[b], np.int32), g[f"b32_{b}_prompt"])


@needs_ref
@pytest.mark.parametrize("temp,k", [(0.0, 2), (0.8, 3)])
def test_reference_session_slices_match_golden(tiny_dir, temp, k):
    """The reference driver's resumable generation (prefill once, decode in
    slices, as the bench's reference arm times it) emits the golden stream
    and round records of the one-shot generation, whatever the slicing."""
    g = load_golden("tiny")
    tag = f"gen_t{int(temp * 10)}_k{k}"
    R = Reference(tiny_dir, 512, 4)
    try:
        for slices in ((40,), (1, 5, 34), (7, 7, 7, 7, 7, 7, 7)):
            R.session_begin(g["prompt"], 40, k, temp=temp, seed=1234)
            toks, rounds = [], []
            for n in slices:
                t, r, _ = R.session_decode(n)
                toks.append(t)
                rounds.append(r)
            # the budget ends the generation: nothing more comes out
            t, r, _ = R.session_decode(8)
            assert len(t) == 0 and len(r) == 0
            R.session_end()
            assert np.array_equal(np.concatenate(toks), g[tag + "_tokens"]), slices
            assert np.array_equal(np.concatenate(rounds), g[tag + "_rounds"]), slices
    finally:
        R.close()
