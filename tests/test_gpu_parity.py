"""GPU parity of the CUDA path (through the C ABI) against the golden
vectors of the reference engine and against the C restatement: integer
and float work bit-exact, draft logits included (the MTP RoPE table is
built with the reference's own float pow / cos / sin)."""
import os

import numpy as np
import pytest

from oracles import Oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.fixture(scope="module", params=["tiny", "mini", "midi", "midi_f16", "tiny_u8"])
def gcase(request):
    from conftest import model_dir
    import lz98
    name = request.param
    d = model_dir(name)
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    m = lz98.Model(d)
    yield name, d, g, m
    m.close()


def test_verify_forward_bit_exact(gcase):
    import lz98
    name, d, g, m = gcase
    s = lz98.State(m, 512, 4)
    p = g["prompt"]
    h = s.batch_capture(p[:-1], 0)
    assert bits_equal(h, g["prefill_hidden"])
    hv, lv = s.verify(g["verify_tokens"], len(p) - 1)
    assert bits_equal(hv, g["verify_hidden"])
    assert bits_equal(lv, g["verify_logits"])
    assert s.positions()[1] == int(g["ring_slot_after_verify"][0])
    s.close()


def test_capture_and_draft(gcase):
    import lz98
    name, d, g, m = gcase
    s = lz98.State(m, 512, 4)
    O = Oracle(d, 512, 4)
    p = g["prompt"]
    hb = s.batch_capture(p[:-1], 0)
    s.mtp_prefill(hb, p[1:], 0)
    lg = s.forward(p[-1], len(p) - 1, capture=True)
    assert bits_equal(s.chain(), g["capture_chain"])
    assert bits_equal(lg, g["capture_logits"])
    hbo, _ = O.forward(p[:-1], 0, 0, want_logits=False)
    O.mtp_prefill(hbo, p[1:], 0)
    O.set_chain(g["capture_chain"])
    for i, t in enumerate(g["draft_tokens"]):
        lgd = s.mtp_draft(int(t), len(p) - 1 + i)
        lgo = O.mtp_draft(int(t), len(p) - 1 + i)
        assert bits_equal(lgd, lgo), f"draft step {i} differs from the oracle"
        assert bits_equal(lgd, g["draft_logits"][i]), f"draft step {i} differs from the reference"
    assert bits_equal(s.chain(), O.chain())
    s.close()
    O.close()


@pytest.mark.parametrize("k", [0, 1, 2, 3])
def test_greedy_generation_token_identical(gcase, k):
    import lz98
    name, d, g, m = gcase
    s = lz98.State(m, 512, 4)
    max_new = 40 if name.startswith("tiny") else 48
    toks, rounds = s.generate(g["prompt"], max_new, k)
    tag = f"gen_t0_k{k}"
    assert np.array_equal(toks, g[tag + "_tokens"])
    assert np.array_equal(rounds, g[tag + "_rounds"])
    s.close()


def test_batched_rounds_match_per_sequence_oracle(gcase):
    """Three sequences in one state, rounds on the device; every sequence's
    emitted stream equals its own oracle generation."""
    import lz98
    name, d, g, m = gcase
    k, B, n_rounds = 2, 3, 6
    s = lz98.State(m, 256, 4, n_seq=B)
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, m.vocab, n).astype(np.int32) for n in (9, 17, 12)]
    emitted = [[] for _ in range(B)]
    for b in range(B):
        emitted[b].append(s.seq_prefill(b, prompts[b]))
    for _ in range(n_rounds):
        toks, cnt = s.round_batch(k)
        for b in range(B):
            emitted[b].extend(toks[b, :cnt[b]].tolist())
    O = Oracle(d, 256, 4)
    for b in range(B):
        n = len(emitted[b])
        want, _ = O.generate(prompts[b], n + 8, k)
        assert emitted[b] == want[:n].tolist(), f"sequence {b}"
    O.close()
    s.close()


def test_recurrence_block_shapes_agree(gcase):
    """The recurrence runs 16 warps per block when few (head, sequence)
    blocks exist and 8 otherwise: 40 sequences (8-warp blocks) reproduce,
    for the first three, the streams of a 3-sequence state (16-warp blocks,
    checked against the oracle above), greedy and at temperature 0.8."""
    import lz98
    name, d, g, m = gcase
    k, n_rounds = 2, 4
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, m.vocab, 9 + (b * 7) % 13).astype(np.int32) for b in range(40)]
    for temp in (0.0, 0.8):
        streams = []
        for B in (3, 40):
            s = lz98.State(m, 256, 4, n_seq=B)
            out = [[] for _ in range(3)]
            for b in range(B):
                s.set_sampler(b, temp, 0.95, 1000 + b)
                t = s.seq_prefill(b, prompts[b])
                if b < 3:
                    out[b].append(t)
            for _ in range(n_rounds):
                toks, cnt = s.round_batch(k)
                for b in range(3):
                    out[b].extend(toks[b, :cnt[b]].tolist())
            streams.append(out)
            s.close()
        assert streams[0] == streams[1], temp


def test_graph_and_eager_rounds_agree(gcase):
    """Graph replay with programmatic dependent launch against plain
    eager launches: identical tokens."""
    import lz98
    name, d, g, m = gcase
    outs = []
    for graphs in (True, False):
        s = lz98.State(m, 256, 4, n_seq=2)
        s.graphs(graphs)
        s.pdl(graphs)
        for b in range(2):
            s.seq_prefill(b, g["prompt"][: 10 + 5 * b])
        res = [s.round_batch(3) for _ in range(4)]
        outs.append([(t.tolist(), c.tolist()) for t, c in res])
        s.close()
    assert outs[0] == outs[1]


@pytest.mark.parametrize("k", [0, 1, 2, 3])
def test_temperature_generation_token_identical(gcase, k):
    """Coupled temperature rounds (temp 0.8, top-p 0.95, seed 1234): the
    device draft sampling, target distributions, acceptance and residual
    resampling reproduce the reference's token stream and round record."""
    import lz98
    name, d, g, m = gcase
    s = lz98.State(m, 512, 4)
    max_new = 40 if name.startswith("tiny") else 48
    toks, rounds = s.generate(g["prompt"], max_new, k, temp=0.8, topp=0.95, seed=1234)
    tag = f"gen_t8_k{k}"
    assert np.array_equal(toks, g[tag + "_tokens"])
    assert np.array_equal(rounds, g[tag + "_rounds"])
    s.close()


def test_pmin_nmin_generation_matches_reference(gcase):
    """Rounds with p_min (draft stops at the first step whose confidence -
    lz_argmax_p1 greedy, q(x) sampled - is below it) and n_min (short drafts
    discarded, then a fresh capture): the token stream and the (k_eff,
    n_accept) record of each round equal the reference engine's."""
    import lz98
    name, d, g, m = gcase
    if "pm_cases" not in g:
        pytest.skip("no p_min vectors for this model")
    max_new = 40 if name.startswith("tiny") else 48
    s = lz98.State(m, 512, 4)
    for j, (pm, nm, temp) in enumerate(g["pm_cases"]):
        toks, rounds = s.generate(g["prompt"], max_new, 3, temp=float(temp), topp=0.95, seed=1234,
                                  p_min=float(pm), n_min=int(nm))
        assert np.array_equal(rounds, g[f"pm{j}_rounds"]), (j, rounds[:, 0], g[f"pm{j}_rounds"][:, 0])
        assert np.array_equal(toks, g[f"pm{j}_tokens"]), j
    s.close()


def test_debug_counters(gcase):
    """With debug timing on, a generation still reproduces the reference's
    stream; lz_debug_n_ring_rollback grows by the rounds with n_accept <
    k_eff, and the event-timed draft and verify microseconds grow."""
    import lz98
    name, d, g, m = gcase
    max_new = 40 if name.startswith("tiny") else 48
    s = lz98.State(m, 512, 4)
    assert lz98.lib().lz_set_debug_timing(s.h, 1) == 0
    c0 = lz98.debug_counters()
    toks, rounds = s.generate(g["prompt"], max_new, 2)
    c1 = lz98.debug_counters()
    assert np.array_equal(toks, g["gen_t0_k2_tokens"])
    assert c1["lz_debug_n_ring_rollback"] - c0["lz_debug_n_ring_rollback"] == int((rounds[:, 1] < rounds[:, 0]).sum())
    assert c1["lz_debug_us_draft"] > c0["lz_debug_us_draft"]
    assert c1["lz_debug_us_verify"] > c0["lz_debug_us_verify"]
    assert lz98.lib().lz_set_debug_timing(s.h, 0) == 0
    s.close()


def test_batched_temperature_rounds_match_per_sequence_oracle(gcase):
    """Three sequences with their own generators in one state: the batched
    device temperature rounds emit each sequence's oracle stream."""
    import lz98
    name, d, g, m = gcase
    k, B, n_rounds = 3, 3, 5
    s = lz98.State(m, 256, 4, n_seq=B)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, m.vocab, n).astype(np.int32) for n in (11, 7, 15)]
    seeds = [1000 + b for b in range(B)]
    emitted = [[] for _ in range(B)]
    for b in range(B):
        s.set_sampler(b, 0.8, 0.95, seeds[b])
        emitted[b].append(s.seq_prefill(b, prompts[b]))
    for _ in range(n_rounds):
        toks, cnt = s.round_batch(k)
        for b in range(B):
            emitted[b].extend(toks[b, :cnt[b]].tolist())
    O = Oracle(d, 256, 4)
    for b in range(B):
        n = len(emitted[b])
        want, _ = O.generate(prompts[b], n + 8, k, temp=0.8, topp=0.95, seed=seeds[b])
        assert emitted[b] == want[:n].tolist(), f"sequence {b}"
    O.close()
    s.close()


def test_temperature_round_abi_advances_generator(gcase):
    """lz_spec_round_temp through the reference-shaped entry point: the
    generator state it returns continues the oracle's stream."""
    import lz98
    name, d, g, m = gcase
    p = g["prompt"]
    max_new = 40 if name.startswith("tiny") else 48
    O = Oracle(d, 512, 4)
    want, want_rounds = O.generate(p, max_new, 2, temp=0.8, topp=0.95, seed=77)
    O.close()
    s = lz98.State(m, 512, 4)
    toks, rounds = s.generate(p, max_new, 2, temp=0.8, topp=0.95, seed=77)
    assert np.array_equal(toks, want) and np.array_equal(rounds, want_rounds)
    s.close()


def test_mixed_batch_is_refused(gcase):
    import lz98
    name, d, g, m = gcase
    s = lz98.State(m, 128, 2, n_seq=2)
    s.set_sampler(0, 0.8, 0.95, 3)
    s.set_sampler(1, 0.0, 0.95, 3)
    for b in range(2):
        s.seq_prefill(b, g["prompt"][:8])
    with pytest.raises(lz98.LzError):
        s.round_batch(2)
    s.close()


def test_headline_config_token_identical():
    """The ~0.5B bench config itself (d 1024, 24 layers, 64 experts top-4,
    vocabulary 64000, MTP depth 2): the device generations reproduce the
    reference's token streams and round records, greedy and temperature,
    plain decode and k = 2, 3."""
    import lz98
    import lz98_synth
    from conftest import model_dir
    d = model_dir("0p5b")
    g = dict(np.load(os.path.join(GOLDEN, "0p5b.npz")))
    assert bytes(g["sha256"]).hex() == lz98_synth.write_model(lz98_synth.CONFIGS["0p5b"], d)
    m = lz98.Model(d)
    s = lz98.State(m, 512, 4)
    try:
        for j, (k, temp) in enumerate(g["runs"]):
            toks, rounds = s.generate(g["prompt"], int(g["max_new"][0]), int(k), temp=float(temp), topp=0.95,
                                      seed=1234)
            assert np.array_equal(toks, g[f"run{j}_tokens"]), (j, k, temp)
            assert np.array_equal(rounds, g[f"run{j}_rounds"]), (j, k, temp)
    finally:
        s.close()
        m.close()


def test_umma_and_mma_sync_gemms_agree(gcase):
    """The dense GEMMs of more than 8 token rows run on tcgen05 (default) or
    on the warp-level mma.sync kernel: the prompt capture (up to 39 rows)
    and 40-sequence rounds (120 verify rows, 40 draft rows, 80 catch-up
    rows) give the same bits either way, greedy and at temperature 0.8."""
    import lz98
    name, d, g, m = gcase
    p = g["prompt"]
    hs = []
    for on in (True, False):
        s = lz98.State(m, 512, 4)
        s.umma(on)
        hs.append(s.batch_capture(p[:-1], 0))
        s.close()
    assert bits_equal(hs[0], hs[1]) and bits_equal(hs[0], g["prefill_hidden"])
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, m.vocab, 9 + (b * 5) % 11).astype(np.int32) for b in range(40)]
    for temp in (0.0, 0.8):
        streams = []
        for on in (True, False):
            s = lz98.State(m, 256, 4, n_seq=40)
            s.umma(on)
            out = []
            for b in range(40):
                s.set_sampler(b, temp, 0.95, 500 + b)
                out.append(s.seq_prefill(b, prompts[b]))
            for _ in range(4):
                toks, cnt = s.round_batch(2)
                out.append((toks.tolist(), cnt.tolist()))
            streams.append(out)
            s.close()
        assert streams[0] == streams[1], temp


def _3b_model():
    import lz98_synth
    from conftest import model_dir
    d = model_dir("3b")
    sha = lz98_synth.write_model(lz98_synth.CONFIGS["3b"], d)
    return d, sha


def test_3b_config_token_identical():
    """configs[3], the ~3B model (d 2048, 32 layers, 32 KDA heads, 128
    experts top-8, latent 768, expert FFN 1536, vocabulary 128000): the
    device generations reproduce the reference's token streams and round
    records, greedy k = 3 and plain decode."""
    import lz98
    d, sha = _3b_model()
    g = dict(np.load(os.path.join(GOLDEN, "3b.npz")))
    assert bytes(g["sha256"]).hex() == sha
    m = lz98.Model(d)
    s = lz98.State(m, 512, 4)
    try:
        for j, (k, temp) in enumerate(g["runs"]):
            toks, rounds = s.generate(g["prompt"], int(g["max_new"][0]), int(k), temp=float(temp), topp=0.95,
                                      seed=1234)
            assert np.array_equal(toks, g[f"run{j}_tokens"]), (j, k, temp)
            assert np.array_equal(rounds, g[f"run{j}_rounds"]), (j, k, temp)
    finally:
        s.close()
        m.close()


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLDEN, "3b_long.npz")), reason="3b_long fixture not generated")
def test_3b_workload_chunked_prefill_token_identical():
    """configs[3]'s own workload shape: 8 sequences with 8192-token prompts
    prefilled in row-capacity chunks inside one 8-sequence state, then
    greedy k = 3 rounds of all 8 together; the first sequence's stream and
    round records equal the reference's (its whole prompt through the
    reference's chunked prefill)."""
    import lz98
    import lz98_synth
    d, sha = _3b_model()
    g = dict(np.load(os.path.join(GOLDEN, "3b_long.npz")))
    assert bytes(g["sha256"]).hex() == sha
    cfg = lz98_synth.CONFIGS["3b"]
    n_prompt, max_new = int(g["prompt_len"][0]), int(g["max_new"][0])
    prompts = lz98_synth.uniform_prompts(cfg, 8, n_prompt)
    m = lz98.Model(d)
    s = lz98.State(m, n_prompt + max_new + 64, 3, n_seq=8)
    try:
        emitted = [s.seq_prefill(b, p) for b, p in enumerate(prompts)]
        emitted = [[int(a)] for a in emitted]
        recs = []
        want_t, want_r = g["tokens"], g["rounds"]
        full = 0
        while full < len(want_r) and want_r[full][0] == 3:
            full += 1
        assert full >= 2, full
        for _ in range(full):
            toks, cnt = s.round_batch(3)
            for b in range(8):
                emitted[b].extend(toks[b, :cnt[b]].tolist())
            recs.append((3, int(cnt[0]) - 1))
        # every round the reference ran at full depth, and the tokens they emitted
        assert recs == [tuple(r) for r in want_r[:full].tolist()]
        n_tok = 1 + sum(int(r[1]) + 1 for r in want_r[:full])
        assert emitted[0][:n_tok] == want_t[:n_tok].tolist()
    finally:
        s.close()
        m.close()
