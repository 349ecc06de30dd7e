"""GPU tests of the drop-in boundary and of the benchmarked shapes:

* the exact bench workloads against the reference's own streams
  (tests/golden/0p5b_bench.npz): the batch-1 headline (512-token prompt,
  greedy, k = 2) and four sequences of the batch-32 workload run inside a
  32-sequence state, so that the timed kernel instances (128 verify rows,
  32 draft rows) are the ones compared;
* the rounds' debug switches (debug_break_rollback, the reference's
  known-bad control, and debug_skip_catchup) against the reference with
  the same switches (tests/golden/round_debug.npz);
* sampler options the device does not carry are refused, not ignored;
* a round whose bounded device wait runs out returns LZ98_ERR_CUDA and the
  context stays usable;
* a generation through the reference-side shim (compiled here with gcc)."""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
LZ98_ERR_FORWARD, LZ98_ERR_CUDA = 20, 1000


@pytest.fixture(scope="module")
def bench_model():
    import lz98
    import lz98_synth
    from conftest import model_dir
    d = model_dir("0p5b")
    g = dict(np.load(os.path.join(GOLDEN, "0p5b_bench.npz")))
    assert bytes(g["sha256"]).hex() == lz98_synth.write_model(lz98_synth.CONFIGS["0p5b"], d)
    m = lz98.Model(d)
    yield m, g
    m.close()


def test_bench_b1_workload_token_identical(bench_model):
    """bench.py's headline workload: the 512-token prompt of
    bench.prompts(1, 0), greedy, k = 2 - the device rounds (batch 1, three
    verify rows) reproduce the reference's stream and round record."""
    import lz98
    import bench
    m, g = bench_model
    prompt = bench.prompts(1, 0)[0]
    assert np.array_equal(prompt, g["b1_prompt"])
    s = lz98.State(m, len(prompt) + 128, 4)
    toks, rounds = s.generate(prompt, int(g["b1_max_new"][0]), 2)
    s.close()
    assert np.array_equal(rounds, g["b1_rounds"])
    assert np.array_equal(toks, g["b1_tokens"])


def test_bench_b32_sequences_inside_32_sequence_state(bench_model):
    """The batch-32 workload itself (32 sequences, Zipf prompts of 256-1024
    tokens, temperature 0.8, top-p 0.95, seeds 1000 + b, k = 3): every round
    runs all 32 sequences (128 verify rows, 32 draft rows); the four pinned
    sequences' streams and (k, n_accept) records equal the reference's over
    every round the reference ran at full depth."""
    import lz98
    import lz98_synth
    m, g = bench_model
    cfg = lz98_synth.CONFIGS["0p5b"]
    prompts = lz98_synth.workload_prompts(cfg, 32, 256, 1024, 1.1, seed=0)
    pick = [int(b) for b in g["b32_pick"]]
    n_rounds = 14
    s = lz98.State(m, 1024 + 4 * n_rounds + 64, 3, n_seq=32)
    emitted = [[] for _ in range(32)]
    recs = [[] for _ in range(32)]
    for b, p in enumerate(prompts):
        s.set_sampler(b, 0.8, 0.95, 1000 + b)
        emitted[b].append(s.seq_prefill(b, p))
    for _ in range(n_rounds):
        toks, cnt = s.round_batch(3)
        for b in range(32):
            emitted[b].extend(toks[b, :cnt[b]].tolist())
            recs[b].append((3, int(cnt[b]) - 1))
    s.close()
    for b in pick:
        assert np.array_equal(np.array(prompts[b], np.int32), g[f"b32_{b}_prompt"])
        want_r = g[f"b32_{b}_rounds"]
        full = 0
        while full < len(want_r) and want_r[full][0] == 3:
            full += 1
        assert full >= 10, (b, full)
        assert recs[b][:full] == [tuple(r) for r in want_r[:full].tolist()], b
        n_tok = 1 + sum(int(r[1]) + 1 for r in want_r[:full])
        assert emitted[b][:n_tok] == g[f"b32_{b}_tokens"][:n_tok].tolist(), b


def _debug_stream(s, m, prompt, k, temp, br, sc, n_rounds):
    """The reference loop's first n_rounds full-depth rounds through
    lz_spec_round / lz_spec_round_temp with the debug switches."""
    s.reset()
    s.set_sampler(0, temp, 0.95, 1234)
    toks = [s.seq_prefill(0, prompt)]
    recs = []
    anchor, pos = toks[0], len(prompt) - 1
    rng = s.get_sampler(0)[2]
    for _ in range(n_rounds):
        if temp > 0:
            out, na, npos, ke, rng = s.spec_round_temp(anchor, pos, k, temp, 0.95, rng, break_rollback=br,
                                                       skip_catchup=sc)
        else:
            out, na, npos, ke = s.spec_round(anchor, pos, k, break_rollback=br, skip_catchup=sc)
        toks += out.tolist()
        recs.append((ke, na))
        anchor, pos = int(out[na]), npos
    return toks, recs


@pytest.mark.parametrize("case", range(5))
def test_round_debug_switches_match_reference(case):
    """debug_break_rollback (a rejecting round leaves the state ring where
    the verify left it) and debug_skip_catchup reproduce the reference's
    streams with the same switch; in the temperature cases those streams
    leave the normal ones, so a broken rollback is detectable."""
    import lz98
    from conftest import model_dir
    g = dict(np.load(os.path.join(GOLDEN, "round_debug.npz")))
    name = str(g["models"][case])
    k, temp, br, sc = g["cases"][case]
    k, br, sc = int(k), int(br), int(sc)
    want_t, want_r = g[f"c{case}_tokens"], g[f"c{case}_rounds"]
    full = 0
    while full < len(want_r) and want_r[full][0] == k:
        full += 1
    m = lz98.Model(model_dir(name))
    s = lz98.State(m, 512, 4)
    toks, recs = _debug_stream(s, m, g[f"c{case}_prompt"], k, float(temp), br, sc, full)
    s.close()
    m.close()
    assert recs == [tuple(r) for r in want_r[:full].tolist()]
    n_tok = 1 + sum(int(r[1]) + 1 for r in want_r[:full])
    assert toks[:n_tok] == want_t[:n_tok].tolist()
    if temp > 0:
        normal = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))[f"gen_t8_k{k}_tokens"]
        assert toks[:n_tok] != normal[:n_tok].tolist()


def test_sampler_options_refused(tiny_dir):
    """Penalties that act, top-k and min-p are refused with LZ_ERR_FORWARD
    (not silently ignored); the greedy round does not read temperature, so
    a sampler at temperature 0.8 with identity penalties gives the
    samp = NULL greedy round."""
    import lz98
    m = lz98.Model(tiny_dir)
    prompt = np.arange(1, 13, dtype=np.int32)
    s = lz98.State(m, 256, 4)
    a = s.seq_prefill(0, prompt)
    bad = [dict(repetition_penalty=1.1, repeat_last_n=64), dict(presence_penalty=0.5, repeat_last_n=-1)]
    for kw in bad:
        with pytest.raises(lz98.LzError) as e:
            s.spec_round(a, len(prompt) - 1, 2, samp=lz98.make_sampler(m.vocab, 0.0, 0.95, 7, **kw))
        assert e.value.code == -LZ98_ERR_FORWARD
    for kw in bad + [dict(topk=40), dict(minp=0.05)]:
        with pytest.raises(lz98.LzError) as e:
            s.spec_round_temp(a, len(prompt) - 1, 2, 0.8, 0.95, 7,
                              samp=lz98.make_sampler(m.vocab, 0.8, 0.95, 7, **kw))
        assert e.value.code == -LZ98_ERR_FORWARD
    # acting penalties with repeat_last_n = 0 are off in the reference too
    ok = lz98.make_sampler(m.vocab, 0.8, 0.95, 7, repetition_penalty=1.3, repeat_last_n=0)
    r1 = s.spec_round(a, len(prompt) - 1, 2, samp=ok)
    s.close()
    s = lz98.State(m, 256, 4)
    a2 = s.seq_prefill(0, prompt)
    r2 = s.spec_round(a2, len(prompt) - 1, 2)
    s.close()
    m.close()
    assert a == a2 and r1[0].tolist() == r2[0].tolist() and r1[1:] == r2[1:]


def test_round_wait_timeout_returns_error(mini_dir):
    """A real round whose TMA producer issues nothing for one pipeline stage
    (test hook, waits limited to 1 ms): the consumers' bounded waits give
    up, the round returns LZ98_ERR_CUDA instead of tokens from a partly
    filled tile, and the CUDA context survives - a fresh state then
    reproduces the reference's stream."""
    import lz98
    L = lz98.lib()
    m = lz98.Model(mini_dir)
    g = dict(np.load(os.path.join(GOLDEN, "mini.npz")))
    s = lz98.State(m, 256, 4, n_seq=3)          # 3 x (3 + 1) = 12 verify rows: TMA-staged kernels
    rng = np.random.default_rng(4)
    for b in range(3):
        s.seq_prefill(b, rng.integers(0, m.vocab, 10 + b).astype(np.int32))
    s.round_batch(3)                            # a normal round first
    assert L.lz_debug_inject_wait_timeout(1, 1.0) == 0
    try:
        with pytest.raises(lz98.LzError) as e:
            s.round_batch(3)
    finally:
        assert L.lz_debug_inject_wait_timeout(0, 0.0) == 0
    assert e.value.code == LZ98_ERR_CUDA and "gave up" in str(e.value)
    s.close()
    s = lz98.State(m, 512, 4)
    toks, rounds = s.generate(g["prompt"], 48, 3, temp=0.8, topp=0.95, seed=1234)
    s.close()
    m.close()
    assert np.array_equal(toks, g["gen_t8_k3_tokens"]) and np.array_equal(rounds, g["gen_t8_k3_rounds"])


def test_generation_through_reference_shim(tmp_path, tiny_dir):
    """The reference-side shim (llama98-zh_b200/shim/lz98_gpu_shim.c),
    compiled with gcc and linked with a small driver: it opens the library
    at run time and runs the reference loop's prefill and temperature
    rounds through gpu_prefill / gpu_spec_round with a caller-owned
    LZSampler; the stream equals the reference's."""
    so = os.path.join(ROOT, "llama98-zh_b200", "liblz98gpu.so")
    exe = str(tmp_path / "shim_main")
    subprocess.run(["gcc", "-std=c99", "-O1", "-I" + os.path.join(ROOT, "include"),
                    "-I" + os.path.join(ROOT, "llama98-zh_b200", "shim"),
                    os.path.join(ROOT, "llama98-zh_b200", "shim", "lz98_gpu_shim.c"),
                    os.path.join(HERE, "abi_c", "shim_main.c"), "-o", exe, "-ldl"], check=True)
    g = dict(np.load(os.path.join(GOLDEN, "tiny.npz")))
    want_r = g["gen_t8_k3_rounds"]
    n_rounds = 6
    assert all(r[0] == 3 for r in want_r[:n_rounds])
    out = subprocess.run([exe, so, "generate", tiny_dir, "3", "0.8", "1234", str(n_rounds)] +
                         [str(int(t)) for t in g["prompt"]], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    toks = [int(t) for t in out.stdout.split()]
    n_tok = 1 + sum(int(r[1]) + 1 for r in want_r[:n_rounds])
    assert toks == g["gen_t8_k3_tokens"][:n_tok].tolist()
