"""Generates the golden vectors of the MTP speculative path by running the
reference engine itself (oracle/_ref/liblz98ref.so, compiled unmodified
from the reference sources) on the synthetic models of lz98_synth.

    python tests/golden/make_golden.py

Writes tests/golden/<model>.npz.  Each file records the sha256 of the
model's tensor stream, so a change of the writer is detected instead of
silently comparing against other weights."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "llama98-zh_b200"))

import lz98_synth  # noqa: E402
from conftest import model_dir  # noqa: E402
from oracles import Reference  # noqa: E402

CASES = {
    # name: (prompt length, verify tokens, draft tokens, max_new)
    "tiny": (24, 4, 3, 40),
    "mini": (40, 4, 3, 48),
    "midi": (40, 4, 3, 48),
    "midi_f16": (40, 4, 3, 48),
    "tiny_u8": (24, 4, 3, 40),
}


# token-stream-only fixtures of larger configs: name: (prompt length,
# max_new, [(k, temperature), ...])
TOKEN_CASES = {
    "0p5b": (12, 12, [(0, 0.0), (2, 0.0), (2, 0.8), (3, 0.8)]),
    "3b": (12, 16, [(3, 0.0), (0, 0.0)]),
}


# configs[3] at its own prompt length: the first sequence of the workload
# (lz98_synth.uniform_prompts(cfg, 8, 8192)), its whole 8192-token prompt
# through the reference's chunked prefill, then greedy k = 3 rounds.
LONG_3B_PROMPT = 8192
LONG_3B_NEW = 16


# The benchmarked workloads themselves (bench.py), on the ~0.5B config:
#  - b1: the headline, bench.prompts(1, 0)[0] (512 uniform ids), greedy,
#    k = 2, BENCH_B1_NEW new tokens;
#  - b32: four sequences of the batch-32 workload
#    (lz98_synth.workload_prompts(cfg, 32, 256, 1024, 1.1, seed=0): the
#    shortest, the longest and two more), each with its own sampler
#    (temperature 0.8, top-p 0.95, seed 1000 + b), k = 3, BENCH_B32_NEW
#    new tokens.
BENCH_B1_NEW = 48
BENCH_B32_NEW = 32
BENCH_B32_SEQS = 32


# The rounds' test-only switches on the reference itself: (model, k,
# temperature, debug_break_rollback, debug_skip_catchup).  The temperature
# rounds both reject and accept runs of drafts, so both switches change the
# stream (it leaves the normal generation within the first 10 tokens on
# every case below); the greedy streams of these random-weight models repeat
# one token, so the greedy case only pins the switch's bookkeeping.
DEBUG_CASES = [("tiny", 3, 0.8, 1, 0), ("tiny", 3, 0.8, 0, 1), ("midi", 3, 0.8, 1, 0),
               ("midi_f16", 3, 0.8, 0, 1), ("tiny", 2, 0.0, 1, 0)]


PM_CASES = {
    "tiny": [(3.5e-4, 0, 0.0), (3.5e-4, 2, 0.0), (2e-4, 0, 0.8), (1e-4, 2, 0.8)],
    "midi": [(1.2e-3, 0, 0.0), (1.2e-3, 2, 0.0), (2e-4, 0, 0.8), (6e-4, 2, 0.8)],
}


def make(name):
    d = model_dir(name)
    cfg = lz98_synth.CONFIGS[name]
    sha = lz98_synth.write_model(cfg, d)
    n_prompt, n_ver, n_draft, max_new = CASES[name]
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, cfg.vocab, n_prompt).astype(np.int32)
    vt = np.concatenate([prompt[-1:], rng.integers(0, cfg.vocab, n_ver - 1)]).astype(np.int32)
    dt = rng.integers(0, cfg.vocab, n_draft).astype(np.int32)
    R = Reference(d, 512, 4)
    out = {"sha256": np.frombuffer(bytes.fromhex(sha), np.uint8), "prompt": prompt, "verify_tokens": vt,
           "draft_tokens": dt}
    # prefill capture, then a (k+1)-row verify through the ring
    out["prefill_hidden"] = R.batch_capture(prompt[:-1], 0)
    h, lg = R.verify(vt, n_prompt - 1)
    out["verify_hidden"], out["verify_logits"] = h, lg
    out["ring_slot_after_verify"] = np.array([R.info()[5]], np.int32)
    # MTP: prompt prefill, capture of the last prompt token, draft chain
    R.reset()
    hb = R.batch_capture(prompt[:-1], 0)
    R.mtp_prefill(hb, prompt[1:], 0)
    ch, lgc = R.forward_capture(int(prompt[-1]), n_prompt - 1)
    out["capture_chain"], out["capture_logits"] = ch, lgc
    dl = []
    for i, t in enumerate(dt):
        lgd, _ = R.mtp_draft(int(t), n_prompt - 1 + i)
        dl.append(lgd)
    out["draft_logits"] = np.stack(dl)
    # whole generations
    for temp in (0.0, 0.8):
        for k in (0, 1, 2, 3):
            toks, rounds = R.generate(prompt, max_new, k, temp=temp, seed=1234)
            tag = f"gen_t{int(temp * 10)}_k{k}"
            out[tag + "_tokens"], out[tag + "_rounds"] = toks, rounds
    # rounds with p_min / n_min: (p_min, n_min, temperature), thresholds
    # where the drafts' confidences straddle them on this model
    cases = PM_CASES.get(name, [])
    if cases:
        out["pm_cases"] = np.array(cases, np.float64)
        for j, (pm, nm, temp) in enumerate(cases):
            toks, rounds = R.generate(prompt, max_new, 3, temp=temp, seed=1234, p_min=pm, n_min=int(nm))
            out[f"pm{j}_tokens"], out[f"pm{j}_rounds"] = toks, rounds
    R.close()
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))


def make_tokens(name):
    """Prompt and whole generations only (no logits), for configs whose
    logits rows would make the fixture large."""
    d = model_dir(name)
    cfg = lz98_synth.CONFIGS[name]
    sha = lz98_synth.write_model(cfg, d)
    n_prompt, max_new, runs = TOKEN_CASES[name]
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, cfg.vocab, n_prompt).astype(np.int32)
    R = Reference(d, 512, 4)
    out = {"sha256": np.frombuffer(bytes.fromhex(sha), np.uint8), "prompt": prompt,
           "runs": np.array(runs, np.float64), "max_new": np.array([max_new], np.int32)}
    for j, (k, temp) in enumerate(runs):
        toks, rounds = R.generate(prompt, max_new, k, temp=temp, seed=1234)
        out[f"run{j}_tokens"], out[f"run{j}_rounds"] = toks, rounds
    R.close()
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))


def b32_pick(prompts):
    """The four pinned batch-32 sequences: shortest, longest, then the
    first two others."""
    lens = [len(p) for p in prompts]
    pick = [int(np.argmin(lens)), int(np.argmax(lens))]
    for b in range(len(prompts)):
        if len(pick) == 4:
            break
        if b not in pick:
            pick.append(b)
    return pick


def _bench_job(job):
    kind, idx = job
    d = model_dir("0p5b")
    if kind == "b1":
        sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
        import bench
        prompt = bench.prompts(1, 0)[0]
        R = Reference(d, len(prompt) + BENCH_B1_NEW + 64, 4)
        toks, rounds = R.generate(prompt, BENCH_B1_NEW, 2)
    else:
        cfg = lz98_synth.CONFIGS["0p5b"]
        prompt = np.array(lz98_synth.workload_prompts(cfg, BENCH_B32_SEQS, 256, 1024, 1.1, seed=0)[idx], np.int32)
        R = Reference(d, len(prompt) + BENCH_B32_NEW + 64, 4)
        toks, rounds = R.generate(prompt, BENCH_B32_NEW, 3, temp=0.8, topp=0.95, seed=1000 + idx)
    R.close()
    return kind, idx, np.asarray(prompt, np.int32), toks, rounds


def make_bench():
    """tests/golden/0p5b_bench.npz: the reference's token streams and round
    records on the benchmarked workloads (one reference process per
    sequence)."""
    import multiprocessing as mp
    d = model_dir("0p5b")
    sha = lz98_synth.write_model(lz98_synth.CONFIGS["0p5b"], d)
    cfg = lz98_synth.CONFIGS["0p5b"]
    pick = b32_pick(lz98_synth.workload_prompts(cfg, BENCH_B32_SEQS, 256, 1024, 1.1, seed=0))
    jobs = [("b1", 0)] + [("b32", b) for b in pick]
    with mp.get_context("spawn").Pool(len(jobs)) as pool:
        res = pool.map(_bench_job, jobs)
    out = {"sha256": np.frombuffer(bytes.fromhex(sha), np.uint8), "b32_pick": np.array(pick, np.int32),
           "b1_max_new": np.array([BENCH_B1_NEW], np.int32), "b32_max_new": np.array([BENCH_B32_NEW], np.int32)}
    for kind, idx, prompt, toks, rounds in res:
        tag = "b1" if kind == "b1" else f"b32_{idx}"
        out[tag + "_prompt"], out[tag + "_tokens"], out[tag + "_rounds"] = prompt, toks, rounds
    path = os.path.join(HERE, "0p5b_bench.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))


def make_3b_long():
    """tests/golden/3b_long.npz (about an hour of reference prefill)."""
    d = model_dir("3b")
    cfg = lz98_synth.CONFIGS["3b"]
    sha = lz98_synth.write_model(cfg, d)
    prompt = lz98_synth.uniform_prompts(cfg, 8, LONG_3B_PROMPT)[0]
    R = Reference(d, LONG_3B_PROMPT + LONG_3B_NEW + 64, 4)
    toks, rounds = R.generate(prompt, LONG_3B_NEW, 3)
    out = {"sha256": np.frombuffer(bytes.fromhex(sha), np.uint8), "prompt_len": np.array([LONG_3B_PROMPT], np.int32),
           "max_new": np.array([LONG_3B_NEW], np.int32), "tokens": toks, "rounds": rounds,
           "prefill_ms": np.array([R.last_prefill_ms])}
    R.close()
    path = os.path.join(HERE, "3b_long.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))


def make_debug():
    """tests/golden/round_debug.npz: generations of the reference with its
    rounds' debug_break_rollback / debug_skip_catchup switches on (the
    prompt of each model's own fixture, seed 1234, top-p 0.95)."""
    out = {"cases": np.array([(k, t, br, sc) for _, k, t, br, sc in DEBUG_CASES], np.float64),
           "models": np.array([m for m, *_ in DEBUG_CASES])}
    for j, (name, k, temp, br, sc) in enumerate(DEBUG_CASES):
        d = model_dir(name)
        g = np.load(os.path.join(HERE, f"{name}.npz"))
        R = Reference(d, 512, 4)
        R.round_debug(br, sc)
        toks, rounds = R.generate(g["prompt"], CASES[name][3], k, temp=temp, seed=1234)
        R.round_debug(0, 0)
        R.close()
        out[f"c{j}_prompt"], out[f"c{j}_tokens"], out[f"c{j}_rounds"] = g["prompt"], toks, rounds
    path = os.path.join(HERE, "round_debug.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    for n in (sys.argv[1:] or list(CASES) + list(TOKEN_CASES) + ["bench", "debug"]):
        if n == "bench":
            make_bench()
        elif n == "debug":
            make_debug()
        elif n == "3b_long":
            make_3b_long()
        elif n in TOKEN_CASES:
            make_tokens(n)
        else:
            make(n)
