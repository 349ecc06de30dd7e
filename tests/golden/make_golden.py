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
}


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


if __name__ == "__main__":
    for n in (sys.argv[1:] or list(CASES) + list(TOKEN_CASES)):
        make_tokens(n) if n in TOKEN_CASES else make(n)
