"""Synthetic KunMoe model writer: random-init weights in the "L98Z" model.bin
format that the reference engine's loader reads.

The reference ships no exporter (its tools/export_q8.py is cited but absent),
so this module writes the file from the loader's side of the contract:

* header words in the exact order ``lz_open_bin`` reads them
  (src/model.c:3993-4340: 28 fixed words, layer_types[128], the 13-word
  KDA/MoE tail, then the v5 tail up to csa2_compress_m_layer[128]);
* tensors in ``model_walk`` order (src/model.c:2240-2630): embed_tokens,
  final norm, then per layer the LAYER_SPECS rows that apply to a KDA +
  latent-MoE layer (src/model.c:1496-1665), then every expert's w1/w2/w3,
  then the MTP block (attention rows of LAYER_SPECS, its dense FFN, then
  fc/norm/pre_fc_norm_hidden/pre_fc_norm_embedding);
* each tensor as ``{dtype u8, n u32, [gs u32], data, [f32 scales]}``
  (src/model.c:3567-3804); scale layouts 1 and 2 with a v6 header
  (src/model.c:3510-3556, 4352-4410).

Weights are N(0, 0.02), rounded to bf16, then quantised to Q8_0 with the
activation quantiser's rule (scale = amax * (1/127), q = rne(x * 127/amax)
clamped to +-127; src/ops_quant.c:1633-1666 and 2152-2282).  1-D and 3-D
tensors are written as F32 holding bf16-rounded values.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import struct

import numpy as np

LZ_MAX_LAYERS = 128
LT_KDA = 2
FMT_F32 = 0
FMT_Q8_0 = 1


@dataclasses.dataclass(frozen=True)
class KunMoeConfig:
    """Architecture of one synthetic KunMoe model (all layers KDA + latent MoE,
    one MTP block with gated full attention and a dense SwiGLU FFN)."""
    name: str
    hidden: int
    n_layers: int
    kda_heads: int
    vocab: int
    n_experts: int
    top_k: int
    latent: int
    moe_ffn: int
    shared_width: int
    seq_len: int
    gs_mode: str = "row"          # "row": one scale per weight row; "32": Q8_0 gs=32
    head_dim: int = 64
    kda_head_dim: int = 64
    conv_kernel: int = 4
    gate_rank: int = 64
    gate_lower_bound: float = -5.0
    rms_eps: float = 1e-6
    rope_theta: float = 10000000.0
    partial_rotary: float = 0.25
    seed: int = 0
    scale_layout: int = 0         # Q8_0 scale planes: 0 f32, 1 binary16, 2 binary16 row base + u8 (v6 header)

    @property
    def n_heads(self) -> int:
        return self.hidden // self.head_dim

    @property
    def n_kv_heads(self) -> int:
        return max(1, self.n_heads // 4)

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)

    @property
    def key_dim(self) -> int:
        return self.kda_heads * self.kda_head_dim

    @property
    def mtp_ffn(self) -> int:
        return self.moe_ffn

    def gs(self, in_dim: int) -> int:
        return in_dim if self.gs_mode == "row" else 32

    def to_json(self) -> dict:
        d = dataclasses.asdict(self)
        d["n_heads"] = self.n_heads
        d["n_kv_heads"] = self.n_kv_heads
        d["rotary_dim"] = self.rotary_dim
        return d


# The BASELINE configurations this path is measured on (weights seed = config
# index).  "tiny" is the reference's CPU-runnable case; "0p5b" is the ~0.5B
# model of the batch-1 and batch-32 workloads; "3b" the ~3B model of the
# 8 x 8192-token chunked-prefill workload.
CONFIGS = {
    "tiny": KunMoeConfig(name="tiny", hidden=256, n_layers=4, kda_heads=4,
                         vocab=8192, n_experts=8, top_k=2, latent=128,
                         moe_ffn=512, shared_width=0, seq_len=512,
                         gs_mode="32", seed=0),
    "0p5b": KunMoeConfig(name="0p5b", hidden=1024, n_layers=24, kda_heads=16,
                         vocab=64000, n_experts=64, top_k=4, latent=512,
                         moe_ffn=1024, shared_width=1024, seq_len=2048,
                         gs_mode="row", seed=1),
    # the ~3B model (no shared expert; the context covers the
    # workload's 8192-token prompts plus the new tokens).
    "3b": KunMoeConfig(name="3b", hidden=2048, n_layers=32, kda_heads=32,
                       vocab=128000, n_experts=128, top_k=8, latent=768,
                       moe_ffn=1536, shared_width=0, seq_len=16384,
                       gs_mode="row", seed=3),
    # Small shapes of the 0p5b family for fast parity tests.
    "mini": KunMoeConfig(name="mini", hidden=128, n_layers=2, kda_heads=2,
                         vocab=1024, n_experts=8, top_k=4, latent=64,
                         moe_ffn=128, shared_width=128, seq_len=256,
                         gs_mode="row", seed=7),
    # Per-row scales with every matmul width a multiple of 128: the shapes
    # that reach the TMA-staged dense and grouped-expert kernels.
    "midi": KunMoeConfig(name="midi", hidden=256, n_layers=2, kda_heads=4,
                         vocab=2048, n_experts=16, top_k=4, latent=128,
                         moe_ffn=256, shared_width=256, seq_len=256,
                         gs_mode="row", seed=11),
    # The v6 scale layouts: binary16 scales (per row) and binary16 row base
    # + u8 codes (per 32).
    "midi_f16": KunMoeConfig(name="midi_f16", hidden=256, n_layers=2, kda_heads=4,
                             vocab=2048, n_experts=16, top_k=4, latent=128,
                             moe_ffn=256, shared_width=256, seq_len=256,
                             gs_mode="row", seed=13, scale_layout=1),
    "tiny_u8": KunMoeConfig(name="tiny_u8", hidden=256, n_layers=2, kda_heads=4,
                            vocab=4096, n_experts=8, top_k=2, latent=128,
                            moe_ffn=512, shared_width=0, seq_len=512,
                            gs_mode="32", seed=17, scale_layout=2),
}


def _bf16_round(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def quantize_q8_rows(w: np.ndarray, gs: int):
    """Q8_0 with the engine's absmax/127 rule; returns (int8 data, f32 scales)."""
    flat = w.astype(np.float32).reshape(-1, gs)
    amax = np.abs(flat).max(axis=1)
    inv127 = np.float32(1.0) / np.float32(127.0)
    scale = (amax * inv127).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(127.0) / amax, np.float32(0.0)).astype(np.float32)
    small = scale < np.float32(1e-30)
    scale = np.where(small | (amax <= 0), np.float32(1.0), scale).astype(np.float32)
    inv = np.where(small, np.float32(0.0), inv).astype(np.float32)
    q = np.rint(flat * inv[:, None]).clip(-127, 127).astype(np.int8)
    return q.reshape(-1), scale


def header_words(cfg: KunMoeConfig) -> bytes:
    c = cfg
    w = []
    i32 = lambda v: w.append(struct.pack("<i", int(v)))
    f32 = lambda v: w.append(struct.pack("<f", float(v)))
    q_dim = c.n_heads * c.head_dim
    kv_dim = c.n_kv_heads * c.head_dim
    kdim = c.key_dim
    # 28 fixed words (src/model.c:4022-4040)
    i32(c.vocab); i32(c.hidden); i32(c.n_layers); i32(c.seq_len)
    i32(c.n_heads); i32(c.n_kv_heads); i32(c.head_dim); i32(c.moe_ffn)
    i32(c.kda_heads); i32(c.kda_heads); i32(c.kda_head_dim); i32(c.kda_head_dim)
    i32(c.conv_kernel); i32(c.n_layers); i32(0); i32(0)
    i32(1); i32(1)
    f32(c.rms_eps); f32(c.rope_theta); f32(c.partial_rotary)
    i32(q_dim); i32(2 * q_dim); i32(kv_dim)
    i32(kdim); i32(kdim); i32(3 * kdim)
    i32(c.rotary_dim)
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS,
                         *([LT_KDA] * c.n_layers + [0] * (LZ_MAX_LAYERS - c.n_layers))))
    # KDA / MoE tail (src/model.c:4082-4094)
    i32(c.gate_rank); i32(1); f32(c.gate_lower_bound)
    i32(c.n_experts); i32(c.top_k); i32(1 if c.shared_width else 0)
    i32(c.moe_ffn); i32(c.latent); i32(0)
    i32(1); i32(1); i32(0); i32(c.shared_width)
    # v5 tail (src/model.c:4106-4301)
    i32(1); i32(c.mtp_ffn)                      # mtp_n_layers, mtp_intermediate_size
    i32(0); f32(1.0); f32(4096.0); f32(32.0); f32(1.0)   # rope scaling off
    i32(0); i32(0); i32(0)                      # use_subn, hadamard_o, hadamard_down
    i32(0); i32(0); i32(0)                      # mla q/o rank, attn_kv_share
    i32(0); i32(0); i32(0); i32(0)              # sink, gated_residual, ced_split, ced_kv
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS, *([0] * LZ_MAX_LAYERS)))      # csa2_on
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS, *([0] * LZ_MAX_LAYERS)))      # csa2_mode
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS, *([-1] * LZ_MAX_LAYERS)))     # csa2_source
    i32(0); i32(4); i32(64); i32(1); i32(64); i32(64)  # replay_w, compress_m, topk, idx heads/dim/rank
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS, *([0] * LZ_MAX_LAYERS)))      # csa2_compress_m_layer
    if not c.scale_layout:
        return b"L98Z" + struct.pack("<I", 5) + b"".join(w)
    # v6 words (src/model.c:4352-4410): the identity layer schedule, one
    # MTP draft, no embedding rotation, then the scale layout
    i32(c.n_layers)
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS, *(list(range(c.n_layers)) + [0] * (LZ_MAX_LAYERS - c.n_layers))))
    w.append(struct.pack("<%di" % LZ_MAX_LAYERS, *([0] * LZ_MAX_LAYERS)))
    i32(1); i32(0); i32(0); i32(c.scale_layout)
    return b"L98Z" + struct.pack("<I", 6) + b"".join(w)


def scale_plane_bytes(cfg: KunMoeConfig, ng: int, rows: int) -> int:
    """Bytes of one Q8_0 tensor's scale plane under the config's layout
    (src/model.c:3510-3556)."""
    return {0: 4 * ng, 1: 2 * ng, 2: 2 * rows + ng}[cfg.scale_layout]


def encode_scales(cfg: KunMoeConfig, scale: np.ndarray, rows: int):
    """The stored scale plane and the f32 scales the engines decode from it:
    layout 1 binary16 (round to nearest even); layout 2 a binary16 base per
    row (the row's largest scale) and a u8 code per group, decoded as
    base * (code / 255) with each step rounded to f32."""
    if cfg.scale_layout == 0:
        return scale.astype("<f4").tobytes(), scale
    if cfg.scale_layout == 1:
        h = scale.astype(np.float16)
        return h.astype("<f2").tobytes(), h.astype(np.float32)
    gpr = scale.size // rows
    s2 = scale.reshape(rows, gpr)
    base = s2.max(axis=1).astype(np.float16)
    b32 = base.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        code = np.where(b32[:, None] > 0, np.rint(s2 / b32[:, None] * np.float32(255.0)), 0.0)
    code = code.clip(0, 255).astype(np.uint8)
    dec = (b32[:, None] * (code.astype(np.float32) / np.float32(255.0)).astype(np.float32)).astype(np.float32)
    return base.astype("<f2").tobytes() + code.tobytes(), dec.reshape(-1)


def tensor_specs(cfg: KunMoeConfig):
    """Every tensor of the file in model_walk order: (kind, shape, std,
    offset) with kind "q8" (shape = (out, in)) or "f32"."""
    c = cfg
    kdim = c.key_dim
    q_dim = c.n_heads * c.head_dim
    kv_dim = c.n_kv_heads * c.head_dim
    specs = []
    q8 = lambda o, i: specs.append(("q8", (o, i), 0.02, 0.0))
    f32 = lambda shape, std=0.02, off=0.0: specs.append(("f32", shape, std, off))
    q8(c.vocab, c.hidden)                          # embed_tokens (tied lm_head)
    f32((c.hidden,))                               # final norm
    for _ in range(c.n_layers):
        f32((c.hidden,)); f32((c.hidden,))         # input / post_attention layernorm
        q8(kdim, c.hidden); q8(kdim, c.hidden); q8(kdim, c.hidden)     # q, k, v proj
        for _c in range(3):
            f32((kdim, 1, c.conv_kernel), std=0.2) # q/k/v conv1d
        f32((c.kda_heads,))                        # A_log
        q8(c.gate_rank, c.hidden)                  # f_a_proj
        q8(kdim, c.gate_rank)                      # f_b_proj
        f32((kdim,))                               # dt_bias
        q8(c.kda_heads, c.hidden)                  # b_proj
        q8(kdim, c.hidden)                         # g_proj
        f32((c.kda_head_dim,), off=1.0)            # o_norm (multiplies directly)
        q8(c.hidden, kdim)                         # o_proj
        q8(c.n_experts, c.hidden)                  # router
        f32((c.n_experts,))                        # e_score_correction_bias
        q8(c.latent, c.hidden)                     # routed_expert_down_proj
        q8(c.hidden, c.latent)                     # routed_expert_up_proj
        if c.shared_width:
            q8(c.shared_width, c.hidden); q8(c.shared_width, c.hidden)   # shared gate / up
            q8(c.hidden, c.shared_width)           # shared down
        for _e in range(c.n_experts):
            q8(c.moe_ffn, c.latent); q8(c.latent, c.moe_ffn); q8(c.moe_ffn, c.latent)  # w1, w2, w3
    f32((c.hidden,)); f32((c.hidden,))             # MTP input / post_attention layernorm
    q8(2 * q_dim, c.hidden)                        # q_proj (q | gate interleaved per head)
    q8(kv_dim, c.hidden); q8(kv_dim, c.hidden)     # k_proj, v_proj
    q8(c.hidden, q_dim)                            # o_proj
    f32((c.head_dim,)); f32((c.head_dim,))         # q_norm, k_norm
    q8(c.mtp_ffn, c.hidden); q8(c.mtp_ffn, c.hidden)   # mlp gate / up
    q8(c.hidden, c.mtp_ffn)                        # mlp down
    q8(c.hidden, 2 * c.hidden)                     # fc
    f32((c.hidden,)); f32((c.hidden,)); f32((c.hidden,))   # norm, pre_fc_norm_hidden/embedding
    out, off = [], len(header_words(cfg))
    for kind, shape, std, o in specs:
        n = int(np.prod(shape))
        size = 5 + 4 * n if kind == "f32" else 9 + n + scale_plane_bytes(cfg, n // cfg.gs(shape[1]), shape[0])
        out.append((kind, shape, std, o, off))
        off += size
    return out, off


def _tensor_bytes(cfg: KunMoeConfig, idx: int, spec) -> bytes:
    kind, shape, std, o, _ = spec
    n = int(np.prod(shape))
    rng = np.random.default_rng([cfg.seed, idx + 1])
    x = rng.standard_normal(n, dtype=np.float32) * np.float32(std)
    if o:
        x = x + np.float32(o)
    x = _bf16_round(x)
    if kind == "f32":
        return struct.pack("<BI", FMT_F32, n) + x.astype("<f4").tobytes()
    gs = cfg.gs(shape[1])
    q, s = quantize_q8_rows(x, gs)
    if cfg.scale_layout:
        # quantise against the scales the engines will decode
        plane, dec = encode_scales(cfg, s, shape[0])
        flat = x.astype(np.float32).reshape(-1, gs)
        with np.errstate(divide="ignore", invalid="ignore"):
            qq = np.where(dec[:, None] > 0, np.rint(flat / dec[:, None]), 0.0)
        q = qq.clip(-127, 127).astype(np.int8).reshape(-1)
        return struct.pack("<BII", FMT_Q8_0, n, gs) + q.tobytes() + plane
    return struct.pack("<BII", FMT_Q8_0, n, gs) + q.tobytes() + s.astype("<f4").tobytes()


def _write_range(args):
    cfg, path, lo, hi = args
    specs, _ = tensor_specs(cfg)
    fd = os.open(path, os.O_WRONLY)
    try:
        for i in range(lo, hi):
            b = _tensor_bytes(cfg, i, specs[i])
            os.pwrite(fd, b, specs[i][4])
    finally:
        os.close(fd)
    return hi - lo


def write_model(cfg: KunMoeConfig, out_dir: str, workers: int | None = None) -> str:
    """Write ``out_dir/model.bin`` (and lz98_synth.json describing it);
    returns the sha256 of the whole file.  Tensor i draws from
    default_rng([seed, i + 1]), so the bytes do not depend on how many
    worker processes share the work.  Idempotent: an existing file whose
    recorded config matches is kept."""
    os.makedirs(out_dir, exist_ok=True)
    meta_path = os.path.join(out_dir, "lz98_synth.json")
    bin_path = os.path.join(out_dir, "model.bin")
    want = cfg.to_json()
    if os.path.exists(meta_path) and os.path.exists(bin_path):
        try:
            with open(meta_path) as f:
                have = json.load(f)
            if have.get("config") == want and os.path.getsize(bin_path) == have.get("bytes"):
                return have["sha256"]
        except (OSError, ValueError, KeyError):
            pass
    specs, total = tensor_specs(cfg)
    tmp = bin_path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header_words(cfg))
        f.truncate(total)
    if workers is None:
        workers = min(32, os.cpu_count() or 1) if total > (64 << 20) else 1
    import sys
    main = sys.modules.get("__main__")
    if workers > 1 and not os.path.isfile(getattr(main, "__file__", "") or ""):
        workers = 1          # spawned workers re-import __main__ from its file
    if workers <= 1:
        _write_range((cfg, tmp, 0, len(specs)))
    else:
        import multiprocessing as mp
        step = max(1, len(specs) // (workers * 4))
        jobs = [(cfg, tmp, i, min(len(specs), i + step)) for i in range(0, len(specs), step)]
        with mp.get_context("spawn").Pool(workers) as pool:
            pool.map(_write_range, jobs)
    h = hashlib.sha256()
    with open(tmp, "rb") as f:
        for blk in iter(lambda: f.read(1 << 24), b""):
            h.update(blk)
    sha = h.hexdigest()
    os.replace(tmp, bin_path)
    with open(meta_path, "w") as f:
        json.dump({"config": want, "sha256": sha, "bytes": total}, f, indent=1)
    return sha


def workload_prompts(cfg: KunMoeConfig, n_seq: int, lo: int, hi: int,
                     zipf: float | None, seed: int = 0):
    """Seeded synthetic prompts: lengths U[lo, hi], ids uniform or Zipf(s)
    over the vocabulary (per-sequence seed = 1000 + seq for Zipf)."""
    prompts = []
    for s in range(n_seq):
        rng = np.random.default_rng([seed, 1000 + s])
        n = int(rng.integers(lo, hi + 1)) if hi > lo else lo
        if zipf is None:
            ids = rng.integers(0, cfg.vocab, size=n)
        else:
            ids = (rng.zipf(zipf, size=n) - 1) % cfg.vocab
        prompts.append([int(x) for x in ids])
    return prompts


def uniform_prompts(cfg: KunMoeConfig, n_seq: int, length: int, rank: int = 0):
    """The configs[3] workload's prompts: n_seq prompts of `length` token
    ids uniform over the vocabulary, sequence s of rank r drawn from
    default_rng([cfg.seed, 1000 + 100000 r + s])."""
    out = []
    for s in range(n_seq):
        rng = np.random.default_rng([cfg.seed, 1000 + 100000 * rank + s])
        out.append(rng.integers(0, cfg.vocab, length).astype(np.int32))
    return out
