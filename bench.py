#!/usr/bin/env python
"""Benchmark of the MTP speculative-decoding step (accepted tokens/s).

Workload: the ~0.5B random-init KunMoe (d 1024, 24
KDA+latent-MoE layers, 16 KDA heads, 64 experts top-4 + shared, latent 512,
FFN 1024, vocab 64000, per-row weight scales), one sequence per GPU, a
512-token uniform-random prompt, greedy decoding, draft depth k = 2.

One step = one speculative round of every sequence on the GPU: k MTP draft
steps, one (k+1)-row verify forward through the int8 body, acceptance,
KDA ring rollback, draft-chain reseed and MTP catch-up.  The timed region
replays K rounds (CUDA graph) on the library's stream, bracketed by a
barrier and device synchronisation, timed with CUDA events; the value is
emitted tokens (n_accept + 1 per round per sequence) of all ranks over
the slowest rank's time.  The round's weight stream (about 0.95 GB) is far
larger than L2, so no explicit flush is used.

The same line carries "batch32": BASELINE configs[2] (32 sequences per GPU,
Zipf prompts of 256-1024 tokens, temperature 0.8, top-p 0.95, k = 3),
measured the same way after the headline workload (--no-b32 skips it).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference runs the reference engine itself (oracle/_ref, compiled
from the reference sources, single-threaded C99) on this host's CPU over a
bounded sample of the same workload and prints the same JSON line."""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "llama98-zh_b200")
sys.path.insert(0, PKG)

METRIC = "accepted tokens/s"
UNIT = "tokens/s"
MODEL = "0p5b"
PROMPT = 512
MAX_NEW = 256
SPEC_K = 2


def model_dir(name: str = MODEL) -> str:
    import lz98_synth
    d = os.path.join(os.environ.get("LZ98_MODEL_DIR", os.path.join(tempfile.gettempdir(), "lz98_models")), name)
    lz98_synth.write_model(lz98_synth.CONFIGS[name], d)
    return d


def prompts(n_seq: int, rank: int):
    import numpy as np
    import lz98_synth
    cfg = lz98_synth.CONFIGS[MODEL]
    out = []
    for s in range(n_seq):
        rng = np.random.default_rng([0, 1000 + rank * 100000 + s])
        out.append(rng.integers(0, cfg.vocab, PROMPT).astype(np.int32))
    return out


def round_bytes(m, R: int, k: int, n_seq: int) -> float:
    """Algorithmic HBM bytes of one round (weights touched once, state
    traffic): verify body over R rows, lm_head, k draft steps, KDA state."""
    d, L, V = m.hidden, m.n_layers, m.vocab
    kdim = m.key_dim
    nvk = kdim
    n_in = 4 * kdim + 64 + m.kda_heads
    per_layer = (n_in * d + nvk * 64 + d * kdim + (m.n_experts + m.latent + 2 * m.shared_w) * d +
                 d * m.latent + d * m.shared_w)
    e_touched = m.n_experts * (1.0 - (1.0 - m.top_k / m.n_experts) ** R)
    per_layer += e_touched * 3 * m.latent * m.moe_ffn
    verify = L * per_layer + V * d
    qd = m.n_heads * m.head_dim
    kvd = m.n_kv_heads * m.head_dim
    draft = d * 2 * d + (2 * qd + 2 * kvd) * d + d * qd + 3 * m.mtp_ffn * d + V * d
    state = n_seq * L * m.kda_heads * 64 * 64 * (2 + 4 / 32) * (1 + (k + 1))
    return verify + k * draft + state


class Clocks:
    """SM clock and clock-event reasons sampled during the timed region:
    NVML read every 2 ms from a thread (reads only; no setting is
    changed), else nvidia-smi at its shortest period."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int, uuid: str | None = None):
        import threading
        self.sm, self.smax, self.reasons, self.p = [], None, set(), None
        self.stop_ev = threading.Event()
        self.thread = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            h = None
            if uuid:
                try:
                    h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
                except nv.NVMLError:
                    h = None
            self.h = h if h is not None else nv.nvmlDeviceGetHandleByIndex(gpu_index)
            self.smax = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                         "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                         "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                         "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nv = None
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "50", "-i", str(gpu_index)], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.p = None

    def _loop(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for n, bit in self.bits.items():
                    if r & bit:
                        self.reasons.add(n)
            except Exception:
                pass
            time.sleep(0.002)

    def stop(self):
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
            if not self.sm:
                return {"sm_mhz": None, "sm_max_mhz": self.smax, "reasons": [], "source": "nvml"}
            return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.smax,
                    "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml, 2 ms"}
        res = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if not self.p:
            return res
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(self.NAMES, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if sm:
            res = {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                   "samples": len(sm), "source": "nvidia-smi, 50 ms"}
        return res


def gpu_uuid(local: int):
    try:
        import torch
        return str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        return None


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def reduce_over_ranks(ms: float, emitted: float, e2e, world: int, device: str):
    """Whole-job figures: the slowest rank's device time (MAX) and the
    tokens of all ranks (SUM); every rank takes the same two collectives."""
    if world <= 1:
        return ms, emitted, e2e
    import torch
    import torch.distributed as dist
    mx = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    sm = torch.tensor([emitted, e2e or 0.0], dtype=torch.float64, device=device)
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx[0]), float(sm[0]), (float(sm[1]) if e2e is not None else None)


GEMV_TRAFFIC_RATIO = 1.045   # ncu dram bytes / algorithmic bytes of the int8 GEMV
# ncu DRAM bytes / algorithmic bytes of the grouped-expert kernels at batch
# 32 (w1/w3: 68.65 MB for 67.6 MB, w2: 34.30 MB for 33.7 MB per launch)
EXPERT_TRAFFIC_RATIO = 1.016
B32 = 32          # configs[2]: sequences per GPU
K32 = 3
NEW32 = 512


def _expert_roofline(prof):
    peak, peak_kind = measured_peak()
    if not prof.get("n_expert"):
        return None
    achieved = prof["expert_bytes"] / (prof["expert_ms"] * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": "moe_tma_kernel (grouped experts w1/w3 and w2, all launches of one round)",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
            "traffic": prof["expert_bytes"] * EXPERT_TRAFFIC_RATIO,
            "traffic_unit": "bytes per round (all grouped-expert launches)",
            "launches": prof["n_expert"], "ms_per_round": prof["expert_ms"]}


def run_batch32(m, args, rank: int, world: int):
    """BASELINE configs[2] on this rank: 32 independent sequences, prompts of
    256-1024 Zipf(1.1) token ids, temperature 0.8, top-p 0.95, per-sequence
    seeds, draft depth 3.  Device-timed rounds (CUDA graph replay), then an
    end-to-end pass through lz_spec_round_batch that reads every round's
    tokens back to the host.  Every rank takes the same collectives."""
    import torch
    import torch.distributed as dist
    import lz98
    import lz98_synth
    cfg = lz98_synth.CONFIGS[MODEL]
    lo, hi = args.b32_prompts                 # 256-1024 for the workload; shorter only to profile
    prompts = lz98_synth.workload_prompts(cfg, B32, lo, hi, 1.1, seed=rank)
    e2e_steps = 8
    steps = max(1, min(args.steps, NEW32 // (K32 + 1) - args.warmup - e2e_steps - 2))
    seq_len = 1024 + (K32 + 1) * (args.warmup + steps + e2e_steps + 2) + 64
    s = lz98.State(m, seq_len, K32, n_seq=B32)
    t0 = time.time()
    for b, p in enumerate(prompts):
        s.set_sampler(b, 0.8, 0.95, 1000 + rank * B32 + b)
        s.seq_prefill(b, p)
    prefill_s = time.time() - t0
    print(f"[bench] b32_prefill_launches={s.launches()}", file=sys.stderr, flush=True)
    stream = torch.cuda.ExternalStream(s.stream())
    for _ in range(args.warmup):
        s.round_batch(K32, fetch=False)
    torch.cuda.synchronize()
    c0 = [s.counters(b) for b in range(B32)]
    local = torch.cuda.current_device()
    clocks = Clocks(physical_gpu(local), gpu_uuid(local))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        s.round_batch(K32, fetch=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    c1 = [s.counters(b) for b in range(B32)]
    emitted = sum(c1[b][1] - c0[b][1] for b in range(B32))
    accepted = sum(c1[b][2] - c0[b][2] for b in range(B32))
    drafted = sum(c1[b][3] - c0[b][3] for b in range(B32))
    rounds = sum(c1[b][0] - c0[b][0] for b in range(B32))
    # end to end: the public batched round with the tokens read back
    torch.cuda.synchronize()
    t_e = time.perf_counter()
    n_e = 0
    for _ in range(e2e_steps):
        toks, cnt = s.round_batch(K32, fetch=True)
        n_e += int(cnt.sum())
    dt_e = time.perf_counter() - t_e
    prof = s.profile_round(K32)
    s.close()
    ms_max, emitted_all, e2e_all = reduce_over_ranks(ms, float(emitted), n_e / dt_e, world, "cuda")
    return {
        "workload": f"configs[2]: ~0.5B KunMoe, 32 sequences per GPU, prompts {lo}-{hi} Zipf(1.1), "
                    "temperature 0.8, top-p 0.95, k=3",
        "value": emitted_all / (ms_max * 1e-3), "unit": UNIT, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms_max / steps, "global_batch": B32 * world, "scaling": "weak",
        "mean_accept_len": (accepted + rounds) / max(1, rounds), "alpha": accepted / max(1, drafted),
        "prefill_s": prefill_s,
        "e2e": {"value": e2e_all, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": B32 * (K32 + 1) * 4 + B32 * 4,
                "api": "lz_spec_round_batch (round state device-resident, tokens and counts read back)"},
        "gemm_ms_per_round": prof["gemv_ms"], "round_ms_eager": prof["round_ms"],
        "gemm_algorithmic_gbs": prof["gemv_bytes"] / (prof["gemv_ms"] * 1e-3) / 1e9,
        # the workload's HBM-bound kernels: every grouped-expert launch of
        # one eager round, event-timed one by one on the state's stream
        "roofline": _expert_roofline(prof),
        "gpu_launches": prof["n_kernels"] * steps,
        "clocks": clk,
    }


def run_ep(m, args, rank: int, world: int):
    """Expert parallelism at N > 1 (configs[2]'s batch-32 temperature
    rounds): each rank's 32 sequences are prefilled with its local experts,
    then lz_ep_init shards the routed experts over the ranks (rank r owns
    E/N of them) and every round exchanges each layer's (token, expert)
    pairs with NCCL send/recv; the rounds run eagerly (no graph).  Same
    prompts as the batch-32 arm.  Device-timed, max over ranks."""
    import torch
    import torch.distributed as dist
    import lz98
    import lz98_synth
    cfg = lz98_synth.CONFIGS[MODEL]
    lo, hi = args.b32_prompts
    prompts = lz98_synth.workload_prompts(cfg, B32, lo, hi, 1.1, seed=rank)
    steps = max(1, min(args.steps, 20))
    s = lz98.State(m, 1024 + (K32 + 1) * (args.warmup + steps + 2) + 64, K32, n_seq=B32)
    for b, p in enumerate(prompts):
        s.set_sampler(b, 0.8, 0.95, 1000 + rank * B32 + b)
        s.seq_prefill(b, p)
    obj = [lz98.ep_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    s.ep_init(obj[0], rank, world)
    stream = torch.cuda.ExternalStream(s.stream())
    for _ in range(args.warmup):
        s.round_batch(K32, fetch=False)
    torch.cuda.synchronize()
    c0 = [s.counters(b) for b in range(B32)]
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        s.round_batch(K32, fetch=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = ev0.elapsed_time(ev1)
    c1 = [s.counters(b) for b in range(B32)]
    emitted = sum(c1[b][1] - c0[b][1] for b in range(B32))
    s.close()
    ms_max, emitted_all, _ = reduce_over_ranks(ms, float(emitted), None, world, "cuda")
    return {"workload": "configs[2] rounds (32 sequences per GPU, temperature 0.8, top-p 0.95, k=3) with the "
                        f"64 routed experts sharded {cfg.n_experts // world} per rank",
            "value": emitted_all / (ms_max * 1e-3), "unit": UNIT, "steps": steps, "ms_per_step": ms_max / steps,
            "parallelism": f"ep{world} (NCCL send/recv of each layer's pairs; eager rounds)",
            "scaling": "weak"}


N3B, P3B, K3B, NEW3B = 8, 8192, 3, 256     # configs[3]: sequences per GPU, prompt, draft depth, new tokens


def run_3b(args):
    """BASELINE configs[3] (--config 3b): the ~3B model, 8 sequences per
    GPU with 8192-token uniform prompts prefilled in row-capacity chunks
    (device-timed: prefill tokens/s), then greedy k = 3 rounds of all 8
    (CUDA graph replay, device-timed), and an end-to-end pass through
    lz_spec_round_batch that reads the tokens back."""
    import torch
    import torch.distributed as dist
    import lz98
    import lz98_synth
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    cfg = lz98_synth.CONFIGS["3b"]
    if world > 1 and rank != 0:
        dist.barrier()
    d = model_dir("3b")
    if world > 1 and rank == 0:
        dist.barrier()
    m = lz98.Model(d)
    e2e_steps = 4
    steps = max(1, min(args.steps, NEW3B - args.warmup - e2e_steps - 2))
    s = lz98.State(m, P3B + (K3B + 1) * (args.warmup + steps + e2e_steps + 2) + 64, K3B, n_seq=N3B)
    prompts = lz98_synth.uniform_prompts(cfg, N3B, P3B, rank)
    stream = torch.cuda.ExternalStream(s.stream())
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    t0 = time.time()
    for b, p in enumerate(prompts):
        s.seq_prefill(b, p)
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_wall = time.time() - t0
    prefill_ms = p0.elapsed_time(p1)
    for _ in range(args.warmup):
        s.round_batch(K3B, fetch=False)
    torch.cuda.synchronize()
    c0 = [s.counters(b) for b in range(N3B)]
    clocks = Clocks(physical_gpu(local), gpu_uuid(local))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        s.round_batch(K3B, fetch=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    c1 = [s.counters(b) for b in range(N3B)]
    emitted = sum(c1[b][1] - c0[b][1] for b in range(N3B))
    accepted = sum(c1[b][2] - c0[b][2] for b in range(N3B))
    drafted = sum(c1[b][3] - c0[b][3] for b in range(N3B))
    rounds = sum(c1[b][0] - c0[b][0] for b in range(N3B))
    torch.cuda.synchronize()
    t_e = time.perf_counter()
    n_e = 0
    for _ in range(e2e_steps):
        toks, cnt = s.round_batch(K3B, fetch=True)
        n_e += int(cnt.sum())
    dt_e = time.perf_counter() - t_e
    prof = s.profile_round(K3B)
    rb = round_bytes(m, N3B * (K3B + 1), K3B, N3B)
    s.close()
    ms_max, emitted_all, e2e_all = reduce_over_ranks(ms, float(emitted), n_e / dt_e, world, "cuda")
    pf_max, pf_tok, _ = reduce_over_ranks(prefill_ms, float(N3B * P3B), None, world, "cuda")
    peak, peak_kind = measured_peak()
    if rank == 0:
        gemv_gbs = prof["gemv_bytes"] / (prof["gemv_ms"] * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": emitted_all / (ms_max * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": ms_max / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights/activations, int32 dot, f32 epilogue",
            "data": "synthetic: random-init weights N(0,0.02)->bf16->Q8_0, uniform prompt ids",
            "config": {"workload": "configs[3]: ~3B KunMoe, 8 sequences per GPU, 8192-token prompts "
                                   "(chunked prefill), greedy, k=3",
                       "model": "KunMoe-3B-synthetic", "global_batch": N3B * world, "seq_len": P3B,
                       "new_tokens_budget": NEW3B, "spec_k": K3B, "parallelism": f"dp{world} (replicas)",
                       "l2": "no flush: per-round weight stream >> 126 MB L2"},
            "prefill": {"tokens_per_s": pf_tok / (pf_max * 1e-3), "ms": pf_max, "wall_s": prefill_wall,
                        "tokens": pf_tok},
            "mean_accept_len": (accepted + rounds) / max(1, rounds), "alpha": accepted / max(1, drafted),
            "hbm_gbs_round": rb / (ms / steps * 1e-3) / 1e9,
            "roofline": _expert_roofline(prof) or {
                "bound": "hbm", "kernel": "gemv_q8_kernel", "achieved": gemv_gbs, "peak": peak, "unit": "GB/s",
                "frac": gemv_gbs / peak, "peak_kind": peak_kind, "traffic": None},
            "e2e": {"value": e2e_all, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": N3B * (K3B + 1) * 4 + N3B * 4,
                    "api": "lz_spec_round_batch (round state device-resident, tokens and counts read back)"},
            "gpu_launches": prof["n_kernels"] * steps, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    import lz98

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    n_seq = args.seqs
    k = SPEC_K
    d = model_dir() if rank == 0 or world == 1 else None
    if world > 1:
        dist.barrier()
        d = model_dir()
    m = lz98.Model(d)
    if args.b32_only:
        b32 = run_batch32(m, args, rank, world)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "n_gpus": world, "batch32": b32}), flush=True)
        m.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return b32
    seq_len = PROMPT + (k + 1) * (args.warmup + args.steps + 2) + 64
    s = lz98.State(m, seq_len, k, n_seq=n_seq)
    t0 = time.time()
    for b, p in enumerate(prompts(n_seq, rank)):
        s.seq_prefill(b, p)
    prefill_s = time.time() - t0
    print(f"[bench] prefill_launches={s.launches()}", file=sys.stderr, flush=True)
    stream = torch.cuda.ExternalStream(s.stream())
    for _ in range(args.warmup):
        s.round_batch(k, fetch=False)
    torch.cuda.synchronize()
    c0 = [s.counters(b) for b in range(n_seq)]
    clocks = Clocks(physical_gpu(local), gpu_uuid(local))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        s.round_batch(k, fetch=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    c1 = [s.counters(b) for b in range(n_seq)]
    emitted = sum(c1[b][1] - c0[b][1] for b in range(n_seq))
    accepted = sum(c1[b][2] - c0[b][2] for b in range(n_seq))
    drafted = sum(c1[b][3] - c0[b][3] for b in range(n_seq))
    rounds = sum(c1[b][0] - c0[b][0] for b in range(n_seq))
    # kernel timing pass (eager round with events around every GEMV)
    prof = s.profile_round(k)
    # end-to-end through the reference-facing C ABI with host buffers:
    # lz_spec_round (one sequence, host anchor in, host tokens out)
    e2e_val, h2d, d2h = None, 0, 0
    if n_seq == 1 and not args.no_e2e:
        s1 = lz98.State(m, seq_len, k, n_seq=1)
        anchor = s1.seq_prefill(0, prompts(1, rank)[0])
        pos = PROMPT
        for _ in range(args.warmup):
            out, na, npos, _ke = s1.spec_round(anchor, pos - 1, k)
            anchor, pos = int(out[na]), npos + 1
        torch.cuda.synchronize()
        t_e = time.perf_counter()
        n_e = 0
        for _ in range(args.steps):
            out, na, npos, _ke = s1.spec_round(anchor, pos - 1, k)
            anchor, pos = int(out[na]), npos + 1
            n_e += na + 1
        torch.cuda.synchronize()
        dt_e = time.perf_counter() - t_e
        e2e_val = n_e / dt_e
        sr_bytes = 112
        h2d, d2h = sr_bytes, 2 * sr_bytes
        s1.close()
    ms_max, emitted_all, e2e_all = reduce_over_ranks(ms, float(emitted), e2e_val, world, "cuda")
    b32 = None if args.no_b32 else run_batch32(m, args, rank, world)
    ep = run_ep(m, args, rank, world) if (world > 1 and not args.no_ep) else None
    peak, peak_kind = measured_peak()
    gemv_gbs = prof["gemv_bytes"] / (prof["gemv_ms"] * 1e-3) / 1e9
    line = None
    if rank == 0:
        cpu = cpu_baseline(args) if (world == 1 and not args.no_cpu) else None
        if b32 is not None and world == 1 and not args.no_cpu:
            b32["cpu_baseline"] = b32_cpu_baseline(args.b32_cpu_seconds, *args.b32_prompts)
        per_round_ms = ms / max(1, args.steps)
        rb = round_bytes(m, n_seq * (k + 1), k, n_seq)
        line = {
            "metric": METRIC, "value": emitted_all / (ms_max * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 weights/activations, int32 dot, f32 epilogue",
            "data": "synthetic: random-init weights N(0,0.02)->bf16->Q8_0, uniform prompt ids",
            "config": {"workload": "configs[1]: ~0.5B KunMoe, batch 1 per GPU, 512-token prompt, greedy, k=2",
                       "model": "KunMoe-0.5B-synthetic", "global_batch": n_seq * world, "seq_len": PROMPT,
                       "new_tokens_budget": MAX_NEW, "spec_k": k, "parallelism": f"dp{world} (replicas)",
                       "l2": "no flush: per-round weight stream ~0.95 GB >> 126 MB L2"},
            "mean_accept_len": (accepted + rounds) / max(1, rounds),
            "alpha": accepted / max(1, drafted),
            "prefill_s": prefill_s,
            "hbm_gbs_round": rb / (per_round_ms * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": "gemv_q8_kernel (int8 weight streaming, all GEMVs of one round)",
                         "achieved": gemv_gbs, "peak": peak, "unit": "GB/s", "frac": gemv_gbs / peak,
                         "peak_kind": peak_kind,
                         # DRAM bytes of the round's GEMV launches: the algorithmic
                         # bytes times the mean DRAM/algorithmic ratio of an ncu
                         # capture of three GEMV launches (1.03-1.06)
                         "traffic": prof["gemv_bytes"] * GEMV_TRAFFIC_RATIO,
                         "traffic_unit": "bytes per round (all GEMV launches)",
                         "gemv_share_of_round": prof["gemv_ms"] / max(1e-9, prof["round_ms"]),
                         "round_algorithmic_bytes": rb},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_all, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "lz_spec_round (host anchor in, host tokens out)"} if e2e_val else None,
            "gpu_launches": prof["n_kernels"] * args.steps,
            "clocks": clk,
            "batch32": b32,
            "expert_parallel": ep,
        }
        print(json.dumps(line), flush=True)
    s.close()
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


def host_cores() -> int:
    """Cores this process may use: its affinity mask, bounded by a cgroup
    CPU quota when one is set."""
    n = len(os.sched_getaffinity(0))
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            q, per = f.read().split()[:2]
        if q != "max":
            n = min(n, max(1, int(q) // int(per)))
    except (OSError, ValueError):
        pass
    return n


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def mem_available_bytes() -> float:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return float(line.split()[1]) * 1024.0
    except (OSError, ValueError):
        pass
    return 0.0


def _reference():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracles import Reference, reference_available
    return Reference, reference_available


def ref_decode_sample(prompt, k: int, temp: float, seed: int, max_new: int, seconds: float, stock_seconds: float = 0.0,
                      barrier=None):
    """The reference engine (oracle/_ref, one thread) on one sequence of the
    workload: the prompt prefilled (untimed), a short warm decode, then
    decode for about `seconds` in the parity float tier and, when
    stock_seconds > 0, for about stock_seconds more in the reference's
    stock tier (the tier is switched between rounds: the decode cost per
    token is what is timed).  A barrier (multiprocessing) is waited on
    before each timed phase.  Returns ((tokens/s, tokens, s) float,
    (tokens/s, tokens, s) stock or None, prefill s)."""
    Reference, available = _reference()
    if not available():
        return None
    R = Reference(model_dir(), len(prompt) + max_new + 64, max(1, k))
    try:
        pf = R.session_begin(prompt, max_new, k, temp=temp, topp=0.95, seed=seed)
        R.session_decode(k + 1)
        if barrier is not None:
            barrier.wait(timeout=1200)
        toks, _, el = R.session_decode(1 << 30, seconds * 1000.0)
        fl = (len(toks) / max(1e-9, el * 1e-3), len(toks), el * 1e-3)
        st = None
        if stock_seconds > 0:
            R.stock_tier()
            if barrier is not None:
                barrier.wait(timeout=1200)
            toks, _, el = R.session_decode(1 << 30, stock_seconds * 1000.0)
            st = (len(toks) / max(1e-9, el * 1e-3), len(toks), el * 1e-3)
    finally:
        R.L.rd_set_tier(7)
        R.close()
    return fl, st, pf * 1e-3


def cpu_baseline(args):
    """Batch-1 CPU baseline: the reference on the headline workload's own
    sequence (the 512-token prompt, greedy, k = 2), float tier, then its
    stock arithmetic on a shorter sample of the same decode."""
    p = prompts(1, 0)[0]
    r = ref_decode_sample(p, SPEC_K, 0.0, 1, MAX_NEW, args.cpu_seconds, max(2.0, args.cpu_seconds / 3))
    if r is None:
        return {"value": None, "unit": UNIT, "cores": 1, "kind": "reference",
                "sample": "oracle/_ref/liblz98ref.so not built"}
    (v, n, el), st, pf = r
    return {"value": v, "unit": UNIT, "cores": 1, "kind": "reference", "cpu": cpu_model(),
            "sample": f"reference C99 engine, float tier (--fixed off, --fastfp off), the bench's 512-token "
                      f"prompt (prefill {pf:.1f} s, untimed), then {n} greedy k=2 tokens in {el:.1f} s of decode",
            "stock_tier": {"value": st[0] if st else None,
                           "sample": f"stock tier (--fixed all, --fastfp on), the same decode continued, {st[1]} "
                                     f"tokens in {st[2]:.1f} s" if st else "not run"}}


def _b32_cpu_worker(prompt, seed, seconds, stock_seconds, barrier, out):
    try:
        r = ref_decode_sample(prompt, K32, 0.8, seed, NEW32, seconds, stock_seconds, barrier)
        (v, n, el), st, _ = r
        out.put((n, el, st[1] if st else 0, st[2] if st else 0.0, None))
    except Exception as e:          # reported, never hangs the parent
        try:
            barrier.abort()
        except Exception:
            pass
        out.put((0, 0.0, 0, 0.0, repr(e)[:200]))


def _collect(procs, q, barrier, n: int, limit_s: float):
    """Results of the worker processes; a worker that died without one
    breaks the barrier (the others report an error instead of waiting),
    and workers still running at the limit are terminated."""
    import queue
    outs, aborted, t_end = [], False, time.time() + limit_s
    while len(outs) < n and time.time() < t_end:
        try:
            outs.append(q.get(timeout=1.0))
            continue
        except queue.Empty:
            pass
        if not aborted and any(pr.exitcode not in (None, 0) for pr in procs):
            barrier.abort()
            aborted = True
        if all(pr.exitcode is not None for pr in procs) and q.empty():
            break
    for pr in procs:
        pr.join(timeout=30)
        if pr.exitcode is None:
            pr.terminate()
            pr.join(timeout=10)
    return outs


def b32_cpu_baseline(seconds: float, lo: int = 256, hi: int = 1024):
    """Batch-32 CPU baseline: one reference process per usable
    host core, each on its own sequence of the workload (the GPU arm's 32
    sequences of rank 0 first, then rank 1's, ...; their seeds), Zipf
    prompts prefilled untimed, temperature 0.8, top-p 0.95, k = 3.  All
    processes start decoding together (a barrier) and decode for about
    `seconds`; the value is the sum of their rates.  Float tier, then
    stock tier.  The process count is also bounded by host memory (each
    process holds the model)."""
    import multiprocessing as mp
    import lz98_synth
    Reference, available = _reference()
    if not available():
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": "oracle/_ref/liblz98ref.so not built"}
    cfg = lz98_synth.CONFIGS[MODEL]
    model_bytes = os.path.getsize(os.path.join(model_dir(), "model.bin")) * 1.1 + 0.3e9
    n_mem = int(0.5 * mem_available_bytes() // model_bytes)
    cores = host_cores()
    n = max(1, min(cores, n_mem, 8 * B32))
    seqs = []
    r = 0
    while len(seqs) < n:
        for b, p in enumerate(lz98_synth.workload_prompts(cfg, B32, lo, hi, 1.1, seed=r)):
            seqs.append((p, 1000 + r * B32 + b))
        r += 1
    seqs = seqs[:n]
    ctx = mp.get_context("spawn")
    t_all = time.time()
    stock_s = max(2.0, seconds / 2)
    barrier, q = ctx.Barrier(n), ctx.Queue()
    procs = [ctx.Process(target=_b32_cpu_worker, args=(p, sd, seconds, stock_s, barrier, q)) for p, sd in seqs]
    for pr in procs:
        pr.start()
    outs = _collect(procs, q, barrier, n, 1800.0)
    errs = [o[4] for o in outs if o[4]]
    if len(outs) < n:
        errs.append(f"{n - len(outs)} processes gave no result")
    fl = sum(o[0] / o[1] for o in outs if o[1] > 0)
    st = sum(o[2] / o[3] for o in outs if o[3] > 0)
    lens = sorted(len(p) for p, _ in seqs)
    return {"value": fl if not errs else None, "unit": UNIT, "cores": n, "kind": "reference",
            "cpu": cpu_model(), "host_cores": cores,
            "sample": f"{n} reference processes (one per core), one configs[2] sequence each (prompts "
                      f"{lens[0]}-{lens[-1]} tokens, prefilled untimed), temperature 0.8, top-p 0.95, k=3, "
                      f"decoding together (a barrier) for ~{seconds:.0f} s in the float tier: "
                      f"{sum(o[0] for o in outs)} tokens; sum of per-process rates",
            "stock_tier": {"value": st if not errs else None, "tokens": sum(o[2] for o in outs),
                           "sample": f"the same processes continuing for ~{stock_s:.0f} s in the stock tier"},
            "errors": errs[:3], "wall_s": time.time() - t_all}


def run_reference(args):
    """The reference arm: the reference engine itself on the headline
    workload (rank 0 only): the bench's 512-token prompt prefilled once
    (untimed), W warm-up decode slices, then K timed slices; the value is
    the tokens of the K slices over their decode time."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    Reference, available = _reference()
    if not available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/liblz98ref.so not built"}), flush=True)
        return None
    p = prompts(1, 0)[0]
    R = Reference(model_dir(), PROMPT + MAX_NEW + 64, SPEC_K)
    slice_s = min(3.0, max(0.3, 25.0 / max(1, args.steps)))
    prefill_s = R.session_begin(p, MAX_NEW, SPEC_K) * 1e-3
    n_prefill = 1

    def one(seconds):
        nonlocal n_prefill
        toks, rounds, el = R.session_decode(1 << 30, seconds * 1000.0)
        if len(toks) == 0:              # the 256-token budget is used up: prefill again
            R.session_begin(p, MAX_NEW, SPEC_K)
            n_prefill += 1
            toks, rounds, el = R.session_decode(1 << 30, seconds * 1000.0)
        return len(toks), len(rounds), el * 1e-3

    for _ in range(args.warmup):
        one(min(slice_s, 1.0))
    steps = [one(slice_s) for _ in range(max(1, args.steps))]
    R.close()
    ntok = sum(s_[0] for s_ in steps)
    nround = sum(s_[1] for s_ in steps)
    dec_s = sum(s_[2] for s_ in steps)
    v = ntok / max(1e-9, dec_s)
    sample = (f"reference C99 engine (oracle/_ref, one thread), float tier (--fixed off, --fastfp off), the "
              f"bench's 512-token prompt (prefill {prefill_s:.1f} s, untimed, {n_prefill}x), greedy k=2; "
              f"{args.steps} decode slices of ~{slice_s:.1f} s: {ntok} tokens, {nround} rounds")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dec_s * 1e3 / max(1, nround),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 weights/activations, int32 dot, f32 epilogue (CPU)",
            "data": "synthetic: random-init weights N(0,0.02)->bf16->Q8_0, uniform prompt ids",
            "config": {"workload": "configs[1]: ~0.5B KunMoe, batch 1 per GPU, 512-token prompt, greedy, k=2",
                       "model": "KunMoe-0.5B-synthetic", "global_batch": 1, "seq_len": PROMPT,
                       "new_tokens_budget": MAX_NEW, "spec_k": SPEC_K,
                       "parallelism": "none (the reference is single-threaded C99)"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": 1, "kind": "reference", "cpu": cpu_model(),
                             "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="0p5b", choices=["0p5b", "3b"],
                    help="0p5b: the headline (configs[1]) with the batch-32 workload (configs[2]); "
                         "3b: configs[3], 8 x 8192-token chunked prefill then greedy k=3")
    ap.add_argument("--seqs", type=int, default=1, help="sequences per GPU")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--b32-cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the C-ABI end-to-end pass")
    ap.add_argument("--no-b32", action="store_true", help="skip the batch-32 temperature workload")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel rounds at N > 1")
    ap.add_argument("--b32-only", action="store_true", help="run only the batch-32 workload (profiling)")
    ap.add_argument("--b32-prompts", type=int, nargs=2, default=[256, 1024], metavar=("LO", "HI"),
                    help="prompt length range of the batch-32 workload (default 256 1024, BASELINE configs[2]; "
                         "shorter ranges only shorten the prefill for profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "3b":
        run_3b(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
