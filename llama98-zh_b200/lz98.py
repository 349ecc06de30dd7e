"""Python binding of the C ABI in include/lz98_gpu.h (liblz98gpu.so, built
in-tree by build.py).  Mirrors the reference's entry points on the MTP
speculative-decoding path: lz_open, lz_state_alloc, lz_forward*,
lz_mtp_draft_step, lz_mtp_prefill, lz_spec_round, lz_spec_accept(_temp),
plus the batched round.  There is no CPU fallback: loading fails loudly
when the library is missing or no CUDA device is visible."""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "liblz98gpu.so")

c_int, c_float, c_void_p, c_char_p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_char_p
P = ctypes.POINTER

_lib = None


class LzError(RuntimeError):
    """A failed call; .code is the library's return code when known."""

    def __init__(self, msg, code=None):
        super().__init__(msg)
        self.code = code


def _ptr(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


def lib():
    """Load liblz98gpu.so and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(SO):
        raise LzError(f"{SO} is missing: build it with llama98-zh_b200/build.py (nvcc, sm_100a)")
    L = ctypes.CDLL(SO)
    sig = {
        "lz_open": (c_int, [P(c_void_p), c_char_p, c_char_p, c_int]),
        "lz_free": (None, [c_void_p]),
        "lz_model_info": (None, [c_void_p, c_void_p]),
        "lz_model_weight_bytes": (ctypes.c_size_t, [c_void_p]),
        "lz_state_alloc": (c_int, [P(c_void_p), c_void_p, c_int, c_int, c_char_p, c_int]),
        "lz_state_alloc_batch": (c_int, [P(c_void_p), c_void_p, c_int, c_int, c_int, c_char_p, c_int]),
        "lz_state_reset": (None, [c_void_p, c_void_p]),
        "lz_state_free": (None, [c_void_p]),
        "lz_state_get": (c_int, [c_void_p, c_int, P(c_int), P(c_int), P(c_int)]),
        "lz_state_set": (c_int, [c_void_p, c_int, c_int, c_int]),
        "lz_state_get_chain": (c_int, [c_void_p, c_int, c_void_p]),
        "lz_state_set_chain": (c_int, [c_void_p, c_int, c_void_p]),
        "lz_forward": (P(c_float), [c_void_p, c_void_p, c_int, c_int]),
        "lz_forward_capture": (P(c_float), [c_void_p, c_void_p, c_int, c_int]),
        "lz_forward_batch_capture": (P(c_float), [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
        "lz_forward_verify": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int]),
        "lz_state_mtp_logits": (P(c_float), [c_void_p]),
        "lz_state_mtp_verify_hidden": (P(c_float), [c_void_p]),
        "lz_mtp_draft_step": (P(c_float), [c_void_p, c_void_p, c_int, c_int]),
        "lz_mtp_prefill": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
        "lz_mtp_catchup": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
        "lz_spec_round": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_int, c_void_p,
                                  c_int, c_int, c_void_p, P(c_int), P(c_int), P(c_int), c_char_p, c_int]),
        "lz_spec_round_temp": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_int, c_void_p,
                                       c_int, c_int, c_void_p, P(c_int), P(c_int), P(c_int), c_char_p, c_int]),
        "lz_spec_accept": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
        "lz_spec_accept_temp": (c_int, [c_void_p, c_void_p, c_int, c_int, c_float,
                                        P(ctypes.c_uint64), P(c_int)]),
        "lz_seq_prefill": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, P(c_int), c_char_p, c_int]),
        "lz_seq_set_sampler": (c_int, [c_void_p, c_int, c_float, c_float, ctypes.c_uint64]),
        "lz_seq_get_sampler": (c_int, [c_void_p, c_int, P(c_float), P(c_float), P(ctypes.c_uint64)]),
        "lz_spec_round_batch": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_char_p, c_int]),
        "lz_set_graphs": (c_int, [c_void_p, c_int]),
        "lz_set_pdl": (c_int, [c_void_p, c_int]),
        "lz_set_umma": (c_int, [c_void_p, c_int]),
        "lz_generate": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                ctypes.c_uint64, c_void_p, c_int, P(c_int), c_void_p, c_int, P(c_int),
                                c_char_p, c_int]),
        "lz_generate_ex": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                   ctypes.c_uint64, c_float, c_int, c_void_p, c_int, P(c_int), c_void_p, c_int,
                                   P(c_int), c_char_p, c_int]),
        "lz_debug_argmax_p1": (c_int, [c_void_p, c_int, P(c_int), P(c_float)]),
        "lz_debug_sumsq_split": (c_int, [c_void_p, c_int, c_int, c_void_p]),
        "lz_read_weights": (c_int, [c_void_p, c_char_p, c_int]),
        "lz_profile_experts": (c_int, [c_void_p, P(ctypes.c_double), P(ctypes.c_double), P(c_int)]),
        "lz_debug_wait_timeout": (c_int, [P(c_int), P(ctypes.c_double)]),
        "lz_debug_inject_wait_timeout": (c_int, [c_int, ctypes.c_double]),
        "lz_set_debug_timing": (c_int, [c_void_p, c_int]),
        "lz_state_counters": (c_int, [c_void_p, c_int, P(c_int), P(c_int), P(c_int), P(c_int)]),
        "lz_profile_round": (c_int, [c_void_p, c_int, P(ctypes.c_double), P(ctypes.c_double), P(c_int),
                                     P(ctypes.c_double), P(c_int)]),
        "lz_profile_launches": (c_int, [c_void_p, c_int, c_char_p, c_int]),
        "lz_lm_head_static": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_char_p, c_int]),
        "lz_state_stream": (c_void_p, [c_void_p]),
        "lz_ckpt_alloc": (c_int, [P(c_void_p), c_void_p, c_char_p, c_int]),
        "lz_ckpt_free": (None, [c_void_p]),
        "lz_ckpt_save": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_char_p, c_int]),
        "lz_ckpt_restore": (c_int, [c_void_p, c_void_p, c_void_p, P(c_int), c_char_p, c_int]),
        "lz_ckpt_save_seq": (c_int, [c_void_p, c_void_p, c_int, c_int, c_char_p, c_int]),
        "lz_ckpt_restore_seq": (c_int, [c_void_p, c_void_p, c_int, P(c_int), c_char_p, c_int]),
        "lz_debug_seq_sum": (c_int, [c_void_p, c_int, c_int, c_float, P(c_float), P(c_int)]),
        "lz_state_launches": (ctypes.c_longlong, [c_void_p]),
        "lz_ep_unique_id": (c_int, [c_void_p, c_char_p, c_int]),
        "lz_ep_init": (c_int, [c_void_p, c_void_p, c_int, c_int, c_char_p, c_int]),
        "lz_generate_resume": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                       ctypes.c_uint64, c_void_p, c_int, P(c_int), c_void_p, c_int, P(c_int),
                                       c_char_p, c_int]),
        "lz_prefix_init": (c_int, [P(c_void_p), c_void_p, c_char_p, c_int]),
        "lz_prefix_free": (None, [c_void_p]),
        "lz_prefix_reset": (None, [c_void_p]),
        "lz_prefix_match": (c_int, [c_void_p, c_void_p, c_int]),
        "lz_prefix_prepare_tokens": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                             c_void_p, c_int, P(c_int), P(c_int), c_char_p, c_int]),
        "lz_prefix_stats": (None, [c_void_p, P(ctypes.c_long), P(ctypes.c_long), P(ctypes.c_long),
                                   P(ctypes.c_long), P(ctypes.c_long)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


EXPORTS = ["lz_profile_experts", "lz_debug_sumsq_split", "lz_debug_wait_timeout", "lz_debug_inject_wait_timeout", "lz_generate_ex", "lz_debug_argmax_p1", "lz_read_weights", "lz_set_debug_timing", "lz_open", "lz_free", "lz_model_info", "lz_model_weight_bytes", "lz_state_alloc",
           "lz_state_alloc_batch", "lz_state_reset", "lz_state_free", "lz_state_get", "lz_state_set",
           "lz_state_get_chain", "lz_state_set_chain", "lz_forward", "lz_forward_capture",
           "lz_forward_batch_capture", "lz_forward_verify", "lz_state_mtp_logits",
           "lz_state_mtp_verify_hidden", "lz_mtp_draft_step", "lz_mtp_prefill", "lz_mtp_catchup",
           "lz_spec_round", "lz_spec_round_temp", "lz_spec_accept", "lz_spec_accept_temp",
           "lz_seq_prefill", "lz_seq_set_sampler", "lz_seq_get_sampler", "lz_spec_round_batch", "lz_set_graphs", "lz_set_pdl", "lz_set_umma", "lz_generate", "lz_state_stream",
           "lz_state_launches", "lz_state_counters", "lz_profile_round", "lz_profile_launches", "lz_lm_head_static", "lz_debug_seq_sum",
           "lz_ckpt_alloc", "lz_ckpt_free", "lz_ckpt_save", "lz_ckpt_restore", "lz_ckpt_save_seq",
           "lz_ckpt_restore_seq", "lz_generate_resume", "lz_prefix_init", "lz_prefix_free", "lz_prefix_reset",
           "lz_prefix_match", "lz_prefix_prepare_tokens", "lz_prefix_stats", "lz_ep_unique_id", "lz_ep_init"]


class LZSampleParams(ctypes.Structure):
    """The reference's LZSampleParams (src/sampler.h:144-173), field for field."""
    _fields_ = [("temperature", c_float), ("temp_think", c_float), ("think_temp_enabled", c_int),
                ("topp", c_float), ("minp", c_float), ("topk", c_int), ("presence_penalty", c_float),
                ("frequency_penalty", c_float), ("repetition_penalty", c_float), ("repeat_last_n", c_int),
                ("minp_llamacpp", c_int)]


class LZSampler(ctypes.Structure):
    """The reference's LZSampler (src/sampler.h:176-186), field for field."""
    _fields_ = [("vocab_size", c_int), ("p", LZSampleParams), ("rng_state", ctypes.c_uint64),
                ("probindex", c_void_p), ("counts", c_void_p), ("ring", c_void_p), ("cap", c_int),
                ("head", c_int), ("n_win", c_int)]


def make_sampler(vocab, temp, topp, rng, **params):
    """An LZSampler with the reference loop's settings (identity penalties,
    no top-k or min-p) and any field of LZSampleParams overridden."""
    smp = LZSampler()
    smp.vocab_size = int(vocab)
    smp.p.temperature = float(temp)
    smp.p.topp = float(topp)
    smp.p.repetition_penalty = 1.0
    for k, v in params.items():
        setattr(smp.p, k, v)
    smp.rng_state = int(rng)
    return smp


class Model:
    def __init__(self, model_dir: str):
        L = lib()
        h = c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.lz_open(ctypes.byref(h), model_dir.encode(), err, 512)
        if rc:
            raise LzError(f"lz_open failed ({rc}): {err.value.decode()}")
        self.h = h
        info = np.zeros(16, np.int32)
        L.lz_model_info(h, _ptr(info))
        (self.vocab, self.hidden, self.n_layers, self.kda_heads, self.key_dim, self.latent,
         self.n_experts, self.top_k, self.shared_w, self.head_dim, self.n_heads, self.n_kv_heads,
         self.rotary_dim, self.seq_len_cfg, self.mtp_ffn, self.moe_ffn) = [int(x) for x in info]
        self.weight_bytes = int(L.lz_model_weight_bytes(h))

    def close(self):
        if self.h:
            lib().lz_free(self.h)
            self.h = None


class State:
    def __init__(self, model: Model, seq_len: int, spec_k_max: int, n_seq: int = 1):
        L = lib()
        h = c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.lz_state_alloc_batch(ctypes.byref(h), model.h, n_seq, seq_len, spec_k_max, err, 512)
        if rc:
            raise LzError(f"lz_state_alloc failed ({rc}): {err.value.decode()}")
        self.h, self.m, self.n_seq, self.k_max = h, model, n_seq, spec_k_max

    def close(self):
        if self.h:
            lib().lz_state_free(self.h)
            self.h = None

    def reset(self):
        lib().lz_state_reset(self.h, self.m.h)

    def positions(self, seq=0):
        a, b, c = c_int(), c_int(), c_int()
        lib().lz_state_get(self.h, seq, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def set_positions(self, seq=0, mtp_pos=-1, ssm_slot=-1):
        lib().lz_state_set(self.h, seq, mtp_pos, ssm_slot)

    def chain(self, seq=0):
        c = np.zeros(self.m.hidden, np.float32)
        lib().lz_state_get_chain(self.h, seq, _ptr(c))
        return c

    def set_chain(self, c, seq=0):
        c = np.ascontiguousarray(c, np.float32)
        lib().lz_state_set_chain(self.h, seq, _ptr(c))

    def counters(self, seq=0):
        v = [c_int() for _ in range(4)]
        lib().lz_state_counters(self.h, seq, *[ctypes.byref(x) for x in v])
        return tuple(x.value for x in v)

    def profile_round(self, k):
        gm, gb, rm = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        ng, nk = c_int(), c_int()
        rc = lib().lz_profile_round(self.h, k, ctypes.byref(gm), ctypes.byref(gb), ctypes.byref(ng),
                                    ctypes.byref(rm), ctypes.byref(nk))
        if rc:
            raise LzError(f"profile round failed ({rc})")
        em, eb, en = ctypes.c_double(), ctypes.c_double(), c_int()
        lib().lz_profile_experts(self.h, ctypes.byref(em), ctypes.byref(eb), ctypes.byref(en))
        return {"gemv_ms": gm.value, "gemv_bytes": gb.value, "n_gemv": ng.value,
                "round_ms": rm.value, "n_kernels": nk.value,
                "expert_ms": em.value, "expert_bytes": eb.value, "n_expert": en.value}

    def profile_launches(self, k):
        """One eager round with every launch event-timed: [(kernel, us), ...]."""
        buf = ctypes.create_string_buffer(1 << 20)
        n = lib().lz_profile_launches(self.h, k, buf, len(buf))
        if n < 0:
            raise LzError(f"profile failed ({n})", n)
        out = []
        for line in buf.value.decode().splitlines():
            name, us = line.rsplit("\t", 1)
            out.append((name, float(us)))
        return out

    def stream(self):
        return lib().lz_state_stream(self.h)

    def launches(self):
        return int(lib().lz_state_launches(self.h))

    def graphs(self, on: bool):
        lib().lz_set_graphs(self.h, int(on))

    def umma(self, on: bool):
        """tcgen05 dense GEMMs for more than 8 token rows (default off: the mma.sync kernel)."""
        lib().lz_set_umma(self.h, 1 if on else 0)

    def pdl(self, on: bool):
        lib().lz_set_pdl(self.h, int(on))

    # --- forwards of sequence 0
    def forward(self, tok, pos, capture=False):
        fn = lib().lz_forward_capture if capture else lib().lz_forward
        p = fn(self.m.h, self.h, int(tok), int(pos))
        if not p:
            raise LzError("forward failed")
        return np.ctypeslib.as_array(p, shape=(self.m.vocab,)).copy()

    def batch_capture(self, tokens, pos0):
        t = np.ascontiguousarray(tokens, np.int32)
        hid = np.zeros((len(t), self.m.hidden), np.float32)
        if not lib().lz_forward_batch_capture(self.m.h, self.h, _ptr(t), len(t), pos0, _ptr(hid)):
            raise LzError("batch capture failed")
        return hid

    def verify(self, tokens, pos0):
        t = np.ascontiguousarray(tokens, np.int32)
        n = len(t)
        if lib().lz_forward_verify(self.m.h, self.h, _ptr(t), n, pos0):
            raise LzError("verify failed")
        lg = np.ctypeslib.as_array(lib().lz_state_mtp_logits(self.h), shape=(n, self.m.vocab)).copy()
        hid = np.ctypeslib.as_array(lib().lz_state_mtp_verify_hidden(self.h), shape=(n, self.m.hidden)).copy()
        return hid, lg

    def mtp_draft(self, tok, pos):
        p = lib().lz_mtp_draft_step(self.m.h, self.h, int(tok), int(pos))
        if not p:
            raise LzError("draft step failed")
        return np.ctypeslib.as_array(p, shape=(self.m.vocab,)).copy()

    def mtp_prefill(self, hidden, nxt, pos0):
        h = np.ascontiguousarray(hidden, np.float32)
        t = np.ascontiguousarray(nxt, np.int32)
        if lib().lz_mtp_prefill(self.m.h, self.h, _ptr(h), _ptr(t), len(t), pos0):
            raise LzError("mtp prefill failed")

    def spec_round(self, anchor, anchor_pos, k, samp=None, break_rollback=0, skip_catchup=0):
        out = np.zeros(8, np.int32)
        na, npos, ke = c_int(), c_int(), c_int()
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_spec_round(self.m.h, self.h, anchor, anchor_pos, k, 0.0, 0,
                                 ctypes.byref(samp) if samp is not None else None, int(break_rollback),
                                 int(skip_catchup), _ptr(out), ctypes.byref(na), ctypes.byref(npos),
                                 ctypes.byref(ke), err, 256)
        if rc < 0:
            raise LzError(f"spec round failed ({rc}): {err.value.decode()}", rc)
        return out[:rc].copy(), na.value, npos.value, ke.value

    def spec_round_temp(self, anchor, anchor_pos, k, temp, topp, rng, break_rollback=0, skip_catchup=0,
                        samp=None):
        """One coupled temperature round of sequence 0; returns the tokens,
        n_accept, the new position, k_eff and the advanced generator."""
        out = np.zeros(8, np.int32)
        na, npos, ke = c_int(), c_int(), c_int()
        err = ctypes.create_string_buffer(256)
        if samp is None:
            samp = make_sampler(self.m.vocab, temp, topp, rng)
        rc = lib().lz_spec_round_temp(self.m.h, self.h, anchor, anchor_pos, k, 0.0, 0, ctypes.byref(samp),
                                      int(break_rollback), int(skip_catchup), _ptr(out), ctypes.byref(na),
                                      ctypes.byref(npos), ctypes.byref(ke), err, 256)
        if rc < 0:
            raise LzError(f"temperature round failed ({rc}): {err.value.decode()}", rc)
        return out[:rc].copy(), na.value, npos.value, ke.value, samp.rng_state

    # --- batched path
    def set_sampler(self, seq, temp, topp, seed):
        rc = lib().lz_seq_set_sampler(self.h, seq, float(temp), float(topp), int(seed))
        if rc:
            raise LzError(f"set sampler failed ({rc})")

    def ep_init(self, uid: bytes, rank: int, world: int):
        """Expert parallelism over `world` ranks (collective: every rank calls
        it with the same id)."""
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_ep_init(self.h, buf, rank, world, err, 256)
        if rc:
            raise LzError(f"ep init failed ({rc}): {err.value.decode()}", rc)

    def get_sampler(self, seq=0):
        """(temperature, top-p, generator state) of sequence `seq` on the device."""
        t, p, r = c_float(), c_float(), ctypes.c_uint64()
        rc = lib().lz_seq_get_sampler(self.h, seq, ctypes.byref(t), ctypes.byref(p), ctypes.byref(r))
        if rc:
            raise LzError(f"get sampler failed ({rc})", rc)
        return t.value, p.value, r.value

    def seq_prefill(self, seq, prompt):
        p = np.ascontiguousarray(prompt, np.int32)
        a = c_int()
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_seq_prefill(self.m.h, self.h, seq, _ptr(p), len(p), ctypes.byref(a), err, 256)
        if rc:
            raise LzError(f"prefill failed ({rc}): {err.value.decode()}")
        return a.value

    def round_batch(self, k, fetch=True):
        err = ctypes.create_string_buffer(256)
        toks = np.zeros((self.n_seq, k + 1), np.int32) if fetch else None
        cnt = np.zeros(self.n_seq, np.int32) if fetch else None
        rc = lib().lz_spec_round_batch(self.m.h, self.h, k, _ptr(toks), _ptr(cnt), err, 256)
        if rc:
            raise LzError(f"batched round failed ({rc}): {err.value.decode()}", rc)
        return toks, cnt

    def generate_resume(self, start_pos, suffix, max_new, spec_k, temp=0.0, topp=0.95, seed=1):
        p = np.ascontiguousarray(suffix, np.int32)
        out = np.zeros(max_new + 16, np.int32)
        rounds = np.zeros(2 * (max_new + 16), np.int32)
        on, nr = c_int(), c_int()
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_generate_resume(self.m.h, self.h, start_pos, _ptr(p), len(p), max_new, spec_k, temp, topp,
                                      seed, _ptr(out), len(out), ctypes.byref(on), _ptr(rounds), len(rounds) // 2,
                                      ctypes.byref(nr), err, 256)
        if rc:
            raise LzError(f"generate resume failed ({rc}): {err.value.decode()}", rc)
        return out[:on.value].copy(), rounds[:2 * nr.value].reshape(-1, 2).copy()

    def generate(self, prompt, max_new, spec_k, temp=0.0, topp=0.95, seed=1, p_min=0.0, n_min=0):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max_new + 16, np.int32)
        rounds = np.zeros(2 * (max_new + 16), np.int32)
        on, nr = c_int(), c_int()
        err = ctypes.create_string_buffer(256)
        if p_min == 0.0 and n_min == 0:
            rc = lib().lz_generate(self.m.h, self.h, _ptr(p), len(p), max_new, spec_k, temp, topp, seed,
                                   _ptr(out), len(out), ctypes.byref(on), _ptr(rounds), len(rounds) // 2,
                                   ctypes.byref(nr), err, 256)
        else:
            rc = lib().lz_generate_ex(self.m.h, self.h, _ptr(p), len(p), max_new, spec_k, temp, topp, seed,
                                      float(p_min), int(n_min), _ptr(out), len(out), ctypes.byref(on),
                                      _ptr(rounds), len(rounds) // 2, ctypes.byref(nr), err, 256)
        if rc:
            raise LzError(f"generate failed ({rc}): {err.value.decode()}")
        return out[:on.value].copy(), rounds[:2 * nr.value].reshape(-1, 2).copy()


class Checkpoint:
    """Device snapshot of one sequence's recurrent state (lz_ckpt_*)."""

    def __init__(self, model: "Model"):
        h = c_void_p()
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_ckpt_alloc(ctypes.byref(h), model.h, err, 256)
        if rc:
            raise LzError(f"lz_ckpt_alloc failed ({rc}): {err.value.decode()}")
        self.h = h

    def close(self):
        if self.h:
            lib().lz_ckpt_free(self.h)
            self.h = None

    def save(self, state: "State", pos: int, seq: int = 0) -> int:
        err = ctypes.create_string_buffer(256)
        return lib().lz_ckpt_save_seq(self.h, state.h, seq, pos, err, 256)

    def restore(self, state: "State", seq: int = 0):
        """(rc, position)."""
        err = ctypes.create_string_buffer(256)
        pos = c_int(-1)
        rc = lib().lz_ckpt_restore_seq(self.h, state.h, seq, ctypes.byref(pos), err, 256)
        return rc, pos.value


DEBUG_COUNTERS = ("lz_debug_us_verify", "lz_debug_us_draft", "lz_debug_us_capture", "lz_debug_us_catchup",
                  "lz_debug_n_capture", "lz_debug_n_catchup", "lz_debug_n_ring_rollback")


class PrefixCache:
    """LZPrefixCache on token ids (one conversation's reusable prefix)."""

    def __init__(self, model: "Model"):
        self.m = model
        self.h = c_void_p()
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_prefix_init(ctypes.byref(self.h), model.h, err, 256)
        if rc:
            raise LzError(f"prefix init failed ({rc}): {err.value.decode()}", rc)

    def close(self):
        if self.h:
            lib().lz_prefix_free(self.h)
            self.h = None

    def match(self, pre):
        p = np.ascontiguousarray(pre, np.int32)
        return lib().lz_prefix_match(self.h, _ptr(p), len(p))

    def prepare(self, state: "State", cur, pre, tail):
        """Returns (start_pos, reused)."""
        c, p, t = (np.ascontiguousarray(a, np.int32) for a in (cur, pre, tail))
        sp, ru = c_int(), c_int()
        err = ctypes.create_string_buffer(256)
        rc = lib().lz_prefix_prepare_tokens(self.h, self.m.h, state.h, _ptr(c), len(c), _ptr(p), len(p), _ptr(t),
                                            len(t), ctypes.byref(sp), ctypes.byref(ru), err, 256)
        if rc:
            raise LzError(f"prefix prepare failed ({rc}): {err.value.decode()}", rc)
        return sp.value, ru.value

    def stats(self):
        v = [ctypes.c_long() for _ in range(5)]
        lib().lz_prefix_stats(self.h, *[ctypes.byref(x) for x in v])
        return dict(zip(("calls", "hits", "tokens_saved", "mismatch", "unsplittable"), (x.value for x in v)))


def ep_unique_id() -> bytes:
    """A fresh NCCL id for lz_ep_init (made on one rank, shared with all)."""
    buf = ctypes.create_string_buffer(128)
    err = ctypes.create_string_buffer(256)
    rc = lib().lz_ep_unique_id(buf, err, 256)
    if rc:
        raise LzError(f"ep unique id failed ({rc}): {err.value.decode()}", rc)
    return buf.raw


def debug_counters():
    """The exported debug data symbols, by name."""
    return {n: ctypes.c_longlong.in_dll(lib(), n).value for n in DEBUG_COUNTERS}


def debug_argmax_p1(vals):
    """The device lz_argmax_p1 of host values: (index, probability)."""
    v = np.ascontiguousarray(vals, np.float32)
    idx, p1 = c_int(), c_float()
    rc = lib().lz_debug_argmax_p1(_ptr(v), len(v), ctypes.byref(idx), ctypes.byref(p1))
    if rc:
        raise LzError(f"lz_debug_argmax_p1 failed ({rc})")
    return idx.value, p1.value


def debug_seq_sum(vals, mode=0, target=0.0):
    """The device's sequential-sum primitive on host values: (value, hit)."""
    v = np.ascontiguousarray(vals, np.float32)
    out, hit = c_float(), c_int()
    rc = lib().lz_debug_seq_sum(_ptr(v), len(v), int(mode), float(target), ctypes.byref(out), ctypes.byref(hit))
    if rc:
        raise LzError(f"debug_seq_sum failed ({rc})")
    return out.value, hit.value


def debug_sumsq_split(rows):
    """The input norms' split sum of squares over 1-4 host rows: float32 [nrows]."""
    v = np.ascontiguousarray(rows, np.float32)
    if v.ndim == 1:
        v = v[None]
    out = np.zeros(v.shape[0], np.float32)
    rc = lib().lz_debug_sumsq_split(_ptr(v), v.shape[0], v.shape[1], _ptr(out))
    if rc:
        raise LzError(f"lz_debug_sumsq_split failed ({rc})")
    return out


def spec_accept(draft, targ, bonus):
    d = np.ascontiguousarray(draft, np.int32)
    t = np.ascontiguousarray(targ, np.int32)
    out = np.zeros(len(d) + 1, np.int32)
    n = lib().lz_spec_accept(_ptr(d), _ptr(t), len(d), int(bonus), _ptr(out))
    return n, out[:n + 1].copy()


def spec_accept_temp(p, q, x, u, rng):
    p = np.ascontiguousarray(p, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    r = ctypes.c_uint64(rng)
    acc = c_int()
    tok = lib().lz_spec_accept_temp(_ptr(p), _ptr(q), int(x), len(p), float(u), ctypes.byref(r), ctypes.byref(acc))
    return tok, acc.value, r.value
