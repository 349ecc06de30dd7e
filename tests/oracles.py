"""ctypes bindings to the two CPU checkers (test infrastructure only).

* ``Oracle``: oracle/liblz98oracle.so, the C restatement of the reference's
  float tier.
* ``Reference``: oracle/_ref/liblz98ref.so, the reference engine compiled
  unmodified from its own sources plus our token-id spec-loop driver
  (present only where the reference sources were available at build time).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "liblz98oracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "liblz98ref.so")

c_int, c_float, c_void_p, c_char_p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_char_p
P = ctypes.POINTER


def _ptr(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


def _f32(n):
    return np.zeros(n, np.float32)


class _Lib:
    _cache: dict = {}

    @classmethod
    def load(cls, path):
        if path not in cls._cache:
            cls._cache[path] = ctypes.CDLL(path)
        return cls._cache[path]


def oracle_available() -> bool:
    return os.path.exists(ORACLE_SO)


def reference_available() -> bool:
    return os.path.exists(REF_SO)


class Oracle:
    """The C restatement (one model + one state)."""

    def __init__(self, model_dir: str, seq_len: int = 512, spec_k_max: int = 4):
        L = self.L = _Lib.load(ORACLE_SO)
        L.lzo_open.restype = c_void_p
        L.lzo_open.argtypes = [c_char_p, c_char_p, c_int]
        L.lzo_state_new.restype = c_void_p
        L.lzo_state_new.argtypes = [c_void_p, c_int, c_int]
        for fn in ("lzo_exp", "lzo_rsqrt", "lzo_sigmoid"):
            getattr(L, fn).restype = c_float
            getattr(L, fn).argtypes = [c_float]
        L.lzo_random_f32.restype = c_float
        L.lzo_forward.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
        L.lzo_mtp_draft.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p]
        L.lzo_mtp_prefill.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]
        L.lzo_generate.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                   ctypes.c_ulonglong, c_void_p, c_int, P(c_int), c_void_p, c_int, P(c_int)]
        L.lzo_generate_pm.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                      ctypes.c_ulonglong, c_float, c_int, c_void_p, c_int, P(c_int), c_void_p,
                                      c_int, P(c_int)]
        L.lzo_set_positions.argtypes = [c_void_p, c_int, c_int]
        L.lzo_get_positions.argtypes = [c_void_p, P(c_int), P(c_int), P(c_int)]
        L.lzo_set_chain.argtypes = [c_void_p, c_void_p]
        L.lzo_get_chain.argtypes = [c_void_p, c_void_p]
        L.lzo_state_reset.argtypes = [c_void_p]
        L.lzo_lm_head_cols.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
        L.lzo_info.argtypes = [c_void_p, c_void_p]
        L.lzo_free.argtypes = [c_void_p]
        L.lzo_state_free.argtypes = [c_void_p]
        err = ctypes.create_string_buffer(512)
        self.m = L.lzo_open(model_dir.encode(), err, 512)
        if not self.m:
            raise RuntimeError("oracle open failed: " + err.value.decode())
        info = np.zeros(16, np.int32)
        L.lzo_info(c_void_p(self.m), _ptr(info))
        (self.vocab, self.hidden, self.n_layers, self.kda_heads, self.key_dim, self.latent,
         self.n_experts, self.top_k, self.shared_w, self.head_dim, self.n_heads,
         self.n_kv_heads, self.rotary_dim, self.seq_len_cfg) = [int(x) for x in info[:14]]
        self.s = L.lzo_state_new(c_void_p(self.m), seq_len, spec_k_max)

    def close(self):
        if self.s:
            self.L.lzo_state_free(c_void_p(self.s))
            self.s = None
        if self.m:
            self.L.lzo_free(c_void_p(self.m))
            self.m = None

    def reset(self):
        self.L.lzo_state_reset(c_void_p(self.s))

    def positions(self):
        a, b, c = c_int(), c_int(), c_int()
        self.L.lzo_get_positions(c_void_p(self.s), ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def set_positions(self, mtp_pos=-1, ssm_slot=-1):
        self.L.lzo_set_positions(c_void_p(self.s), mtp_pos, ssm_slot)

    def chain(self):
        c = _f32(self.hidden)
        self.L.lzo_get_chain(c_void_p(self.s), _ptr(c))
        return c

    def set_chain(self, c):
        c = np.ascontiguousarray(c, np.float32)
        self.L.lzo_set_chain(c_void_p(self.s), _ptr(c))

    def forward(self, tokens, pos0, advance_ring, want_logits=True):
        t = np.ascontiguousarray(tokens, np.int32)
        n = len(t)
        hid = _f32(n * self.hidden)
        lg = _f32(n * self.vocab) if want_logits else None
        rc = self.L.lzo_forward(c_void_p(self.m), c_void_p(self.s), _ptr(t), n, pos0,
                                int(advance_ring), _ptr(hid), _ptr(lg))
        if rc:
            raise RuntimeError("oracle forward failed")
        return hid.reshape(n, -1), (lg.reshape(n, -1) if lg is not None else None)

    def lm_head_cols(self, hidden, v0, nv):
        """Logits of the hidden rows over vocabulary rows [v0, v0 + nv)."""
        h = np.ascontiguousarray(hidden, np.float32)
        out = _f32(len(h) * nv)
        if self.L.lzo_lm_head_cols(c_void_p(self.m), _ptr(h), len(h), v0, nv, _ptr(out)):
            raise RuntimeError("oracle lm_head failed")
        return out.reshape(len(h), nv)

    def mtp_draft(self, tok, pos):
        lg = _f32(self.vocab)
        if self.L.lzo_mtp_draft(c_void_p(self.m), c_void_p(self.s), tok, pos, _ptr(lg)):
            raise RuntimeError("oracle draft failed")
        return lg

    def mtp_prefill(self, hidden, nxt, pos0):
        h = np.ascontiguousarray(hidden, np.float32)
        t = np.ascontiguousarray(nxt, np.int32)
        return self.L.lzo_mtp_prefill(c_void_p(self.m), c_void_p(self.s), _ptr(h), _ptr(t), len(t), pos0)

    def generate(self, prompt, max_new, spec_k, temp=0.0, topp=0.95, seed=1, p_min=0.0, n_min=0):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max_new + 16, np.int32)
        rounds = np.zeros(2 * (max_new + 16), np.int32)
        on, nr = c_int(), c_int()
        rc = self.L.lzo_generate_pm(c_void_p(self.m), c_void_p(self.s), _ptr(p), len(p), max_new, spec_k,
                                    temp, topp, seed, c_float(p_min), int(n_min), _ptr(out), len(out),
                                    ctypes.byref(on), _ptr(rounds), len(rounds) // 2, ctypes.byref(nr))
        if rc:
            raise RuntimeError(f"oracle generate failed rc={rc}")
        return out[:on.value].copy(), rounds[:2 * nr.value].reshape(-1, 2).copy()


class Reference:
    """The unmodified reference engine behind our token-id driver."""

    def __init__(self, model_dir: str, seq_len: int = 512, spec_k_max: int = 4,
                 nt_cap: int = 8, kernel: int = 7):
        L = self.L = _Lib.load(REF_SO)
        L.rd_open.restype = c_void_p
        L.rd_open.argtypes = [c_char_p, c_int, c_int, c_int, c_int, c_char_p, c_int]
        for fn in ("rd_exp", "rd_rsqrt", "rd_sigmoid"):
            getattr(L, fn).restype = c_float
            getattr(L, fn).argtypes = [c_float]
        L.rd_generate.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                  ctypes.c_ulonglong, c_void_p, c_int, P(c_int), c_void_p, c_int,
                                  P(c_int), P(ctypes.c_double), P(ctypes.c_double)]
        L.rd_generate_pm.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                     ctypes.c_ulonglong, c_float, c_int, c_void_p, c_int, P(c_int), c_void_p,
                                     c_int, P(c_int), P(ctypes.c_double), P(ctypes.c_double)]
        L.rd_session_begin.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float,
                                       ctypes.c_ulonglong, c_float, c_int, P(ctypes.c_double)]
        L.rd_session_decode.argtypes = [c_void_p, c_int, ctypes.c_double, c_void_p, c_int, P(c_int), c_void_p,
                                        c_int, P(c_int), P(ctypes.c_double)]
        L.rd_session_end.argtypes = [c_void_p]
        L.rd_forward_verify.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]
        L.rd_batch_capture.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p]
        L.rd_forward_capture.argtypes = [c_void_p, c_int, c_int, c_void_p, c_void_p]
        L.rd_mtp_draft.argtypes = [c_void_p, c_int, c_int, c_void_p, c_void_p]
        L.rd_mtp_prefill.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int]
        L.rd_set_positions.argtypes = [c_void_p, c_int, c_int]
        L.rd_set_chain.argtypes = [c_void_p, c_void_p]
        L.rd_info.argtypes = [c_void_p, c_void_p]
        L.rd_reset.argtypes = [c_void_p]
        L.rd_set_stock_tier.argtypes = [c_int]
        L.rd_set_tier.argtypes = [c_int]
        L.rd_set_round_debug.argtypes = [c_int, c_int]
        L.rd_close.argtypes = [c_void_p]
        err = ctypes.create_string_buffer(512)
        self.h = L.rd_open(model_dir.encode(), seq_len, spec_k_max, nt_cap, kernel, err, 512)
        if not self.h:
            raise RuntimeError("reference open failed: " + err.value.decode())
        info = np.zeros(16, np.int32)
        L.rd_info(c_void_p(self.h), _ptr(info))
        self.vocab, self.hidden = int(info[0]), int(info[1])

    def info(self):
        info = np.zeros(16, np.int32)
        self.L.rd_info(c_void_p(self.h), _ptr(info))
        return info

    def stock_tier(self, kernel: int = 7):
        """Switch the (process-global) reference arithmetic to its CLI
        defaults, --fixed all and --fastfp on, for timing the reference as
        shipped; its tokens then differ from the parity tier's."""
        self.L.rd_set_stock_tier(kernel)

    def round_debug(self, break_rollback: int = 0, skip_catchup: int = 0):
        """The rounds' test-only switches (process-global in the driver):
        debug_break_rollback and debug_skip_catchup of lz_spec_round."""
        self.L.rd_set_round_debug(int(break_rollback), int(skip_catchup))

    def close(self):
        if self.h:
            self.L.rd_close(c_void_p(self.h))
            self.h = None

    def reset(self):
        self.L.rd_reset(c_void_p(self.h))

    def set_positions(self, mtp_pos=-1, ssm_slot=-1):
        self.L.rd_set_positions(c_void_p(self.h), mtp_pos, ssm_slot)

    def set_chain(self, c):
        c = np.ascontiguousarray(c, np.float32)
        self.L.rd_set_chain(c_void_p(self.h), _ptr(c))

    def verify(self, tokens, pos0):
        t = np.ascontiguousarray(tokens, np.int32)
        n = len(t)
        lg, hid = _f32(n * self.vocab), _f32(n * self.hidden)
        if self.L.rd_forward_verify(c_void_p(self.h), _ptr(t), n, pos0, _ptr(lg), _ptr(hid)):
            raise RuntimeError("reference verify failed")
        return hid.reshape(n, -1), lg.reshape(n, -1)

    def batch_capture(self, tokens, pos0):
        t = np.ascontiguousarray(tokens, np.int32)
        hid = _f32(len(t) * self.hidden)
        if self.L.rd_batch_capture(c_void_p(self.h), _ptr(t), len(t), pos0, _ptr(hid)):
            raise RuntimeError("reference batch capture failed")
        return hid.reshape(len(t), -1)

    def forward_capture(self, tok, pos):
        lg, ch = _f32(self.vocab), _f32(self.hidden)
        if self.L.rd_forward_capture(c_void_p(self.h), tok, pos, _ptr(lg), _ptr(ch)):
            raise RuntimeError("reference capture failed")
        return ch, lg

    def mtp_draft(self, tok, pos):
        lg, ch = _f32(self.vocab), _f32(self.hidden)
        if self.L.rd_mtp_draft(c_void_p(self.h), tok, pos, _ptr(lg), _ptr(ch)):
            raise RuntimeError("reference draft failed")
        return lg, ch

    def mtp_prefill(self, hidden, nxt, pos0):
        h = np.ascontiguousarray(hidden, np.float32)
        t = np.ascontiguousarray(nxt, np.int32)
        return self.L.rd_mtp_prefill(c_void_p(self.h), _ptr(h), _ptr(t), len(t), pos0)

    def session_begin(self, prompt, max_new, spec_k, temp=0.0, topp=0.95, seed=1, p_min=0.0, n_min=0):
        """Reset and prefill `prompt` for a generation of up to max_new
        tokens that session_decode then runs in slices; returns the
        prefill's wall time in ms."""
        p = np.ascontiguousarray(prompt, np.int32)
        pf = ctypes.c_double()
        rc = self.L.rd_session_begin(c_void_p(self.h), _ptr(p), len(p), max_new, spec_k, temp, topp, seed,
                                     c_float(p_min), int(n_min), ctypes.byref(pf))
        if rc:
            raise RuntimeError(f"reference session prefill failed rc={rc}")
        return pf.value

    def session_decode(self, max_tokens, budget_ms=0.0):
        """Decode until max_tokens more tokens, the generation's budget or
        budget_ms of wall time (checked between rounds): (tokens, rounds,
        elapsed ms)."""
        out = np.zeros(max_tokens + 16, np.int32)
        rounds = np.zeros(2 * (max_tokens + 16), np.int32)
        on, nr, el = c_int(), c_int(), ctypes.c_double()
        rc = self.L.rd_session_decode(c_void_p(self.h), max_tokens, budget_ms, _ptr(out), len(out),
                                      ctypes.byref(on), _ptr(rounds), len(rounds) // 2, ctypes.byref(nr),
                                      ctypes.byref(el))
        if rc:
            raise RuntimeError(f"reference session decode failed rc={rc}")
        n = min(on.value, len(out))
        return out[:n].copy(), rounds[:2 * min(nr.value, len(rounds) // 2)].reshape(-1, 2).copy(), el.value

    def session_end(self):
        self.L.rd_session_end(c_void_p(self.h))

    def generate(self, prompt, max_new, spec_k, temp=0.0, topp=0.95, seed=1, p_min=0.0, n_min=0):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max_new + 16, np.int32)
        rounds = np.zeros(2 * (max_new + 16), np.int32)
        on, nr = c_int(), c_int()
        el, pf = ctypes.c_double(), ctypes.c_double()
        rc = self.L.rd_generate_pm(c_void_p(self.h), _ptr(p), len(p), max_new, spec_k, temp, topp, seed,
                                   c_float(p_min), int(n_min), _ptr(out), len(out), ctypes.byref(on),
                                   _ptr(rounds), len(rounds) // 2, ctypes.byref(nr), ctypes.byref(el),
                                   ctypes.byref(pf))
        if rc:
            raise RuntimeError(f"reference generate failed rc={rc}")
        self.last_elapsed_ms, self.last_prefill_ms = el.value, pf.value
        return out[:on.value].copy(), rounds[:2 * nr.value].reshape(-1, 2).copy()
