"""The allocation-free lm_head entry point, for callers that cannot
allocate device memory: through the C ABI, its logits equal those of the
allocating path (lz_forward_verify) bit for bit, on two calls in a row, and
- at the row counts where the allocating path switches kernels (9 to 64
rows, hidden size 1024) - the oracle's lm_head bit for bit.  Collected last
on purpose; passes alone in a fresh process too."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LZ98_ERR_SIZE = 1002


def _static(L, m, rows, err):
    import torch
    h_dev = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).cuda()
    out = torch.full((len(rows), m.vocab), float("nan"), device="cuda")
    rc = L.lz_lm_head_static(m.h, ctypes.c_void_p(h_dev.data_ptr()), len(rows), ctypes.c_void_p(out.data_ptr()),
                             None, err, 256)
    assert rc == 0, err.value.decode()
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_lm_head_static_matches_verify(mini_dir, tiny_dir):
    import lz98
    L = lz98.lib()
    for d in (mini_dir, tiny_dir):
        m = lz98.Model(d)
        s = lz98.State(m, 256, 4)
        rng = np.random.default_rng(3)
        prompt = rng.integers(0, m.vocab, 12).astype(np.int32)
        s.batch_capture(prompt[:-1], 0)
        vt = np.array([prompt[-1], 5, 9, 13], np.int32)
        hid, logits = s.verify(vt, len(prompt) - 1)          # allocating path
        err = ctypes.create_string_buffer(256)
        for call, rows in enumerate((hid, hid[::-1].copy())):
            want = logits if call == 0 else logits[::-1]
            got = _static(L, m, rows, err)
            assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want).view(np.uint32)), \
                f"call {call}: static-scratch logits differ"
        # sizes beyond the static maximum are refused with their own code and a message
        import torch
        h_dev = torch.zeros((65, m.hidden), device="cuda")
        out = torch.zeros((65, m.vocab), device="cuda")
        rc = L.lz_lm_head_static(m.h, ctypes.c_void_p(h_dev.data_ptr()), 65, ctypes.c_void_p(out.data_ptr()),
                                 None, err, 256)
        assert rc == LZ98_ERR_SIZE and b"exceed" in err.value
        s.close()
        m.close()


def test_lm_head_static_row_counts_match_oracle():
    """Hidden size 1024 (~0.5B config): 9, 33 and the maximum 64 rows, the
    row counts at which the allocating path leaves the single-row GEMV,
    against the oracle's lm_head on two vocabulary slices, two calls in a
    row (the second on the rows reversed)."""
    import lz98
    from conftest import model_dir
    from oracles import Oracle
    d = model_dir("0p5b")
    m = lz98.Model(d)
    s = lz98.State(m, 256, 4)
    rng = np.random.default_rng(9)
    hid = s.batch_capture(rng.integers(0, m.vocab, 65).astype(np.int32), 0)   # 65 final-normed rows
    s.close()
    O = Oracle(d, 256, 4)
    L = lz98.lib()
    err = ctypes.create_string_buffer(256)
    V, W = m.vocab, 1024
    for n in (9, 33, 64):
        rows = hid[:n]
        want = {v0: O.lm_head_cols(rows, v0, W) for v0 in (0, V - W)}
        for call, rr in enumerate((rows, rows[::-1].copy())):
            got = _static(L, m, rr, err)
            for v0, w in want.items():
                w = w if call == 0 else w[::-1]
                assert np.array_equal(got[:, v0:v0 + W].view(np.uint32), np.ascontiguousarray(w).view(np.uint32)), \
                    (n, call, v0)
    O.close()
    m.close()
