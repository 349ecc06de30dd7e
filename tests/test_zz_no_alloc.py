"""The allocation-free lm_head entry point, for callers that cannot
allocate device memory: through the C ABI, its logits equal those of the
allocating path (lz_forward_verify) bit for bit, on two calls in a row.
Collected last on purpose; passes alone in a fresh process too."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_lm_head_static_matches_verify(mini_dir, tiny_dir):
    import torch
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
            h_dev = torch.from_numpy(np.ascontiguousarray(rows)).cuda()
            out = torch.full((len(rows), m.vocab), float("nan"), device="cuda")
            rc = L.lz_lm_head_static(m.h, ctypes.c_void_p(h_dev.data_ptr()), len(rows),
                                     ctypes.c_void_p(out.data_ptr()), None, err, 256)
            assert rc == 0, err.value.decode()
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want).view(np.uint32)), \
                f"call {call}: static-scratch logits differ"
        # sizes beyond the static maximum are refused with a message
        rc = L.lz_lm_head_static(m.h, ctypes.c_void_p(h_dev.data_ptr()), 65, ctypes.c_void_p(out.data_ptr()),
                                 None, err, 256)
        assert rc != 0 and b"exceed" in err.value
        s.close()
        m.close()
