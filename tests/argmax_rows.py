"""Rows for the lz_argmax_p1 checks: random, every element a new maximum,
none after the first, repeated maxima with signed zeros, spreads that
underflow exp, and a full 64000-wide vocabulary row."""
import numpy as np


def argmax_rows():
    rng = np.random.default_rng(5)
    rows = [
        (rng.standard_normal(8192) * 2.0).astype(np.float32),
        (rng.standard_normal(64000) * 0.5).astype(np.float32),
        np.linspace(-3.0, 3.0, 5000).astype(np.float32),                 # ascending: all records
        np.linspace(3.0, -3.0, 5000).astype(np.float32),                 # descending: no record
        np.array([0.0, -0.0, 0.0, 1.0, 1.0, -0.0, 1.0, 0.5] * 300, np.float32),
        (rng.standard_normal(3000) * 60.0).astype(np.float32),           # exp underflows to 0
        np.full(2048, 0.25, np.float32),
    ]
    r = (rng.standard_normal(20000) * 1.0).astype(np.float32)
    r[[17, 999, 15000, 19999]] = [4.0, 4.5, 4.5, 5.0]                   # late records
    rows.append(r)
    return rows
