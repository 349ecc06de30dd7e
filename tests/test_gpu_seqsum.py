"""The device primitive behind every sequential float sum of the sampler
(softmax normaliser, cumulative distributions, top-p mass): it runs the
sum in parallel by binade segments and must equal the sequential
float32 cumulatives bit for bit, including exact ties, zeros, subnormals
and large jumps, and find the same first index against a threshold."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _seq(v):
    out = np.empty(len(v), np.float32)
    s = np.float32(0)
    for j, x in enumerate(v):
        s = np.float32(s + x)
        out[j] = s
    return out


def families(rng):
    for n in (1, 7, 1000, 1024, 1025, 5000, 8193, 9217, 20000, 64000, 70001):
        yield f"uniform{n}", rng.random(n).astype(np.float32)
    n = 64000
    yield "softmax-like", np.exp(rng.normal(0, 1, n) - 4).astype(np.float32)
    yield "probabilities", (rng.random(n) / (n / 2)).astype(np.float32)
    yield "few-bit ties", (rng.integers(0, 16, n) * 2.0 ** rng.integers(-30, 3, n)).astype(np.float32)
    sub = (rng.integers(0, 1 << 20, n) * 2.0 ** -149).astype(np.float32)
    sub[rng.random(n) < 0.3] = 0
    yield "subnormal+zeros", sub
    z = rng.random(n).astype(np.float32)
    z[rng.random(n) < 0.5] = 0
    z[rng.random(n) < 0.01] = 1e6
    yield "zeros+jumps", z
    lead = np.zeros(n, np.float32)
    lead[3000:] = rng.random(n - 3000)
    yield "leading zeros", lead
    yield "all zeros", np.zeros(5000, np.float32)
    yield "sorted desc", np.sort(rng.random(n).astype(np.float32) / 1000)[::-1].copy()


def test_sum_and_find_bit_exact():
    import lz98
    rng = np.random.default_rng(3)
    for name, v in families(rng):
        c = _seq(v)
        tot, hit = lz98.debug_seq_sum(v, 0)
        assert np.float32(tot).view(np.uint32) == c[-1].view(np.uint32), name
        assert hit == -1
        for frac in (0.0, 0.3, 0.999, 1.5):
            target = np.float32(c[-1] * frac)
            for mode, cond in ((1, target < c), (2, c >= target)):
                idx = np.nonzero(cond)[0]
                val, hit = lz98.debug_seq_sum(v, mode, float(target))
                want = int(idx[0]) if len(idx) else -1
                assert hit == want, (name, frac, mode, hit, want)
                want_val = c[want] if want >= 0 else c[-1]
                assert np.float32(val).view(np.uint32) == want_val.view(np.uint32), (name, frac, mode)


def test_argmax_p1_bit_exact():
    """The device lz_argmax_p1 (records by a block scan, exact sequential
    sums between them) against the oracle's sequential loop."""
    import ctypes
    import lz98
    from argmax_rows import argmax_rows
    from oracles import _Lib, ORACLE_SO
    L = _Lib.load(ORACLE_SO)
    L.lzo_argmax_p1.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
    for row in argmax_rows():
        ref = ctypes.c_float()
        ri = L.lzo_argmax_p1(ctypes.c_void_p(row.ctypes.data), len(row), ctypes.byref(ref))
        gi, gp = lz98.debug_argmax_p1(row)
        assert gi == ri
        assert np.float32(gp).view(np.uint32) == np.float32(ref.value).view(np.uint32), (len(row), gp, ref.value)


def test_bounded_wait_reports_and_context_survives():
    """A wait that never completes (an mbarrier nothing arrives on) gives up
    after about a second and reports through the error word; the context
    stays usable (the next device call works)."""
    import ctypes
    import lz98
    err, ms = ctypes.c_int(-1), ctypes.c_double()
    assert lz98.lib().lz_debug_wait_timeout(ctypes.byref(err), ctypes.byref(ms)) == 0
    assert err.value == 2
    assert 500.0 < ms.value < 20000.0
    v, hit = lz98.debug_seq_sum(np.ones(100, np.float32))
    assert v == 100.0



def _seq_sumsq(row):
    s = np.float32(0)
    with np.errstate(over="ignore"):
        for x in row:
            s = np.float32(s + np.float32(x * x))
    return s


def sumsq_rows(rng, n):
    """Rows for the input norms' split sum of squares: ordinary activations,
    rows whose sequential sum drifts far from the tree estimate (a few huge
    entries early, then values the accumulator absorbs), zeros, subnormal
    squares, squares that overflow, and constant rows."""
    yield "normal", rng.standard_normal(n).astype(np.float32)
    yield "scaled", (rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 2)).astype(np.float32)
    r = (rng.standard_normal(n) * 0.05).astype(np.float32)
    r[rng.integers(0, 64, 3)] = rng.standard_normal(3).astype(np.float32) * 300
    yield "early outliers", r
    r = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    r[0] = 4096.0
    yield "absorbed tail", r
    r = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    r[n // 2] = 4096.0
    yield "mid jump", r
    r = rng.standard_normal(n).astype(np.float32)
    r[rng.random(n) < 0.7] = 0
    yield "sparse", r
    yield "zeros", np.zeros(n, np.float32)
    yield "subnormal squares", (rng.standard_normal(n) * 1e-22).astype(np.float32)
    r = rng.standard_normal(n).astype(np.float32)
    r[n - 5] = 3e19
    yield "overflow", r
    yield "constant", np.full(n, 0.1, np.float32)


def test_sumsq_split_bit_exact():
    """The segment-split sum of squares of the input norms equals the
    sequential float32 sum (src/ops_norm.c:718) bit for bit, including rows
    where no candidate start matches and a segment is chained again."""
    import lz98
    rng = np.random.default_rng(7)
    for n in (512, 1024, 2048, 4096):
        rows = list(sumsq_rows(rng, n))
        want = [_seq_sumsq(v) for _, v in rows]
        for nr in (1, 3, 4):
            for i in range(0, len(rows), nr):
                got = lz98.debug_sumsq_split(np.stack([v for _, v in rows[i:i + nr]]))
                for j, g in enumerate(got):
                    name = rows[i + j][0]
                    assert np.float32(g).view(np.uint32) == want[i + j].view(np.uint32), (n, nr, name, g, want[i + j])
