"""The C-ABI library loads and exports every entry point that
include/lz98_gpu.h declares (no compute call, no GPU needed); the pure
host entry points (model-free acceptance) agree with the oracle."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lz98_gpu.h")
SO = os.path.join(ROOT, "llama98-zh_b200", "liblz98gpu.so")


def declared():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(lz_[a-z0-9_]+)\s*\(", txt)))


@pytest.fixture(scope="module")
def so():
    if not os.path.exists(SO):
        import build
        build.build()
    return ctypes.CDLL(SO)


def test_every_declared_symbol_is_exported(so):
    names = declared()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing


def declared_data():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    out = []
    for decl in re.findall(r"extern\s+long\s+long\s+([^;]+);", txt):
        out += [n.strip() for n in decl.split(",")]
    return sorted(out)


def test_debug_data_symbols_exported(so):
    """The reference's debug data (src/forward.c:86-124, src/generate.c:226)
    are exported as 64-bit integers that start at 0."""
    import lz98
    names = declared_data()
    assert "lz_debug_n_ring_rollback" in names and "lz_debug_us_verify" in names
    assert sorted(lz98.DEBUG_COUNTERS) == names
    for n in names:
        assert ctypes.c_longlong.in_dll(so, n).value >= 0


def test_binding_covers_header():
    import lz98
    assert sorted(lz98.EXPORTS) == declared()


def test_spec_accept_host(so):
    import lz98
    n, out = lz98.spec_accept([1, 2, 3], [1, 2, 3], 9)
    assert n == 3 and out.tolist() == [1, 2, 3, 9]
    n, out = lz98.spec_accept([1, 5, 3], [1, 2, 3], 9)
    assert n == 1 and out.tolist() == [1, 2]
    n, out = lz98.spec_accept([4], [1], 9)
    assert n == 0 and out.tolist() == [1]


def test_spec_accept_temp_host_matches_oracle(so):
    import lz98
    from oracles import Oracle, oracle_available
    if not oracle_available():
        pytest.skip("oracle not built")
    import oracles
    L = oracles._Lib.load(oracles.ORACLE_SO)
    rng = np.random.default_rng(4)
    V = 500
    for trial in range(200):
        p = rng.dirichlet(np.ones(V)).astype(np.float32)
        q = rng.dirichlet(np.ones(V)).astype(np.float32)
        if trial % 7 == 0:
            p = q.copy()
        x = int(rng.integers(0, V))
        u = float(np.float32(rng.random()))
        seed = int(rng.integers(1, 2**63))
        tok, acc, r_after = lz98.spec_accept_temp(p, q, x, u, seed)
        r = ctypes.c_ulonglong(seed)
        a = ctypes.c_int()
        L.lzo_spec_accept_temp.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_float, ctypes.POINTER(ctypes.c_ulonglong),
                                           ctypes.POINTER(ctypes.c_int)]
        t2 = L.lzo_spec_accept_temp(p.ctypes.data, q.ctypes.data, x, V, u, ctypes.byref(r), ctypes.byref(a))
        assert (tok, acc, r_after) == (t2, a.value, r.value)
    # invalid input keeps the reference's -1 sentinel
    tok, acc, _ = lz98.spec_accept_temp(np.ones(4, np.float32), np.ones(4, np.float32), 7, 0.5, 1)
    assert tok == -1 and acc == 0


def test_writer_header_layout():
    import lz98_synth
    h = lz98_synth.header_words(lz98_synth.CONFIGS["tiny"])
    # magic + version + 28 words + 128 layer types + 13 + 17 + 3*128 + 6 + 128
    assert len(h) == 4 + 4 + 4 * (28 + 128 + 13 + 17 + 3 * 128 + 6 + 128)
    assert h[:4] == b"L98Z"


def test_build_tracks_every_source():
    """The in-tree build rebuilds the library when any source or header of
    csrc/ (or the C-ABI header) is newer than it, and compiles the one
    translation unit that includes them all."""
    import build
    csrc = os.path.join(ROOT, "llama98-zh_b200", "csrc")
    files = {os.path.join(csrc, f) for f in os.listdir(csrc) if f.endswith((".cu", ".cuh", ".h"))}
    assert files <= set(build.DEPS)
    assert HEADER in build.DEPS
    engine = open(os.path.join(csrc, "lz98_engine.cu")).read()
    included = set(re.findall(r'#include "([^"]+)"', engine))
    for f in files:
        name = os.path.basename(f)
        if name.endswith(".cuh"):
            reach = name in included or any(
                name in open(os.path.join(csrc, g)).read() for g in included if os.path.exists(os.path.join(csrc, g)))
            assert reach, f"{name} is not included by the engine"
