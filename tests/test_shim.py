"""The reference-side shim (llama98-zh_b200/shim/lz98_gpu_shim.c) as a
reference maintainer would build it: compiled with gcc against the
reference's own headers and include/lz98_gpu.h, the reference's LZSampler
layout equal to the library header's field for field, and the model-free
acceptance entry points reached through the shim's run-time binding (no
GPU needed).  The GPU half (a generation through the shim) is in
test_gpu_boundary.py."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
SHIM = os.path.join(ROOT, "llama98-zh_b200", "shim")
ABI_C = os.path.join(ROOT, "tests", "abi_c")
SO = os.path.join(ROOT, "llama98-zh_b200", "liblz98gpu.so")
REF_SRC = os.path.join(os.environ.get("LZ98_REFERENCE_DIR", os.path.join(os.path.dirname(ROOT), "reference")), "src")


def gcc(args, tmp_path):
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-Wno-unused-parameter", *args],
                       cwd=tmp_path, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return r


@pytest.mark.skipif(not os.path.isdir(REF_SRC), reason="reference sources not present")
def test_shim_compiles_in_the_reference_tree(tmp_path):
    """With the reference's src/ on the include path the shim takes the
    reference's own LZSampler (sampler.h) and still compiles warning-free."""
    gcc(["-I" + INC, "-I" + SHIM, "-I" + REF_SRC, "-c", os.path.join(SHIM, "lz98_gpu_shim.c"), "-o",
         str(tmp_path / "shim_ref.o")], tmp_path)


@pytest.mark.skipif(not os.path.isdir(REF_SRC), reason="reference sources not present")
def test_sampler_layout_matches_reference(tmp_path):
    """Every LZSampler / LZSampleParams field sits at the same offset, and
    the structs have the same sizes, under both headers."""
    exe = str(tmp_path / "layout")
    subprocess.run(["gcc", "-std=c99", "-I" + REF_SRC, "-I" + ABI_C, "-c", os.path.join(ABI_C, "layout_ref.c"),
                    "-o", str(tmp_path / "a.o"), "-w"], check=True)
    gcc(["-I" + INC, "-I" + ABI_C, "-c", os.path.join(ABI_C, "layout_ours.c"), "-o", str(tmp_path / "b.o")],
        tmp_path)
    gcc([os.path.join(ABI_C, "layout_main.c"), str(tmp_path / "a.o"), str(tmp_path / "b.o"), "-o", exe], tmp_path)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.startswith("same 22"), out.stdout


def test_shim_binds_the_library_at_run_time(tmp_path):
    """The shim built against lz98_gpu.h alone, linked with a driver, opens
    liblz98gpu.so with dlopen and answers the model-free acceptance cases
    exactly as the reference's contract (src/generate.c:232-349) does."""
    import build
    build.build()                                # no-op when the library is up to date
    exe = str(tmp_path / "shim_main")
    gcc(["-I" + INC, "-I" + SHIM, os.path.join(SHIM, "lz98_gpu_shim.c"), os.path.join(ABI_C, "shim_main.c"),
         "-o", exe, "-ldl"], tmp_path)
    out = subprocess.run([exe, SO, "accept"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.split("\n")
    assert lines[0] == "accept 2 5 7 1"          # rejection at the third draft
    assert lines[1] == "accept 3 5 7 9 11"       # all accepted, bonus appended
    assert lines[2] == "temp 1 1"                # p/q = 3 > u: accepted
    tok, acc, rng = lines[3].split()[1:]
    assert acc == "0" and tok in ("1", "2") and rng != "42"   # residual sample advanced the generator
