"""Build of the CUDA library liblz98gpu.so for sm_100a (in-tree, next to
this file).  -fmad=false keeps every float multiply and add separately
rounded, as the reference float tier is (its gcc build uses
-ffp-contract=off; the host side, which builds the RoPE table, is compiled
with it too); division and square root stay IEEE-rounded and
denormals are kept (no --use_fast_math, no -ftz)."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SO = os.path.join(HERE, "liblz98gpu.so")
SRCS = [os.path.join(HERE, "csrc", "lz98_engine.cu")]
# every source and header of csrc/ (the engine includes them all) and the C ABI header
DEPS = SRCS + sorted(os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))
                     if f.endswith((".cu", ".cuh", ".h"))) + [os.path.join(ROOT, "include", "lz98_gpu.h")]

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off", "-shared", "-Xlinker", "-Bsymbolic",
]


def needs_build() -> bool:
    if not os.path.exists(SO):
        return True
    t = os.path.getmtime(SO)
    return any(os.path.getmtime(d) > t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if force or needs_build():
        nvcc = os.environ.get("NVCC", "nvcc")
        cmd = [nvcc, *NVCC_FLAGS, "-o", SO + ".tmp", *SRCS, "-lcudart", "-ldl"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(SO + ".tmp", SO)
    return SO


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
