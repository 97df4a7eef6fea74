"""Builds libnavsampler.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library is plain CUDA C++ with an extern "C" surface (include/navsampler.h);
no torch types cross it, so it is compiled directly with nvcc rather than as a
torch extension. Cross-compiles without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libnavsampler.so")
OBJDIR = os.path.join(HERE, "_build")
DEPS = [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))] + [
    os.path.join(ROOT, "include", "navsampler.h")]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]
# translation unit -> its own floating-point flags
UNITS = {
    # every float expression that decides a token must round exactly as written
    "navsampler.cu": ["-fmad=false"],
    # the reference's softmax is compiled with nvcc's default contraction; so is ours
    "softmax_rows.cu": [],
}
def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in DEPS if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OBJDIR, exist_ok=True)
    objs = []
    for unit, flags in UNITS.items():
        obj = os.path.join(OBJDIR, unit.replace(".cu", ".o"))
        cmd = [nvcc(), *COMMON, *flags, "-c", "-o", obj, os.path.join(HERE, "csrc", unit)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", LIB, *objs], check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
