"""Build the in-tree C-ABI library ``logkv_b200/liblogkv_b200.so`` for sm_100a with nvcc.

Three translation units with different numerics:
  flush.cu      -fmad=false: every float expression of the flush is rounded
                 exactly as written (bit-exact with the reference's CPU path);
  attention.cu  default contraction (FMA) for the attention math;
  plugin.cu     -fmad=false: the operator-level plugin functions, same contract as flush.cu.
Run ``python -m logkv_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "liblogkv_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          f"-I{ROOT}", "--expt-relaxed-constexpr"]

UNITS = [
    ("flush.cu", ["-fmad=false"]),
    ("attention.cu", []),
    ("plugin.cu", ["-fmad=false"]),
    ("unified.cu", ["-fmad=false"]),
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build logkv_b200")
    return path


def sources_newer_than(target: str) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    for root in (CSRC, os.path.join(ROOT, "include")):
        for name in os.listdir(root):
            if os.path.getmtime(os.path.join(root, name)) > t:
                return True
    return False


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not sources_newer_than(LIB):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for unit, extra in UNITS:
        src = os.path.join(CSRC, unit)
        if not os.path.exists(src):
            continue
        obj = os.path.join(objdir, unit.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *COMMON, *extra, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
