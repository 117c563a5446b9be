"""Builds libkq.so in-tree: every CUDA source of kernite_b200/csrc, compiled by nvcc for sm_100a.

    python -m kernite_b200.build [--verbose]

The library links the CUDA runtime statically, so it carries no dependency on the runtime
version that torch bundles; it runs in the GPU's primary context, the one torch and kernite-cuda
use, so their device pointers and streams are valid here.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libkq.so")
BUILD = os.path.join(ROOT, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
         "-cudart", "static"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps += glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(verbose=args.verbose, force=args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
