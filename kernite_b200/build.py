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


# The sources whose kernels also ship as a module image inside the library (kq_module_image):
# compiled a second time to an sm_100a cubin and embedded as read-only data.
IMAGE_SOURCES = {"kq_warpmma.cu": "kq_image_warpmma"}


def _image_asm(symbol: str, cubin: str) -> str:
    return (f"\t.section .rodata\n\t.balign 64\n\t.global {symbol}\n\t.type {symbol}, @object\n"
            f"{symbol}:\n\t.incbin \"{cubin}\"\n\t.global {symbol}_end\n{symbol}_end:\n"
            f"\t.section .note.GNU-stack,\"\",@progbits\n")


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(BUILD, exist_ok=True)
    jobs, objs = [], []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        jobs.append(cmd)
        objs.append(obj)
        sym = IMAGE_SOURCES.get(os.path.basename(src))
        if sym:
            cubin = os.path.join(BUILD, os.path.basename(src) + ".cubin")
            jobs.append([nvcc(), *ARCH, "-O3", "-std=c++17", "--expt-relaxed-constexpr",
                         "-I", INCLUDE, "-I", CSRC, "-cubin", src, "-o", cubin])
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for r in pool.map(lambda c: subprocess.run(c, capture_output=not verbose, text=True), jobs):
            if r.returncode:
                raise RuntimeError(f"{' '.join(r.args)}\n{r.stdout or ''}{r.stderr or ''}")
    for src, sym in IMAGE_SOURCES.items():
        cubin = os.path.join(BUILD, src + ".cubin")
        asm = os.path.join(BUILD, sym + ".S")
        with open(asm, "w") as f:
            f.write(_image_asm(sym, cubin))
        obj = os.path.join(BUILD, sym + ".o")
        subprocess.run(["gcc", "-c", asm, "-o", obj], check=True)
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
