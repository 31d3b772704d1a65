"""Build ``gpa_b200/libgpa_b200.so`` (sm_100a) in-tree with nvcc.

    python -m gpa_b200.build [--debug] [--verbose] [--jobs N]

Each CUDA source compiles to its own object (in parallel) under
``gpa_b200/_build/``; one nvcc link step writes the shared library.  The library
has a plain C ABI (include/gpa_b200.h) and links the CUDA runtime statically,
so it carries no dependency on torch's own CUDA libraries.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
SOURCES = ("api.cu", "decode.cu", "gdn.cu", "gdn_tc.cu", "level.cu", "level_tc.cu", "tc5_probe.cu",
           "gdn_tc5.cu", "moments.cu", "outer_tc5.cu")
OUTPUT = os.path.join(HERE, "libgpa_b200.so")
OBJDIR = os.path.join(HERE, "_build")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def build(debug: bool = False, verbose: bool = False, extra=(), jobs: int | None = None) -> str:
    nvcc = nvcc_path()
    os.makedirs(OBJDIR, exist_ok=True)
    flags = ["-std=c++20", "-O3", "-lineinfo", ARCH, "-Xcompiler", "-fPIC", *extra]
    if debug:
        flags.append("-DGPA_DEBUG=1")
    if verbose:
        flags += ["-Xptxas", "-v"]

    def compile_one(src: str) -> str:
        obj = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".o")
        subprocess.run([nvcc, *flags, "-c", "-o", obj, os.path.join(CSRC, src)], check=True)
        return obj

    jobs = jobs or min(len(SOURCES), os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    subprocess.run([nvcc, ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", OUTPUT, *objs],
                   check=True)
    return OUTPUT


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    print(build(args.debug, args.verbose, jobs=args.jobs))


if __name__ == "__main__":
    sys.exit(main())
