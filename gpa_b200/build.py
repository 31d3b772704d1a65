"""Build ``gpa_b200/libgpa_b200.so`` (sm_100a) in-tree with nvcc.

    python -m gpa_b200.build [--debug]

The library has a plain C ABI (include/gpa_b200.h) and links the CUDA runtime
statically, so it carries no dependency on torch's own CUDA libraries.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
SOURCES = ("api.cu", "decode.cu", "gdn.cu", "gdn_tc.cu", "level.cu", "level_tc.cu")
OUTPUT = os.path.join(HERE, "libgpa_b200.so")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def build(debug: bool = False, verbose: bool = False, extra=()) -> str:
    cmd = [nvcc_path(), "-std=c++20", "-O3", "-lineinfo", ARCH, "-Xcompiler", "-fPIC", "-shared",
           "-o", OUTPUT, *(os.path.join(CSRC, s) for s in SOURCES), *extra]
    if debug:
        cmd.append("-DGPA_DEBUG=1")
    if verbose:
        cmd += ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    return OUTPUT


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(args.debug, args.verbose))


if __name__ == "__main__":
    sys.exit(main())
