"""Build libdeltacore.so in-tree for sm_100a with nvcc.

    python burn-deltanet_b200/build.py          # incremental (skips when up to date)
    python burn-deltanet_b200/build.py --force

The library is the C ABI of include/deltacore.h.  It is built in the package
directory so it travels with the source tree; nothing is installed.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdeltacore.so")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the delta-rule core needs the CUDA toolkit to build")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + [os.path.join(ROOT, "include", "deltacore.h")])


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [
        nvcc(), ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-v" if verbose else "-O3",
        "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
        os.path.join(CSRC, "deltacore.cu"), "-o", LIB + ".tmp", "-lcuda",
    ]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
