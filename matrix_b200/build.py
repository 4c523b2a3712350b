"""Build libdwa.so (all CUDA sources under csrc/) for sm_100a, in-tree.

    python -m matrix_b200.build [--verbose-ptxas]

The library is written next to this file (``matrix_b200/libdwa.so``) so it
travels with the source tree; it is rebuilt only when a source is newer.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.abspath(os.path.join(HERE, "..", "include"))
LIB = os.path.join(HERE, "libdwa.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return all(os.path.getmtime(p) <= t for p in deps)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", "-o", LIB + ".tmp", *sources(), "-lcudart"]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libdwa.so")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas))
