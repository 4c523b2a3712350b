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
OBJ_DIR = os.path.join(HERE, "_build")

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


def _compile(src: str, obj: str, verbose_ptxas: bool) -> subprocess.CompletedProcess:
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", "-c", "-o", obj, src]
    cmd = [c for c in cmd if c != "-shared"]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    return subprocess.run(cmd, capture_output=True, text=True)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile every ``csrc/*.cu`` to an object (in parallel, one nvcc per
    source; each is its own translation unit as in one combined nvcc call)
    and link them into ``libdwa.so``."""
    if not force and up_to_date():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    objs = [os.path.join(OBJ_DIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    t_hdr = max([os.path.getmtime(h) for h in headers] + [os.path.getmtime(__file__)])

    def stale(so):
        src, obj = so
        return force or verbose_ptxas or not os.path.exists(obj) or \
            os.path.getmtime(obj) < max(t_hdr, os.path.getmtime(src))

    todo = [so for so in zip(srcs, objs) if stale(so)]
    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        procs = list(ex.map(lambda so: _compile(so[0], so[1], verbose_ptxas), todo))
    srcs = [so[0] for so in todo]
    failed = [(s, p) for s, p in zip(srcs, procs) if p.returncode != 0]
    for s, p in failed:
        sys.stderr.write(f"--- {os.path.basename(s)}\n" + p.stdout + p.stderr)
    if failed:
        raise RuntimeError("nvcc failed building libdwa.so")
    if verbose_ptxas:
        for s, p in zip(srcs, procs):
            sys.stderr.write(f"--- {os.path.basename(s)}\n" + p.stderr)
    link = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB + ".tmp", *objs, "-lcudart"]
    proc = subprocess.run(link, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("linking libdwa.so failed")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas))
