"""Builds libblk_world.so in-tree for sm_100a with nvcc.

    python blocklab_b200/build.py [--verbose-ptxas]

The library is written next to this file (blocklab_b200/libblk_world.so) so it
travels with the source tree; it is rebuilt when any source is newer.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libblk_world.so")
SOURCES = ["blk_light.cu", "blk_relight.cu", "blk_api.cu", "blk_render.cu"]
HEADERS = ["blk_common.cuh", "blk_bits.cuh", "blk_internal.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(ROOT, "include", "blk_world.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and not verbose_ptxas and up_to_date():
        return LIB
    cmd = [nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC", "-shared",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp"]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    cmd += ["-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libblk_world.so")
    if verbose_ptxas:
        sys.stderr.write(res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))


if __name__ == "__main__":
    main()
