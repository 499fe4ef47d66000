"""Build libgdnr.so (all CUDA sources of this directory) for sm_100a.

    python fp8-replayssm-gdn-kernel_b200/csrc/build.py [--verbose-ptxas] [--force]

Objects go to ``csrc/_build/``; the shared library is written next to the
Python host package (``gdnr/libgdnr.so``) so that it travels with the tree.
Incremental: a source is recompiled when it or any header is newer than its
object.
"""

from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
PKG = HERE.parent / "gdnr"
INCLUDE = HERE.parent.parent / "include"
BUILD = HERE / "_build"
TARGET = PKG / "libgdnr.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(HERE.glob("*.cu"))
    headers = list(HERE.glob("*.cuh")) + list(HERE.glob("*.h")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    objects = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
                and obj.stat().st_mtime >= newest_header):
            continue
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not TARGET.exists() or any(o.stat().st_mtime > TARGET.stat().st_mtime for o in objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(TARGET), *map(str, objects), "-lcuda"]
        print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return TARGET


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
