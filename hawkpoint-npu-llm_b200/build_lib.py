#!/usr/bin/env python3
"""Build libhawkb200.so in-tree for sm_100a (B200) with nvcc.

    python hawkpoint-npu-llm_b200/build_lib.py [--verbose-ptxas]

The library lands in hawkpoint-npu-llm_b200/lib/ so it travels with the
repository snapshot; nothing is installed into site-packages.
"""

import argparse
import os
from pathlib import Path
import shutil
import subprocess
import sys

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libhawkb200.so"
SOURCES = [CSRC / "hb_engine.cu", CSRC / "hb_batch.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO / "include" / "hawkb200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for candidate in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found (set NVCC)")


def up_to_date():
    if not LIB.exists():
        return False
    built = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in SOURCES + HEADERS + [Path(__file__)])


def build(force=False, verbose_ptxas=False, quiet=False):
    if not force and not verbose_ptxas and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-O2", "-shared",
        "-I", str(REPO / "include"), "-I", str(CSRC),
        "-o", str(tmp), *map(str, SOURCES),
    ]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    args = parser.parse_args()
    try:
        print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))
    except subprocess.CalledProcessError as exc:
        sys.exit(exc.returncode)
