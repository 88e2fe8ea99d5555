"""Builds libtt_b200.so in-tree with nvcc for sm_100a.

    python -m tiktoktechjam2026_b200.build [--force] [--verbose]

The library is a plain C-ABI shared object (no PyTorch types cross its
boundary); Python reaches it through ctypes.  It is built next to this file so
that it travels with the source tree.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
MAIN_SRC = os.path.join(CSRC, "tt_b200.cu")
LIB_PATH = os.path.join(PKG_DIR, "libtt_b200.so")
HEADER = os.path.join(REPO_DIR, "include", "tt_b200.h")

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=default",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(home, "bin", "nvcc")
    if os.path.exists(path):
        return path
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _sources() -> list:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))) + [HEADER]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library unless it is newer than every source; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = [_nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-o", tmp, MAIN_SRC]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libtt_b200.so")
    if verbose:
        sys.stderr.write(proc.stdout + proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
