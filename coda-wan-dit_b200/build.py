"""Build libwdit.so (sm_100a) in-tree with nvcc.

    python coda-wan-dit_b200/build.py [--verbose]

The shared library is written next to this file so it travels with the source tree
(it is git-ignored). Rebuilds only when a source under csrc/ or include/ is newer.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libwdit.so"
SOURCES = ["gemm.cu", "aux.cu", "comm.cu", "p2p.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the wdit CUDA library cannot be built")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))
    return files


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs() if p.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not needs_build():
        return LIB_PATH
    cmd = [
        _nvcc(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC",
        "-I",
        str(ROOT / "include"),
        "-o",
        str(LIB_PATH) + ".tmp",
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {LIB_PATH.name}")
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
