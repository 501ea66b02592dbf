"""Build libpab200.so in-tree with nvcc for sm_100a.

    python -m pagedattention_b200.build [--verbose]

The shared library lands next to this file (pagedattention_b200/libpab200.so),
which is where ``pagedattention_b200._lib`` loads it from.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libpab200.so"
SOURCES = [CSRC / "pab200.cu"]
HEADERS = [CSRC / "decode.cuh", CSRC / "ptx.cuh", REPO_DIR / "include" / "pab200.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libpab200.so")
    return cand


def nvcc_command(out: Path, verbose_ptxas: bool = False) -> list[str]:
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
        "-I", str(REPO_DIR / "include"), "-I", str(CSRC),
        "-o", str(out), *map(str, SOURCES),
    ]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    return cmd


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = nvcc_command(tmp, verbose_ptxas=verbose)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
