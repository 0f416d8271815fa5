"""Builds libfrx.so (the sm_100a CUDA engine behind the C ABI in include/frx.h) in-tree.

Usage:  python fast-reduction_b200/build.py [--verbose] [--force] [--checked]

The library lands in fast-reduction_b200/fast_reduction/_native/libfrx.so, next to the
Python package that loads it with ctypes. Objects are rebuilt only when a source or header
is newer than the library (or with --force). --checked builds libfrx_checked.so with
FRX_CHECKED=1: every entry point verifies that each buffer it will touch lies inside a device
allocation, and device-side invariant checks report FRX_STATUS_CHECK_FAILED instead of touching
memory (FRX_LIB=checked makes the Python package load it).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
OUT_DIR = PKG_ROOT / "fast_reduction" / "_native"
LIB = OUT_DIR / "libfrx.so"
LIB_CHECKED = OUT_DIR / "libfrx_checked.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put it on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(lib: Path) -> bool:
    if not lib.exists():
        return True
    lib_mtime = lib.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > lib_mtime for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False, checked: bool = False) -> Path:
    lib = LIB_CHECKED if checked else LIB
    if not force and not _stale(lib):
        return lib
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-shared", "-o", str(tmp)]
    if checked:
        cmd.append("-DFRX_CHECKED=1")
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(s) for s in sources()]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    if verbose or ptxas_verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, lib)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills/smem per kernel")
    ap.add_argument("--checked", action="store_true", help="build libfrx_checked.so (FRX_CHECKED=1)")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose, checked=args.checked))


if __name__ == "__main__":
    main()
