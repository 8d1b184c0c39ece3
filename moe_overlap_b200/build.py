"""Builds the in-tree C-ABI library ``libmoe_overlap_b200.so`` for sm_100a.

Every ``csrc/*.cu`` file is compiled by nvcc into ``_build/`` at the repository
root and linked into ``moe_overlap_b200/libmoe_overlap_b200.so``.  The CUDA
runtime is linked statically and the driver API is reached through
``cudaGetDriverEntryPoint``, so the library loads (and its symbols can be
inspected) on a machine without a GPU or driver.

Usage: ``python -m moe_overlap_b200.build [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIB_NAME = "libmoe_overlap_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the library")
    return cand


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, force: bool, verbose: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.stem + ".o")
    if (
        not force
        and obj.exists()
        and obj.stat().st_mtime >= max(src.stat().st_mtime, _deps_mtime())
    ):
        return obj, ""
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, (proc.stdout + proc.stderr) if verbose else ""


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles (if stale) and links the library; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose), sources))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            print(log, file=sys.stderr)
    if (
        not force
        and LIB_PATH.exists()
        and LIB_PATH.stat().st_mtime >= max(o.stat().st_mtime for o in objs)
    ):
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
