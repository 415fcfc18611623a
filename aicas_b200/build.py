"""Builds the sm_100a shared library ``aicas_b200/lib/libaicas_b200.so``.

The library is a plain C-ABI object (no torch headers, no Python): every kernel
source under ``aicas_b200/csrc`` is compiled by nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and linked with the static CUDA
runtime, so any host language can bind it through ``include/aicas_b200.h``.

Usage: ``python -m aicas_b200.build [--force] [--verbose]``.
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
LIB_DIR = PKG_DIR / "lib"
OBJ_DIR = REPO_DIR / "_build" / "obj"
LIB_PATH = LIB_DIR / "libaicas_b200.so"
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
    "-O3",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build aicas_b200")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO_DIR / "include").glob("*.h"))


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool, ptxas_verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(REPO_DIR / "include"), "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if ptxas_verbose or verbose:
        sys.stdout.write(res.stdout + res.stderr)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles what changed and links the shared library; returns its path."""
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objs = []
    for src in _sources():
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        stale = (
            force
            or ptxas_verbose
            or not obj.exists()
            or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        )
        if stale:
            jobs.append((src, obj))
    if jobs:
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(workers) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose, ptxas_verbose) for s, o in jobs]
            for f in futs:
                f.result()
    if jobs or not LIB_PATH.exists():
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills/shared memory per kernel")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
