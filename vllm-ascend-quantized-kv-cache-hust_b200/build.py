"""Builds libqkv_sm100.so (the sm_100a kernels behind qkv_b200) in-tree.

Every ``csrc/*.cu`` file (and host-only ``csrc/*.cpp``) is compiled by nvcc
for ``sm_100a`` into
``_build/*.o`` (incrementally, in parallel) and linked into
``qkv_b200/libqkv_sm100.so`` with the CUDA runtime linked statically, so the
library only needs the NVIDIA driver at run time.

Usage: ``python build.py [-v] [--force]`` or ``build.build_library()``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD_DIR = HERE / "_build"
LIB_PATH = HERE / "qkv_b200" / "libqkv_sm100.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def _compile(src: Path, obj: Path, verbose: bool, ptxas_verbose: bool) -> str:
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build_library(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles stale objects and (re)links the shared library; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_verbose or _stale(obj, src, headers):
            jobs.append((src, obj))
    logs = []
    if jobs:
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with futures.ThreadPoolExecutor(workers) as pool:
            for src, log in zip(
                [j[0] for j in jobs],
                pool.map(lambda j: _compile(j[0], j[1], verbose, ptxas_verbose), jobs),
            ):
                if log.strip():
                    logs.append(f"--- {src.name}\n{log}")
    relink = force or bool(jobs) or not LIB_PATH.exists() or any(
        o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs
    )
    if relink:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    if logs and (verbose or ptxas_verbose):
        print("\n".join(logs), file=sys.stderr)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    path = build_library(args.verbose, args.force, args.ptxas_verbose)
    print(path)


if __name__ == "__main__":
    main()
