"""Builds libgnnc_b200.so (the CUDA runtime behind include/gnnc_b200.h) in-tree.

    python ml-reentry-mlir_b200/build_ext.py [--force] [-j N]

Every csrc/*.cu is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`)
and linked with the static CUDA runtime into gnnc/b200/libgnnc_b200.so, next to the
Python bindings that load it. Objects go to csrc/_build/. A target is rebuilt when any
source or header is newer than it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
BUILD = CSRC / "_build"
INCLUDE = REPO_ROOT / "include"
LIB = PKG_ROOT / "gnnc" / "b200" / "libgnnc_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-diag-suppress",
    "177",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile and link; returns the library path. Raises on compiler failure."""
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    exe = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [exe, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}{res.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, sources))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [exe, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static", "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
