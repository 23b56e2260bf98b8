"""Builds the sm_100a library `staleynet_b200/_lib/libsnb_b200.so` from `csrc/` with nvcc, in-tree.

    python -m staleynet_b200.build [--force] [--verbose-ptxas]

Each .cu file compiles to an object in parallel (`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`); the
objects link into one shared library with the CUDA runtime linked statically, so the library loads wherever the
driver is present. Rebuilds only when a source or header is newer than the library.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_PATH = LIB_DIR / "libsnb_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xcompiler", "-Wall"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _newest_input() -> float:
    files = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files if f.is_file())


def _compile(nvcc: str, src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stdout + res.stderr


def build_library(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compiles every CUDA source for sm_100a and links the shared library; returns its path."""
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= _newest_input():
        return LIB_PATH
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as pool:
        for obj, log in pool.map(lambda s: _compile(nvcc, s, verbose_ptxas), sources()):
            objs.append(obj)
            if verbose_ptxas and log.strip():
                print(log)
    tmp = LIB_PATH.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcuda"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        # libcuda.so may only exist as a stub at build time; the driver entry point is resolved at run time.
        cmd = [c for c in cmd if c != "-lcuda"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    path = build_library(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
