"""Builds the sm_100a shared library libgsqrco_b200.so in-tree (gsq_rco_mlx_b200/lib/).

nvcc cross-compiles without a GPU. Usage: python -m gsq_rco_mlx_b200.build [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libgsqrco_b200.so"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--shared",
         "-Xptxas", "-v", "--expt-relaxed-constexpr"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-o", str(tmp),
           *[str(s) for s in sources()]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = LIB_DIR / "build.log"
    log.write_text(r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(r.stderr[-8000:])
        raise RuntimeError(f"nvcc failed ({r.returncode}); see {log}")
    os.replace(tmp, LIB)
    if verbose:
        print(r.stderr[-4000:])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
