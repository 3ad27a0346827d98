"""Builds the sm_100a shared library libgsqrco_b200.so in-tree (gsq_rco_mlx_b200/lib/).

nvcc cross-compiles without a GPU. Each .cu file compiles to its own object (in parallel, and
only when it or a header is newer than its object), then one nvcc call links the library.
Usage: python -m gsq_rco_mlx_b200.build [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = PKG / "_build"
LIB = LIB_DIR / "libgsqrco_b200.so"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
         "--expt-relaxed-constexpr"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _stale() -> bool:
    if not LIB.exists():
        return True
    return _newest(list(sources()) + _headers()) > LIB.stat().st_mtime


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _compile(src: Path, force: bool, hdr_time: float):
    obj = OBJ_DIR / (src.stem + ".o")
    if (not force and obj.exists()
            and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time)):
        return src, 0, ""
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r.returncode, r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    OBJ_DIR.mkdir(exist_ok=True)
    hdr_time = _newest(_headers())
    srcs = sources()
    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda s: _compile(s, force, hdr_time), srcs))
    log_text = "".join(f"== {s.name}\n{out}" for s, _, out in results)
    log = LIB_DIR / "build.log"
    failed = [s.name for s, rc, _ in results if rc != 0]
    if failed:
        log.write_text(log_text)
        sys.stderr.write(log_text[-8000:])
        raise RuntimeError(f"nvcc failed on {failed}; see {log}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "--shared", "-o", str(tmp),
           *[str(OBJ_DIR / (s.stem + ".o")) for s in srcs]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(log_text + "== link\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(r.stderr[-8000:])
        raise RuntimeError(f"nvcc link failed ({r.returncode}); see {log}")
    os.replace(tmp, LIB)
    if verbose:
        print(log_text[-4000:])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
