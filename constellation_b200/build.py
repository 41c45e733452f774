"""Builds the in-tree CUDA library ``constellation_b200/libconstellation_b200.so`` for sm_100a.

    python -m constellation_b200.build        (or __graft_entry__.build())

nvcc compiles every ``csrc/*.cu`` with ``-gencode arch=compute_100a,code=sm_100a`` and links
one shared library that exports the C ABI of ``include/constellation_b200.h``.  Objects go
to ``constellation_b200/_build/``; the build is skipped when nothing changed.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libconstellation_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", *ARCH]


def nvcc() -> str:
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(cand) if cand.is_file() else "nvcc"


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.is_file():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, extra_flags=()) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            cmd = [nvcc(), *NVCC_FLAGS, *extra_flags, "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(src),
                   "-o", str(obj)]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)
        return r

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if jobs or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        run(cmd)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
