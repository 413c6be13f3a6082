"""Build the in-tree CUDA library ``libnifre_b200.so`` for sm_100a.

``python -m nifre_b200.build`` (or ``build()`` from Python) compiles every
``csrc/*.cu`` with nvcc into object files under ``nifre_b200/_build`` and links
them into ``nifre_b200/libnifre_b200.so``.  Sources are rebuilt only when a
source or header is newer than its object.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libnifre_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the nifre_b200 CUDA library cannot be built")


def _newest_header() -> float:
    heads = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in heads), default=0.0)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr = _newest_header()
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or ptxas_verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
    objs = [str(BUILD / (s.stem + ".o")) for s in sources]
    if jobs or not LIB.exists():
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("linking libnifre_b200.so failed")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
