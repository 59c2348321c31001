"""Build libwalsh.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m walsh_research_b200.build [--force] [-j N]

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (skipped when
the object is newer than its sources), then linked into
``walsh_research_b200/libwalsh.so``.  Only ``sm_100a`` code is generated.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libwalsh.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + INCLUDE, "-I" + CSRC]
# developer hook: extra nvcc arguments (e.g. -D tuning constants); objects are
# not rebuilt when only these change, so delete the affected _build/*.o first
FLAGS += os.environ.get("WALSH_NVCC_FLAGS", "").split()


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if _stale(obj, [src] + _deps()):
        cmd = [nvcc()] + ARCH + FLAGS + extra + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 8, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    extra = list(extra or [])
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(force=a.force or a.ptxas_verbose, jobs=a.j, extra=extra))


if __name__ == "__main__":
    main()
