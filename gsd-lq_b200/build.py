"""Build ``libgsdlq_cuda.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m gsdlq_b200.build`` (from the repository root) or
``gsdlq_b200.build.build_library()``.  Objects go to ``_build/`` next to the
sources; the shared library lands in the package directory, where ``_lib``
loads it.  Rebuilds only what changed (by modification time).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libgsdlq_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-rdc=true",
              "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps(src: str) -> list[str]:
    return [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(verbose: bool = False, extra_flags: list[str] | None = None, ptxas_v: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    cc = nvcc()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    flags = NVCC_FLAGS + ARCH + (extra_flags or []) + (["-Xptxas", "-v"] if ptxas_v else [])
    jobs = []
    for s in srcs:
        o = os.path.join(OBJDIR, os.path.basename(s) + ".o")
        if ptxas_v or _stale(o, _deps(s)):
            jobs.append([cc, "-c", s, "-o", o] + flags)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode != 0 or ptxas_v:
                sys.stdout.write(" ".join(cmd[:3]) + "\n" + r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {cmd[2]}")
    objs = [os.path.join(OBJDIR, os.path.basename(s) + ".o") for s in srcs]
    if jobs or _stale(LIB, objs):
        cmd = [cc, "-shared", "-o", LIB] + objs + ARCH + ["-Xcompiler", "-fPIC", "-rdc=true", "-lcudart_static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build_library(verbose=True, ptxas_v="-v" in sys.argv))
