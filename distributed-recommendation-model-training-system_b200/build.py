"""Builds libeps_b200.so in-tree with nvcc for sm_100a (B200).

Usage: python build.py [--force]

Every object is compiled with ``-gencode arch=compute_100a,code=sm_100a`` and
``--fmad=false`` (no FMA contraction anywhere on the parity path, as in the
reference's CUDA build) and linked into one shared library whose only exported
symbols are the ``eps_b200_*`` entry points declared in include/eps_b200.h.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libeps_b200.so")

SOURCES = ["store.cu", "lookup.cu", "sort.cu", "push.cu", "route.cu", "noalloc.cu", "runtime.cu",
           "comm.cu", "client.cu", "sync.cu", "runtime_api.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    headers.append(os.path.join(INCLUDE, "eps_b200.h"))
    objs = []
    procs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [nvcc(), *ARCH, *FLAGS, "-c", path, "-o", obj]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                                stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    if force or _stale(LIB, objs):
        # static cudart: the library needs only the driver (libcuda) at run time
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-ldl"]
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
