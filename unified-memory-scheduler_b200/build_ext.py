"""Builds libumsx.so in-tree with nvcc for sm_100a (no JIT cache, no torch extension).

Each source compiles to its own object under _build/ (in parallel, only when it or a header
changed), then nvcc links the shared library next to this file.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "..", "_build", "umsx")
LIB = os.path.join(PKG, "libumsx.so")
SOURCES = ["umsx_api.cu", "umsx_kernels.cu", "umsx_decode.cu", "umsx_gguf.cpp", "umsx_prefill.cu", "umsx_static.cu", "umsx_ep.cu"]
HEADERS = ["umsx_internal.h", "umsx_device.cuh", "umsx_mx.cuh", "umsx_tc.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-c",
           "-Xptxas", "-v" if verbose else "-O3", "-o", obj + ".tmp", src]
    res = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)} ({res.returncode}):\n{res.stderr[-6000:]}")
    os.replace(obj + ".tmp", obj)
    return res.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(PKG, "..", "include", "umsx.h")]
    jobs = []
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJ, s + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for log in ex.map(lambda j: _compile(j[0], j[1], verbose), jobs):
            if verbose and log:
                print(log)
    if force or jobs or _stale(LIB, objs):
        res = subprocess.run([nvcc(), *ARCH, "-shared", "-o", LIB + ".tmp", *objs], capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stderr[-6000:]}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
