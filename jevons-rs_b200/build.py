"""Builds libjk.so (the C ABI of include/jk.h) in-tree for sm_100a with nvcc.

    python jevons-rs_b200/build.py [--force] [-j N]

Every CUDA translation unit under csrc/ is compiled to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into
``jevons_kernels/libjk.so``; the CUDA runtime is linked statically so the library only needs the
driver at run time. Objects go to ``_build/`` (git-ignored).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "jevons_kernels", "libjk.so")
INCLUDE = os.path.join(REPO, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "-Xcompiler", "-ffp-contract=off",
    "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE,
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, obj: str, extra) -> str:
    cmd = [nvcc()] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int = 8, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = headers()
    objs, todo = [], []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = {ex.submit(_compile, s, o, extra): s for s, o in todo}
            for f in cf.as_completed(futs):
                log = f.result()
                if verbose and log:
                    print(log, file=sys.stderr)
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-lcuda"]
        # libcuda is resolved at run time from the driver; link against the stub when present.
        stub = "/usr/local/cuda/lib64/stubs"
        if os.path.isdir(stub):
            cmd += ["-L", stub]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage (-Xptxas -v)")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, jobs=a.j, verbose=a.v or a.ptxas_v, extra=extra))
