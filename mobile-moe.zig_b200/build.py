"""Build libkvcuda.so (in-tree) with nvcc for sm_100a.

    python mobile-moe.zig_b200/build.py [--verbose] [--ptxas-v]

Each csrc/*.cu is compiled separately into _build/ and linked into
mobile-moe.zig_b200/libkvcuda.so.  No fast-math: the Q8_0 arithmetic must
round exactly like the reference's CPU code (IEEE division, round-half-away).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build", "kvcuda")
LIB = os.path.join(HERE, "libkvcuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libkvcuda.so")


def _digest(src: str) -> str:
    """Content hash of a source, every header it may include and the flags (a
    checkout can leave any mtimes, so reuse is decided by content)."""
    h = hashlib.sha256()
    deps = [src] + sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")))
    deps.append(os.path.join(ROOT, "include", "kvcuda.h"))
    for d in deps:
        h.update(d.encode())
        with open(d, "rb") as f:
            h.update(f.read())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()


def _compile(src: str, ptxas_v: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    stamp = obj + ".sha256"
    digest = _digest(src)
    if os.path.exists(obj) and os.path.exists(stamp) and not ptxas_v:
        with open(stamp) as f:
            if f.read().strip() == digest:
                return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    with open(stamp, "w") as f:
        f.write(digest)
    return obj, r.stdout + r.stderr


def build(verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_v), srcs))
    objs = [o for o, _ in results]
    if verbose or ptxas_v:
        for _, log in results:
            if log:
                print(log)
    # relink when any object changed (by content) or the library is missing
    link_digest = hashlib.sha256("".join(open(o + ".sha256").read() for o in objs).encode()).hexdigest()
    lib_stamp = os.path.join(BUILD, "libkvcuda.so.sha256")
    old = open(lib_stamp).read().strip() if os.path.exists(lib_stamp) else ""
    if not os.path.exists(LIB) or old != link_digest:
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        with open(lib_stamp, "w") as f:
            f.write(link_digest)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_v))
    sys.exit(0)
