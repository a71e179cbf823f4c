"""Builds libvkb.so (and the bakeoff harness binary) in-tree for sm_100a with nvcc.

    python volta-kernel-bakeoff_b200/build.py          # incremental
    python volta-kernel-bakeoff_b200/build.py --force  # everything

Outputs: volta-kernel-bakeoff_b200/lib/libvkb.so, volta-kernel-bakeoff_b200/bin/bakeoff. Objects go to _build/.
The library links the CUDA runtime statically (nvcc's default) and NCCL and cuBLAS dynamically.
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
HOST = os.path.join(PKG, "host")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
BINDIR = os.path.join(PKG, "bin")
LIB = os.path.join(LIBDIR, "libvkb.so")
BAKEOFF = os.path.join(BINDIR, "bakeoff")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include")]

LIB_SOURCES = ["vkb_api.cu", "comm.cu", "gguf.cu", "dequant.cu", "formats.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, obj: str, extra: list[str]) -> None:
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _nccl_flags() -> list[str]:
    inc = ["-I/usr/include"] if os.path.exists("/usr/include/nccl.h") else []
    return inc


def build(force: bool = False, verbose: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for s in LIB_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, os.path.splitext(s)[0] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs.append((src, obj, _nccl_flags()))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            futs = [ex.submit(_compile, *j) for j in jobs]
            for f in futs:
                f.result()
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcuda", "-lnccl", "-lcublas"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"built {os.path.relpath(LIB, ROOT)}")
    harness = os.path.join(HOST, "bakeoff.cpp")
    if os.path.exists(harness):
        os.makedirs(BINDIR, exist_ok=True)
        hsrcs = glob.glob(os.path.join(HOST, "*.cpp")) + glob.glob(os.path.join(HOST, "*.h"))
        if force or _stale(BAKEOFF, hsrcs + hdrs + [LIB]):
            cmd = [nvcc()] + NVCC_FLAGS + ["-o", BAKEOFF, harness, "-L" + LIBDIR, "-lvkb", "-lcublas",
                                            "-Xlinker", "-rpath=$ORIGIN/../lib"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"harness build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
            if verbose:
                print(f"built {os.path.relpath(BAKEOFF, ROOT)}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    try:
        build(force=a.force)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
