"""Builds libb200_decode.so in-tree with nvcc for sm_100a.

    python llama-cpp-ascend310b4-addon_b200/build.py [--force]

The library holds every CUDA kernel of the decode path, the C ABI declared in
include/b200_decode.h and the native host runtime (graph runner, decode
driver, NCCL tensor parallelism).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libb200_decode.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = [
    "kernels.cu",
    "host.cpp",
    "model.cpp",
    "upload.cpp",
    "graph.cpp",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _deps(src: str) -> list[str]:
    """The source and the headers it may include: host .cpp files see only
    the .h headers; the device unit (.cu) sees every header."""
    host = src.endswith(".cpp")
    own = [os.path.join(CSRC, f) for f in os.listdir(CSRC)
           if f == src or f.endswith(".h") or (not host and f.endswith(".cuh"))]
    return own + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]


def _compile(src: str, force: bool) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    if not force and os.path.exists(obj):
        newest = max(os.path.getmtime(d) for d in _deps(src))
        if os.path.getmtime(obj) >= newest:
            return obj
    cmd = [nvcc()] + ARCH + COMMON + ["-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(SOURCES))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lnccl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


def build_ggml_backend(ggml_dir: str, verbose: bool = False) -> str:
    """libggml-b200.so: the ggml backend adapter (ggml-b200/ggml-b200.cpp)
    compiled against an upstream ggml tree (llama.cpp 37b3a9e0's ggml/, which
    holds include/ggml*.h and src/ggml-backend-impl.h) and linked to
    libb200_decode.so.  Upstream ggml is not part of this repository, so this
    runs only when its path is given (or GGML_DIR is set)."""
    lib = build(verbose=False)
    out = os.path.join(HERE, "libggml-b200.so")
    inc = [os.path.join(ggml_dir, "include"), os.path.join(ggml_dir, "src")]
    for d in inc:
        if not os.path.isdir(d):
            raise RuntimeError(f"{d} not found: --ggml-dir must be a ggml source tree")
    cmd = ([shutil.which("g++") or "g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I" + INCLUDE] +
           ["-I" + d for d in inc] + ["-I/usr/local/cuda/include", os.path.join(HERE, "ggml-b200", "ggml-b200.cpp"),
                                      "-o", out, "-L" + HERE, "-lb200_decode", "-Wl,-rpath,$ORIGIN",
                                      "-L/usr/local/cuda/lib64", "-lcudart"])
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ggml backend build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ggml-dir", default=os.environ.get("GGML_DIR"),
                    help="upstream ggml tree: also build the ggml backend adapter libggml-b200.so")
    a = ap.parse_args()
    build(force=a.force, verbose=True)
    if a.ggml_dir:
        build_ggml_backend(a.ggml_dir, verbose=True)
    sys.exit(0)
