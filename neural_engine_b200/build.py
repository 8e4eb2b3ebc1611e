"""Build libne.so in-tree for sm_100a with nvcc.

    python neural_engine_b200/build.py   (or __graft_entry__.build(); the package
    itself cannot be imported before the library exists)

Every .cu under csrc/ is compiled for ``-gencode arch=compute_100a,code=sm_100a``
with ``-lineinfo`` into _build/, then linked (static cudart) into
neural_engine_b200/libne.so.  Objects are rebuilt when their source or any
header under csrc/ or include/ is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libne.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler",
         "-fvisibility=hidden", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
         "--expt-relaxed-constexpr"]


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _newest_header()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = True, extra: list[str] | None = None) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = list(extra or [])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        build_host(verbose)
        return LIB
    cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {LIB}")
    build_host(verbose)
    return LIB


HOST_SRC = os.path.join(PKG, "host", "ne_train.cpp")
HOST_BIN = os.path.join(PKG, "ne_train")
CONV_SRC = os.path.join(PKG, "host", "ne_convert.cpp")
CONV_BIN = os.path.join(PKG, "ne_convert")


def build_convert(verbose: bool = True) -> str:
    """ne_convert: HF safetensors <-> v4 checkpoint (plain C++, no CUDA)."""
    if os.path.exists(CONV_BIN) and os.path.getmtime(CONV_BIN) >= os.path.getmtime(CONV_SRC):
        return CONV_BIN
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-Wall", CONV_SRC, "-o", CONV_BIN]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ne_convert build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {CONV_BIN}")
    return CONV_BIN


def build_host(verbose: bool = True) -> str:
    """The ne_train command-line driver (plain C++ over the C ABI of libne.so)."""
    build_convert(verbose)
    if os.path.exists(HOST_BIN) and os.path.getmtime(HOST_BIN) >= max(
            os.path.getmtime(HOST_SRC), os.path.getmtime(LIB),
            os.path.getmtime(os.path.join(ROOT, "include", "ne.h"))):
        return HOST_BIN
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-Wall", "-I",
           os.path.join(ROOT, "include"), HOST_SRC, "-o", HOST_BIN, "-L", PKG, "-lne",
           "-Wl,-rpath,$ORIGIN", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ne_train build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {HOST_BIN}")
    return HOST_BIN


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
