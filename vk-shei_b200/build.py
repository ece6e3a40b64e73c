"""Build recipe of the sm_100a CUDA library (in-tree, so the built files
travel with the source tree to the GPU host).

Produces, next to the Python binding:
  mslim_b200/libmslim_cuda.so   shared library loaded by the Python binding
  mslim_b200/libmslim_cuda.a    static archive for a Rust build.rs link
Each .cu is compiled once for sm_100a (`-gencode arch=compute_100a,code=sm_100a`)
with -lineinfo; translation units are rebuilt only when they or a header
changed.  Usage: python vk-shei_b200/build.py [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "mslim_b200")
OBJ_DIR = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
SOURCES = ["capi.cu", "decode.cu", "prologue.cu", "prefill.cu", "layer_ops.cu", "tp_allreduce.cu", "gemv.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
HOST_CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ccbin", HOST_CXX,
         "-I", INCLUDE, "-I", CSRC]
SO = os.path.join(OUT_DIR, "libmslim_cuda.so")
AR = os.path.join(OUT_DIR, "libmslim_cuda.a")


def digest_files() -> list[str]:
    """The files whose bytes define the library: the CUDA sources in build
    order, the device headers (sorted), the C ABI header and this recipe."""
    heads = sorted(f for f in os.listdir(CSRC) if f.endswith((".cuh", ".h")))
    return ([os.path.join(CSRC, f) for f in SOURCES] + [os.path.join(CSRC, f) for f in heads] +
            [os.path.join(INCLUDE, "mslim_cuda.h"), os.path.abspath(__file__)])


def source_digest() -> str:
    """SHA-256 over every digest file as (length u64 LE, bytes), then the
    target architecture flags -- the library's counterpart of the reference's
    implementation_digest (src/calibration_profile.rs:90-125), which hashes
    its kernel and runtime sources the same way."""
    import hashlib
    import struct
    h = hashlib.sha256()
    for f in digest_files():
        data = open(f, "rb").read()
        h.update(struct.pack("<Q", len(data)))
        h.update(data)
    h.update(" ".join(ARCH).encode())
    return h.hexdigest()


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    extra, deps = [], [path] + _headers()
    if src == "capi.cu":
        # the C ABI carries the digest of every source, so it follows all of them
        extra = [f"-DMSLIM_SOURCE_DIGEST=\"{source_digest()}\""]
        deps = digest_files()
    if force or _stale(obj, deps):
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", path, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or _stale(SO, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", SO, *objs, "-ccbin", HOST_CXX]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if force or _stale(AR, objs):
        cmd = [NVCC, *ARCH, "-lib", "-o", AR, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"archive failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {SO}")
    return SO


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
