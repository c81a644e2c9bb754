"""Build libxq_b200.so (the C-ABI CUDA library) in-tree for sm_100a.

    python xllama-qwen35-xbox_b200/build.py [--force] [-j N]

Each csrc/*.cu compiles to an object with nvcc -gencode
arch=compute_100a,code=sm_100a, then one shared library is linked at
xllama-qwen35-xbox_b200/lib/libxq_b200.so.  The library depends only on the
CUDA runtime (no torch).  Objects are rebuilt when a source or header changed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib", "libxq_b200.so")
GGML_LIB = os.path.join(PKG, "lib", "libxq_ggml_b200.so")
RKVA_SERVER = os.path.join(PKG, "bin", "xq_rkva_server")
RKVA_SRC = os.path.join(PKG, "rkva", "rkva_server.cpp")
GGML_SRC = os.path.join(PKG, "ggml", "ggml_xq_backend.cpp")
INCLUDE = os.path.join(REPO, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force, verbose_ptxas):
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    if not force and not _stale(obj, [src] + _headers()):
        return obj, None
    cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + \
        ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), srcs))
    objs = [o for o, _ in results]
    if verbose_ptxas:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if force or _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    build_ggml_backend(force)
    build_rkva_server(force)
    return LIB


def build_ggml_backend(force: bool = False) -> str:
    """libxq_ggml_b200.so: the ggml backend over libxq_b200.so.  ggml's own
    symbols stay undefined here; the host process (llama.cpp's libggml-base,
    or the test harness) provides them at load time."""
    hdr = os.path.join(PKG, "ggml", "ggml_abi_mirror.h")
    if not force and not _stale(GGML_LIB, [GGML_SRC, hdr, LIB] + _headers()):
        return GGML_LIB
    cuda = os.path.dirname(os.path.dirname(NVCC))
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-I" + INCLUDE,
           "-I" + os.path.join(PKG, "ggml"), "-I" + os.path.join(cuda, "include"), GGML_SRC,
           "-o", GGML_LIB, "-L" + os.path.dirname(LIB), "-lxq_b200",
           "-L" + os.path.join(cuda, "lib64"), "-lcudart", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ggml backend build failed:\n{r.stderr}")
    return GGML_LIB


def build_rkva_server(force: bool = False) -> str:
    """bin/xq_rkva_server: the RKVA range server over libxq_b200.so."""
    hdr = os.path.join(PKG, "rkva", "rkva_wire.h")
    if not force and not _stale(RKVA_SERVER, [RKVA_SRC, hdr, LIB] + _headers()):
        return RKVA_SERVER
    os.makedirs(os.path.dirname(RKVA_SERVER), exist_ok=True)
    cuda = os.path.dirname(os.path.dirname(NVCC))
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-I" + INCLUDE, "-I" + os.path.join(PKG, "rkva"),
           "-I" + os.path.join(cuda, "include"), RKVA_SRC, "-o", RKVA_SERVER,
           "-L" + os.path.dirname(LIB), "-lxq_b200", "-L" + os.path.join(cuda, "lib64"),
           "-lcudart", "-Wl,-rpath,$ORIGIN/../lib"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"RKVA server build failed:\n{r.stderr}")
    return RKVA_SERVER


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas))
