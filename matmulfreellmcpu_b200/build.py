"""Build libmmfree_cuda.so (sm_100a) in-tree: ``python -m matmulfreellmcpu_b200.build``.

Every CUDA source is compiled by nvcc for ``-gencode arch=compute_100a,code=sm_100a`` with
``-lineinfo``; objects go to ``_build/`` and the shared library to ``_lib/``. A source is
recompiled when it or any header of ``csrc/`` is newer than its object.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libmmfree_cuda.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills", "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def host_compiler() -> list[str]:
    # /usr/bin/g++ is the system compiler of the image; nvcc picks whatever g++ is first on
    # PATH otherwise.
    return ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max(os.path.getmtime(src), _headers_mtime())
    if force or not os.path.exists(obj) or os.path.getmtime(obj) < newest:
        cmd = [nvcc(), *host_compiler(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile every source and link the library; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(map(os.path.getmtime, objs)):
        cmd = [nvcc(), *host_compiler(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static",
               "-lrt", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_cli(force)
    return LIB


CLI = os.path.join(LIBDIR, "mmfree-cli")
CLI_SRC = os.path.join(PKG, "cli", "mmfree_cli.cpp")


def build_cli(force: bool = False) -> str:
    """The CUDA-backed mmfree-cli (host C++ over the C ABI, rpath to the library)."""
    srcs = [CLI_SRC, os.path.join(PKG, "cli", "tokenizer.cpp")]
    deps = srcs + [LIB, os.path.join(PKG, "cli", "tokenizer.hpp"), os.path.join(INCLUDE, "mmfree_cuda.h"),
                   os.path.join(INCLUDE, "mmfree_cuda.hpp")]
    if force or not os.path.exists(CLI) or os.path.getmtime(CLI) < max(map(os.path.getmtime, deps)):
        cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
        cmd = [cxx, "-O2", "-std=c++17", "-I" + INCLUDE, *srcs, "-L" + LIBDIR, "-lmmfree_cuda",
               "-Wl,-rpath,$ORIGIN", "-o", CLI]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"cli build failed:\n{r.stdout}\n{r.stderr}")
    return CLI


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
