"""Build ``ferrograd_b200/libferro_cuda.so`` with nvcc for sm_100a.

The library is built in-tree so it travels with the repository snapshot.
Run ``python -m ferrograd_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libferro_cuda.so")
OBJDIR = os.path.join(HERE, "_build")

SOURCES = ["fg_runtime.cu", "fg_kernels.cu", "fg_gemm.cu", "fg_mlp.cu", "fg_comm.cu", "fg_peer.cu",
           "fg_init.cpp"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "-ccbin", "g++", f"-I{os.path.join(ROOT, 'include')}"]
LIBS = ["-L/usr/local/cuda/lib64", "-lcudart", "-lnvrtc", "-ldl"]


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False) -> str:
    """Build the CUDA library, then the front end on top of it."""
    lib = build_cuda(verbose)
    build_front(verbose)
    return lib


def build_cuda(verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "ferro_cuda.h"))
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".o")
        objs.append(o)
        if _stale(o, [s] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, *LIBS]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


FRONT = os.path.join(CSRC, "front")
FRONT_SOURCES = ["graph.cpp", "render.cpp", "exec.cpp", "tensor.cpp"]
FRONT_LIB = os.path.join(HERE, "libferro_front.so")
CXX = os.environ.get("CXX_FRONT", "g++")
CXXFLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter",
            f"-I{os.path.join(ROOT, 'include')}"]


def _front_module_path() -> str:
    return os.path.join(HERE, "_front" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_front(verbose: bool = False) -> str:
    """Build ``libferro_front.so`` (the C++ lazy-graph front end, linked to
    ``libferro_cuda.so``) and its Python module ``_front`` with g++."""
    import pybind11

    os.makedirs(OBJDIR, exist_ok=True)
    headers = [os.path.join(FRONT, f) for f in os.listdir(FRONT) if f.endswith(".h")]
    headers.append(os.path.join(ROOT, "include", "ferro_cuda.h"))
    objs = []
    for src in FRONT_SOURCES:
        s = os.path.join(FRONT, src)
        o = os.path.join(OBJDIR, "front_" + src.replace(".cpp", ".o"))
        objs.append(o)
        if _stale(o, [s] + headers):
            cmd = [CXX, *CXXFLAGS, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    link = ["-L" + HERE, "-lferro_cuda", "-Wl,-rpath,$ORIGIN"]
    if _stale(FRONT_LIB, objs + [LIB]):
        cmd = [CXX, "-shared", "-o", FRONT_LIB, *objs, *link]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    mod = _front_module_path()
    py_src = os.path.join(FRONT, "front_py.cpp")
    if _stale(mod, [py_src, FRONT_LIB] + headers):
        cmd = [CXX, *CXXFLAGS, "-shared", f"-I{pybind11.get_include()}",
               f"-I{sysconfig.get_paths()['include']}", py_src, "-o", mod,
               "-L" + HERE, "-lferro_front", "-lferro_cuda", "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return mod


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
