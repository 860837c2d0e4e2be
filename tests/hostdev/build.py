"""Builds the front end against the host test device (TEST INFRASTRUCTURE).

Produces, under tests/hostdev/_build/: libferro_cuda.so (hostdev.cpp + the
shared host-side init, implementing the device part of include/ferro_cuda.h
on the CPU), libferro_front.so (the unchanged front-end sources linked
against it) and the _front Python module.  The product build
(ferrograd_b200/build.py) is not involved.
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "_build")
FRONT = os.path.join(ROOT, "ferrograd_b200", "csrc", "front")
FLAGS = ["-O2", "-std=c++17", "-fPIC", "-w", f"-I{os.path.join(ROOT, 'include')}"]


def _stale(target, deps):
    return not os.path.exists(target) or any(os.path.getmtime(d) > os.path.getmtime(target)
                                             for d in deps)


def build(noexec: bool = False) -> str:
    """noexec: a variant under _build_noexec whose compute entry points
    return without computing (FG_HOSTDEV_NOEXEC), for timing host work."""
    import pybind11
    out = OUT + "_noexec" if noexec else OUT
    os.makedirs(out, exist_ok=True)
    dev = os.path.join(out, "libferro_cuda.so")
    dev_src = [os.path.join(HERE, "hostdev.cpp"),
               os.path.join(ROOT, "ferrograd_b200", "csrc", "fg_init.cpp")]
    defs = ["-DFG_HOSTDEV_NOEXEC"] if noexec else []
    if _stale(dev, dev_src + [os.path.join(ROOT, "include", "ferro_cuda.h")]):
        subprocess.run(["g++", *FLAGS, *defs, "-shared", *dev_src, "-ldl", "-o", dev], check=True)
    front_src = [os.path.join(FRONT, f) for f in ("graph.cpp", "render.cpp", "exec.cpp", "tensor.cpp")]
    headers = [os.path.join(FRONT, f) for f in os.listdir(FRONT) if f.endswith(".h")]
    lib = os.path.join(out, "libferro_front.so")
    if _stale(lib, front_src + headers + [dev]):
        subprocess.run(["g++", *FLAGS, "-shared", *front_src, "-L" + out, "-lferro_cuda",
                        "-Wl,-rpath,$ORIGIN", "-o", lib], check=True)
    mod = os.path.join(out, "_front" + sysconfig.get_config_var("EXT_SUFFIX"))
    py_src = os.path.join(FRONT, "front_py.cpp")
    if _stale(mod, [py_src, lib] + headers):
        subprocess.run(["g++", *FLAGS, "-shared", f"-I{pybind11.get_include()}",
                        f"-I{sysconfig.get_paths()['include']}", py_src, "-L" + out,
                        "-lferro_front", "-lferro_cuda", "-Wl,-rpath,$ORIGIN", "-o", mod],
                       check=True)
    return out


if __name__ == "__main__":
    print(build())
