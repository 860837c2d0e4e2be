"""Builds the restated reference lowering (TEST INFRASTRUCTURE).

Produces tests/lowering/_build/_lowering.<ext>: the kernel IR and passes
(kir.cpp, passes.cpp), the reference's own unit tests of them (cases.cpp),
gcc-compiled execution of the emitted C (runc.cpp) and the bridge from the
front end's scheduled items (bridge.cpp), linked against the front end of the
host test device (tests/hostdev/build.py), so it shares that process's graph
and buffers.  The product build is not involved.
"""
import importlib.util
import os
import subprocess
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "_build")
SRC = ["kir.cpp", "passes.cpp", "cases.cpp", "runc.cpp", "bridge.cpp"]


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def build() -> str:
    import pybind11
    hd = _load("hostdev_build", os.path.join(ROOT, "tests", "hostdev", "build.py")).build()
    os.makedirs(OUT, exist_ok=True)
    mod = os.path.join(OUT, "_lowering" + sysconfig.get_config_var("EXT_SUFFIX"))
    srcs = [os.path.join(HERE, f) for f in SRC]
    deps = srcs + [os.path.join(HERE, f) for f in ("kir.h", "lowering.h")]
    deps += [os.path.join(hd, "libferro_front.so")]
    front = os.path.join(ROOT, "ferrograd_b200", "csrc", "front")
    deps += [os.path.join(front, f) for f in os.listdir(front) if f.endswith(".h")]
    if not os.path.exists(mod) or any(os.path.getmtime(d) > os.path.getmtime(mod) for d in deps):
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall",
                        f"-I{os.path.join(ROOT, 'include')}", f"-I{pybind11.get_include()}",
                        f"-I{sysconfig.get_paths()['include']}", *srcs, "-L" + hd,
                        "-lferro_front", "-lferro_cuda", f"-Wl,-rpath,{hd}", "-ldl", "-o", mod],
                       check=True)
    return OUT


if __name__ == "__main__":
    print(build())
