"""Regenerate tests/golden/c1_step_reference_c.txt, a regression pin of the
restated reference lowering (tests/lowering/): the C the reference's passes,
as written and with every OPT pass on, emit for the kernels of Sgd::step's
realize in a config-1 step (784-128-10, batch 256).  Run from the repo root:
python tests/golden/make_lowering_golden.py
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from ferrograd_b200 import data  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "c1_step_reference_c.txt")


def emit() -> str:
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "lowering_build", os.path.join(ROOT, "tests", "lowering", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    dims, batch = (784, 128, 10), 256
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 13, 14)
    with tempfile.TemporaryDirectory() as d:
        src, dst, c = (os.path.join(d, n) for n in ("in.npz", "out.npz", "kernels.c"))
        np.savez(src, x=x, t=t, dims=np.array(dims), lr=np.array(0.01), steps=np.array(1))
        env = dict(os.environ)
        env.pop("OPT", None)
        env["FG_LOWERING_REPAIR"] = "0"
        subprocess.run([sys.executable, os.path.join(ROOT, "tests", "lowering", "run_step.py"),
                        src, dst, c], check=True, timeout=900, env=env)
        return open(c).read()


if __name__ == "__main__":
    text = emit()
    with open(OUT, "w") as f:
        f.write(text)
    print("wrote", OUT, len(text), "bytes")
