"""Times one MLP training step as the reference runs it -- its generated C
for every scheduled kernel, through the restated lowering -- beside the
oracle port on one core (TEST INFRASTRUCTURE; a measurement, not a test).

    FG_LOWERING_CFLAGS="-O3 -march=native" python tests/lowering/time_step.py 784,128,10 256

argv: layer widths (comma-separated), batch.  Prints the best of three steps:
the wall time, the part spent in the kernels' C functions, and the oracle's
step time with one thread.
"""
import os
import sys
import time

import numpy as np

os.environ["FG_FRONT_EXACT"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(ROOT, "tests", "hostdev", "_build", "kcache"))
os.environ.setdefault("FG_LOWERING_CACHE", os.path.join(HERE, "_build", "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, os.path.join(ROOT, "tests", "hostdev", "_build"))
sys.path.insert(0, os.path.join(HERE, "_build"))
sys.path.insert(0, ROOT)
import _front as F  # noqa: E402
import _lowering as L  # noqa: E402

from ferrograd_b200 import data  # noqa: E402
from oracle import oracle  # noqa: E402


def main(dims_arg, batch_arg):
    dims = tuple(int(v) for v in dims_arg.split(","))
    batch = int(batch_arg)
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 13, 14)
    F.reset_init_seed(42)
    layers = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    params = [p for l in layers for p in l.parameters()]
    xt, tt = F.Tensor.new(x), F.Tensor.new(t)
    ws = [l.weight.numpy() for l in layers]
    bs = [l.bias.numpy() for l in layers]

    def step():  # examples/mnist.rs:90-97 with Sgd::step's graph (src/optim.rs:60-71)
        h = xt
        for i, l in enumerate(layers):
            h = l.forward(h)
            if i + 1 < len(layers):
                h = h.relu()
        loss = h.cross_entropy(tt)
        F.Sgd(params, 0.0).zero_grad()
        loss.backward()
        g = [p.grad() for p in params]
        for p, gp in zip(params, g):
            p.assign(p.detach().sub(gp.mul(F.Tensor.scalar(0.01))))
        L.realize(params)
        L.realize([loss])
        return loss.to_vec()[0]

    step()  # compiles every kernel
    runs = []
    for _ in range(3):
        L.kernel_seconds(True)
        t0 = time.perf_counter()
        step()
        runs.append((time.perf_counter() - t0, L.kernel_seconds(False)))
    wall, kern = min(runs)
    oracle.set_threads(1)
    orc = []
    for _ in range(3):
        t0 = time.perf_counter()
        oracle.mlp_step(ws, bs, x, t, 0.01)
        orc.append(time.perf_counter() - t0)
    print(f"reference step: {wall:.4f} s wall, {kern:.4f} s in its kernels; "
          f"oracle port, one thread: {min(orc):.4f} s")


if __name__ == "__main__":
    main(*sys.argv[1:3])
