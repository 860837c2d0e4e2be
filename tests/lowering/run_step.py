"""Training steps of the front end with every kernel lowered by the restated
reference pipeline and run as the reference's C (TEST INFRASTRUCTURE;
executed in a subprocess by tests/test_lowering.py).

The step is the reference's (examples/mnist.rs:90-97): forward, cross_entropy,
zero_grad, backward, Sgd::step's assignments (src/optim.rs:60-71, p -= lr * g
for every parameter, then one realize of all of them), and the loss read.  The
graph is built by the front end (exact mode, so its kernel boundaries are the
reference's); each realize goes through _lowering.realize.

argv: input .npz (x, t, dims, lr, steps), output .npz; optional third
argument: a file to write the C sources of the first step's kernels to.
"""
import os
import sys

import numpy as np

os.environ["FG_FRONT_EXACT"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(ROOT, "tests", "hostdev", "_build", "kcache"))
os.environ.setdefault("FG_LOWERING_CACHE", os.path.join(HERE, "_build", "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, os.path.join(ROOT, "tests", "hostdev", "_build"))
sys.path.insert(0, os.path.join(HERE, "_build"))
import _front as F  # noqa: E402
import _lowering as L  # noqa: E402


def main(src, dst, source_file=None):
    L.set_repair(os.environ.get("FG_LOWERING_REPAIR") == "1")
    d = np.load(src)
    dims = [int(v) for v in d["dims"]]
    lr = float(d["lr"])
    F.reset_init_seed(42)
    twin = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    ws = [l.weight.numpy() for l in twin]
    bs = [l.bias.numpy() for l in twin]
    F.reset_init_seed(42)
    layers = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    params = [p for l in layers for p in l.parameters()]
    x, t = F.Tensor.new(d["x"]), F.Tensor.new(d["t"])
    losses, grads = [], None
    for step in range(int(d["steps"])):
        h = x
        for i, l in enumerate(layers):
            h = l.forward(h)
            if i + 1 < len(layers):
                h = h.relu()
        loss = h.cross_entropy(t)
        opt_zero(params)
        loss.backward()
        g = [p.grad() for p in params]
        for p, gp in zip(params, g):  # Sgd::step's graph, as the front end builds it
            p.assign(p.detach().sub(gp.mul(F.Tensor.scalar(lr))))
        if step == 0 and source_file:
            with open(source_file, "w") as f:
                f.write("\n".join(L.sources(params)))
        L.realize(params)
        L.realize([loss])
        losses.append(loss.to_vec()[0])
        L.realize(g)
        grads = [gg.numpy() for gg in g]
    out = {"loss": np.array(losses, np.float32)}
    nl = len(layers)
    for i, l in enumerate(layers):
        out[f"w0_{i}"], out[f"b0_{i}"] = ws[i], bs[i]
        out[f"w_{i}"], out[f"b_{i}"] = l.weight.numpy(), l.bias.numpy()
        out[f"dw_{i}"], out[f"db_{i}"] = grads[2 * i], grads[2 * i + 1].ravel()
    st = L.stats()
    out["launches"] = np.array(st["launches"])
    out["front_kernels"] = np.array(F.stats()["kernels"])
    np.savez(dst, **out)


def opt_zero(params):
    """Sgd::zero_grad (src/optim.rs:50-58): drop every parameter's gradient."""
    F.Sgd(params, 0.0).zero_grad()


if __name__ == "__main__":
    main(*sys.argv[1:])
