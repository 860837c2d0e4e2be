"""The examples/mnist.rs loop over narrow() batches of a resident dataset on
the host test device (TEST INFRASTRUCTURE; run in a subprocess by
tests/test_hostdev_front.py): each batch is a Shrink view whose start is a
kernel argument, in exact mode (FG_FRONT_EXACT=1, the default here) or the
routed mode (FG_FRONT_EXACT=0, where the narrowed input reaches the GEMM
contract as a strided view).

argv: input .npz (x, t, dims, lr, batch), output .npz.
"""
import os
import sys

import numpy as np

os.environ.setdefault("FG_FRONT_EXACT", "1")
_BUILD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(_BUILD, "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, _BUILD)
import _front as F  # noqa: E402


def main(src, dst):
    d = np.load(src)
    dims = [int(v) for v in d["dims"]]
    lr, batch = float(d["lr"]), int(d["batch"])
    F.reset_init_seed(42)
    twin = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    out = {}
    for i, l in enumerate(twin):
        out[f"w0_{i}"], out[f"b0_{i}"] = l.weight.numpy(), l.bias.numpy()
    F.reset_init_seed(42)
    layers = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    opt = F.Sgd([p for l in layers for p in l.parameters()], lr)
    images, targets = F.Tensor.new(d["x"]), F.Tensor.new(d["t"])
    losses, compiled = [], []
    for b in range(d["x"].shape[0] // batch):
        h = images.narrow(0, b * batch, batch)
        tb = targets.narrow(0, b * batch, batch)
        for i, l in enumerate(layers):
            h = l.forward(h)
            if i + 1 < len(layers):
                h = h.relu()
        loss = h.cross_entropy(tb)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(loss.to_vec()[0])
        compiled.append(F.stats()["compiled"])
    for i, l in enumerate(layers):
        out[f"w_{i}"], out[f"b_{i}"] = l.weight.numpy(), l.bias.numpy()
    st = F.stats()
    np.savez(dst, loss=np.array(losses, np.float32), compiled=np.array(compiled),
             gemm=np.array(st["gemm"]), **out)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
