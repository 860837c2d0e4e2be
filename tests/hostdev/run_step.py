"""Runs training steps of the front end on the host test device (TEST
INFRASTRUCTURE; executed in a subprocess by tests/test_hostdev_front.py so
that this _front module never shares a process with the GPU build's).

argv: input .npz (x, t, dims, lr, steps), output .npz.  Exact mode unless
the caller's environment sets FG_FRONT_EXACT=0 (the routed default mode).
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
    lr = float(d["lr"])
    # Initial values from a twin built from the same seed, so the trained
    # model's parameters are not read (and so not allocated) before the first
    # step: their first write is the in-place SGD store.
    F.reset_init_seed(42)
    twin = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    ws = [l.weight.numpy() for l in twin]
    bs = [l.bias.numpy() for l in twin]
    F.reset_init_seed(42)
    layers = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    params = [p for l in layers for p in l.parameters()]
    opt = F.Sgd(params, lr)
    x, t = F.Tensor.new(d["x"]), F.Tensor.new(d["t"])
    losses, grads, acts = [], None, None
    for step in range(int(d["steps"])):
        h, hs = x, []
        for i, l in enumerate(layers):
            h = l.forward(h)
            if i + 1 < len(layers):
                h = h.relu()
                hs.append(h)
        loss = h.cross_entropy(t)
        opt.zero_grad()
        loss.backward()
        g = [l.weight.grad() for l in layers] + [l.bias.grad() for l in layers]
        opt.step()
        losses.append(loss.to_vec()[0])
        grads = [gg.numpy() for gg in g]
        if step == 0:
            acts = [a.numpy() for a in hs]
    out = {"loss": np.array(losses, np.float32)}
    for i, l in enumerate(layers):
        out[f"w0_{i}"], out[f"b0_{i}"] = ws[i], bs[i]
        out[f"w_{i}"], out[f"b_{i}"] = l.weight.numpy(), l.bias.numpy()
        out[f"dw_{i}"], out[f"db_{i}"] = grads[i], grads[len(layers) + i].ravel()
    for i, a in enumerate(acts):
        out[f"act_{i}"] = a
    st = F.stats()
    out["compiled"] = np.array(st["compiled"])
    out["gemm"] = np.array(st["gemm"])
    out["hand_reduce"] = np.array(st["hand_reduce"])
    out["schedule_hits"] = np.array(st["schedule_hits"])
    for k in ("xent", "xent_reused", "sgd", "gemm_bias", "gemm_mask"):
        out[k] = np.array(st[k])
    np.savez(dst, **out)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
