"""The front end's routed (default-mode) paths checked against the reference's
C on graphs other than the MLP step (TEST INFRASTRUCTURE; run in a
subprocess by tests/test_lowering.py).

Each graph is built and realized twice in one process: once in the default
mode (FG_FRONT_EXACT=0: contractions on the 3xTF32 GEMM contract, large
reductions on the HBM reduction contracts, the fused cross-entropy and SGD
routes -- their host restatements on the host test device), once in exact
mode with every kernel lowered as the reference lowers it (repaired, so the
reference's C computes what its passes intend).  Prints one JSON object:
graph -> {"max_rel", "routes"}; the routes are the front end's counters for
the default-mode realize.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(ROOT, "tests", "hostdev", "_build", "kcache"))
os.environ.setdefault("FG_LOWERING_CACHE", os.path.join(HERE, "_build", "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, os.path.join(ROOT, "tests", "hostdev", "_build"))
sys.path.insert(0, os.path.join(HERE, "_build"))
import _front as F  # noqa: E402
import _lowering as L  # noqa: E402

RNG = np.random.default_rng(21)
A = RNG.standard_normal((256, 192), dtype=np.float32)
W = RNG.standard_normal((160, 192), dtype=np.float32) * 0.1
BIAS = RNG.standard_normal((160,), dtype=np.float32)
X = RNG.standard_normal((1024, 1536), dtype=np.float32)
LOGITS = RNG.standard_normal((512, 10), dtype=np.float32) * 3
TGT = np.zeros((512, 10), np.float32)
TGT[np.arange(512), RNG.integers(0, 10, 512)] = 1
P0 = RNG.standard_normal((96, 64), dtype=np.float32)
G0 = RNG.standard_normal((96, 64), dtype=np.float32)
M = RNG.standard_normal((512, 192), dtype=np.float32)
N = RNG.standard_normal((192, 128), dtype=np.float32) * 0.1


def graphs():
    t = F.Tensor.new
    lin = lambda: t(A).matmul(t(W).permute([1, 0])) + t(BIAS).reshape([1, 160]).expand([256, 160])  # noqa: E731
    g = {
        "matmul": lambda: t(A).matmul(t(W).permute([1, 0])),
        "linear_bias": lin,
        "linear_bias_relu": lambda: lin().relu(),
        "row_sum": lambda: t(X).sum([1]),
        "col_sum": lambda: t(X).sum([0]),
        "row_max": lambda: t(X).max([1]),
        "cross_entropy": lambda: t(LOGITS).cross_entropy(t(TGT)),
    }

    def grad(build, wrt, i=0):
        def f():
            leaves = [t(x).with_requires_grad(True) for x in wrt]
            return build(*leaves).gradient(leaves)[i]
        return f
    g["grad_cross_entropy"] = grad(lambda z: z.cross_entropy(t(TGT)), [LOGITS])
    # dX of a ReLU layer: the masked backward contraction
    g["grad_relu_layer_dx"] = grad(
        lambda a, w: (a.matmul(w.permute([1, 0])).relu() * t(np.ones((256, 160), np.float32))).sum([0, 1]),
        [A, W], 0)
    g["grad_relu_layer_dw"] = grad(
        lambda a, w: (a.matmul(w.permute([1, 0])).relu()).sum([0, 1]), [A, W], 1)
    g["matmul_chain"] = lambda: t(M).matmul(t(N)).relu().matmul(t(N).permute([1, 0]))

    def sgd():
        p = t(P0)
        p.realize()
        p.assign(p.detach().sub(t(G0).mul(F.Tensor.scalar(0.01))))
        return p
    g["sgd_update"] = sgd
    return g


def realize(build, exact):
    os.environ["FG_FRONT_EXACT"] = "1" if exact else "0"
    x = build()
    if exact:
        L.realize([x])
    else:
        F.reset_stats()
        x.realize()
    out = x.numpy().astype(np.float64)
    return out, (None if exact else F.stats())


def main():
    L.set_repair(True)
    res = {}
    for name, build in graphs().items():
        routed, st = realize(build, False)
        ref, _ = realize(build, True)
        scale = max(1.0, float(np.max(np.abs(ref))))
        res[name] = {"max_rel": float(np.max(np.abs(routed - ref)) / scale),
                     "routes": {k: st[k] for k in ("gemm", "hand_reduce", "xent", "sgd",
                                                   "gemm_bias", "gemm_mask")}}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
