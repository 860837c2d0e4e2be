"""A zoo of Tensor-API graphs realized twice in one process: through the
front end's own exact-mode executor (its rendered kernels on the host test
device) and through the restated reference lowering (the reference's C), the
two results compared bit for bit (TEST INFRASTRUCTURE; run in a subprocess
by tests/test_lowering.py with the OPT / FG_LOWERING_REPAIR setting under
test).  Prints one JSON object: graph name -> {"equal", "max_abs", "kernels"}.
"""
import json
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

RNG = np.random.default_rng(11)
A = RNG.standard_normal((12, 20), dtype=np.float32)
B = RNG.standard_normal((12, 20), dtype=np.float32)
C = RNG.standard_normal((20, 9), dtype=np.float32)
V = RNG.standard_normal((20,), dtype=np.float32)
P = np.abs(RNG.standard_normal((12, 20), dtype=np.float32)) + 0.1
I = RNG.integers(-50, 50, (24, 16)).astype(np.int32)
T = np.zeros((12, 20), np.float32)
T[np.arange(12), RNG.integers(0, 20, 12)] = 1
Q = RNG.standard_normal((3, 8, 16), dtype=np.float32)
TIE = np.array([[1, 3, 3, 2], [5, 5, 5, 1], [0, -1, 0, -1]], np.float32)


def graphs():
    t = F.Tensor.new
    g = {}
    g["broadcast_chain"] = lambda: (t(A) * t(B) + t(V).reshape([1, 20]).expand([12, 20])).relu()
    g["unary_math"] = lambda: (t(P).log2() + t(A).exp2() * t(P).sqrt()).reciprocal()
    g["exp_log"] = lambda: t(P).log() - t(A).exp()
    g["where_cmplt"] = lambda: t(A).max([1]).expand([12, 20]) - t(A)
    g["row_sum"] = lambda: t(A).sum([1])
    g["col_sum"] = lambda: t(A).sum([0])
    g["all_sum"] = lambda: t(A).sum([0, 1])
    g["row_max"] = lambda: t(A).max([1])
    g["col_max"] = lambda: t(A).max([0])
    g["sum_3d_middle"] = lambda: t(Q).sum([1])
    g["sum_3d_outer_inner"] = lambda: t(Q).sum([0, 2])
    g["permute_contiguous"] = lambda: t(Q).permute([2, 0, 1]).contiguous() * t(Q).permute([2, 0, 1])
    g["narrow_rows"] = lambda: t(A).narrow(0, 3, 5).exp2()
    g["narrow_cols_sum"] = lambda: t(A).narrow(1, 4, 12).sum([1])
    g["matmul"] = lambda: t(A).matmul(t(C))
    g["matmul_bias_relu"] = lambda: (t(A).matmul(t(C)) + t(C).sum([0]).reshape([1, 9]).expand([12, 9])).relu()
    g["i32_sum"] = lambda: t(I).sum([1])
    g["i32_col_sum"] = lambda: t(I).sum([0])
    g["log_softmax"] = lambda: t(A).log_softmax(1)
    g["cross_entropy"] = lambda: t(A).cross_entropy(t(T))
    g["reshape_chain"] = lambda: t(Q).reshape([24, 16]).sum([0]).reshape([4, 4]).permute([1, 0]).contiguous()

    def grad_of(build, wrt):
        def f():
            leaves = [t(x).with_requires_grad(True) for x in wrt]
            loss = build(*leaves)
            return loss.gradient(leaves)[0]
        return f
    g["grad_max_ties"] = grad_of(lambda x: x.max([1]).sum([0, 1]), [TIE])
    g["grad_matmul"] = grad_of(lambda a, c: (a.matmul(c)).relu().sum([0, 1]), [A, C])
    g["grad_cross_entropy"] = grad_of(lambda a: a.cross_entropy(t(T)), [A])
    g["grad_log_softmax"] = grad_of(lambda a: a.log_softmax(1).sum([0, 1]), [A])
    return g


def main():
    L.set_repair(os.environ.get("FG_LOWERING_REPAIR") == "1")
    out = {}
    for name, build in graphs().items():
        front = build().numpy()
        before = L.stats()["launches"]
        x = build()
        try:
            L.realize([x])
        except RuntimeError as e:  # a lowering the reference's passes reject too
            out[name] = {"error": str(e)}
            continue
        ours = x.numpy()
        ka = front.astype(np.float64).ravel()
        kb = ours.astype(np.float64).ravel()
        out[name] = {"equal": bool(np.array_equal(front, ours) and front.dtype == ours.dtype),
                     "max_abs": float(np.max(np.abs(ka - kb))) if ka.size else 0.0,
                     "kernels": int(L.stats()["launches"] - before)}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
