"""The reference's own end-to-end unit tests (tests/golden/known_answers.json,
each naming its file:line) realized as the reference's C through the
restated lowering (TEST INFRASTRUCTURE; run in a subprocess by
tests/test_lowering.py with the OPT setting under test).  Prints one JSON
object: case -> {"got", "expected", "tol"}.
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


def value(t):
    L.realize([t])
    return t.numpy().astype(np.float64).ravel().tolist()


def main():
    kat = json.load(open(os.path.join(ROOT, "tests", "golden", "known_answers.json")))
    T = lambda x: F.Tensor.new(np.array(x, np.float32))  # noqa: E731
    out = {}
    k = kat["log_softmax"]
    out["log_softmax"] = (value(T(k["input"]).log_softmax(1)), k["expected"], k["tol"])
    k = kat["cross_entropy"]
    out["cross_entropy"] = (value(T(k["logits"]).cross_entropy(T(k["targets"]))), [k["expected"]],
                            k["tol"])
    k = kat["sum_axis0"]
    out["sum_axis0"] = (value(T(k["input"]).sum([0])), k["expected"], 0.0)
    k = kat["relu"]
    out["relu"] = (value(T(k["input"]).relu()), k["expected"], 0.0)
    k = kat["max_reduce"]
    out["max_reduce"] = (value(T(k["input"]).max([1])), k["expected"], 0.0)
    k = kat["narrow_matmul_grad"]
    x = T(k["x"]).narrow(0, 1, 1)
    w = T(k["w"]).with_requires_grad(True)
    out["narrow_matmul_grad"] = (value(x.matmul(w).sum([0, 1]).gradient([w])[0]), k["expected"],
                                 0.0)
    k = kat["mul_backward"]
    xs = T([k["x"]]).with_requires_grad(True)
    ys = T([k["y"]]).with_requires_grad(True)
    gx, gy = xs.mul(ys).sum([0]).gradient([xs, ys])
    out["mul_backward"] = (value(gx) + value(gy), [k["dx"], k["dy"]], 0.0)
    k = kat["sgd"]  # src/optim.rs:80-94: one step moves the parameter toward the target
    p = T([k["param"]]).with_requires_grad(True)
    d = p.sub(T([k["target"]]))
    loss = d.mul(d).sum([0])
    F.Sgd([p], 0.0).zero_grad()
    loss.backward()
    g = p.grad()
    p.assign(p.detach().sub(g.mul(F.Tensor.scalar(k["lr"]))))
    L.realize([p])
    step = k["param"] - k["lr"] * 2.0 * (k["param"] - k["target"])
    out["sgd"] = (p.numpy().astype(np.float64).ravel().tolist(), [step], 1e-6)
    k = kat["assign_in_place"]
    a = T(k["initial"])
    a.realize()
    a.assign(T(k["assigned"]))
    L.realize([a])
    out["assign_in_place"] = (a.numpy().astype(np.float64).ravel().tolist(), k["assigned"], 0.0)
    print(json.dumps({n: {"got": g_, "expected": e, "tol": tol} for n, (g_, e, tol) in out.items()}))


if __name__ == "__main__":
    main()
