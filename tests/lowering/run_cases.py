"""Runs the restated reference unit tests of the lowering passes and two
probes of the upcast path (TEST INFRASTRUCTURE; executed in a subprocess by
tests/test_lowering.py).  Prints one JSON object.

Probes (exact mode, every OPT pass on): a column sum of a [16, 8] integer matrix
(reduced axis 0 numbered before the upcast output axis 1) and a [16, 8] x
[8, 16]^T integer contraction stored as is (a reduction inside a nested output loop):
their C and their values from the reference's lowering as restated, and
with the repairs of kir.h.
"""
import json
import os
import sys

import numpy as np

os.environ["FG_FRONT_EXACT"] = "1"
os.environ.pop("OPT", None)
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(ROOT, "tests", "hostdev", "_build", "kcache"))
os.environ.setdefault("FG_LOWERING_CACHE", os.path.join(HERE, "_build", "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, os.path.join(ROOT, "tests", "hostdev", "_build"))
sys.path.insert(0, os.path.join(HERE, "_build"))
import _front as F  # noqa: E402
import _lowering as L  # noqa: E402


def probe(build, repair):
    L.set_repair(repair)
    t, expect = build()
    src = L.sources([t])
    L.realize([t])
    got = t.numpy()
    L.set_repair(False)
    return {"source": src[-1], "values": got.ravel().tolist(), "expect": expect.ravel().tolist()}


def column_sum():
    x = np.random.default_rng(4).integers(-5, 6, (16, 8)).astype(np.float32)
    return F.Tensor.new(x).sum([0]), x.astype(np.float64).sum(axis=0)


def nested_contraction():
    rng = np.random.default_rng(5)
    a = rng.integers(-3, 4, (16, 8)).astype(np.float32)
    b = rng.integers(-3, 4, (16, 8)).astype(np.float32)
    return F.Tensor.new(a).matmul(F.Tensor.new(b).permute([1, 0])), a.astype(np.float64) @ b.T


def main():
    out = {"cases": {}}
    for name in L.case_names():
        try:
            L.run_case(name)
            out["cases"][name] = "ok"
        except Exception as e:  # reported per case
            out["cases"][name] = str(e)
    for pname, build in (("column_sum", column_sum), ("nested_contraction", nested_contraction)):
        out[pname] = {"reference": probe(build, False), "repaired": probe(build, True)}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
