"""Random Tensor-API graphs (the generator of tests/hostdev/run_fuzz.py)
realized twice in one process: by the front end's exact mode on the host
test device and as the reference's C through the restated lowering (TEST
INFRASTRUCTURE; run in a subprocess by tests/test_lowering.py with the OPT /
FG_LOWERING_REPAIR setting under test).

argv: seed count.  Prints one JSON object: {"checked": n, "differ": [...],
"rejected": {message kind: count}, "other": [...]} -- a graph the passes
lower must give the front end's bits; one they reject is counted by the kind
of rejection, and a rejection of another kind is listed under "other".
"""
import importlib.util
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
import _lowering as L  # noqa: E402

_spec = importlib.util.spec_from_file_location(
    "hostdev_fuzz", os.path.join(ROOT, "tests", "hostdev", "run_fuzz.py"))
gen = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(gen)

# How the reference's passes, as read, reject a graph:
#  - a reshape that is not a pure squeeze, above a multi-axis view that is
#    not a buffer, pushes one flat index into a source indexed by several
#    (src/schedule/indexing.rs:143-174), which flat_index's length check
#    (:43) or the Permute / Reshape branches (:136-170, indexing past that
#    one index) stop;
#  - with upcast on, a reduction over an axis of size 1: the linearizer's run
#    count is the product of the enclosing ranges' extents
#    (src/linearize.rs:49-58,101-107), so it does not tell a node inside the size-1
#    loop from one after it, and an index shared by the loop's loads and the
#    store after the loop is declared inside the loop -- the C does not
#    compile.
KINDS = {
    "flat_index: rank mismatch": "flat index into a multi-axis source",
    "permute index out of range": "flat index into a multi-axis source",
    "reshape index out of range": "flat index into a multi-axis source",
    "undeclared": "index declared inside a size-1 loop",
}


def main(seed, count):
    L.set_repair(os.environ.get("FG_LOWERING_REPAIR") == "1")
    out = {"checked": 0, "differ": [], "rejected": {}, "other": []}
    for i in range(count):
        rng = np.random.default_rng(seed * 100000 + i)
        node = gen.rand_graph(rng)
        front = node.build(gen.Env(False)).numpy()
        x = node.build(gen.Env(False))
        try:
            L.realize([x])
        except RuntimeError as e:
            kind = next((v for k, v in KINDS.items() if k in str(e)), None)
            if kind is None:
                out["other"].append(f"{i}: {str(e)[:300]}")
            else:
                out["rejected"][kind] = out["rejected"].get(kind, 0) + 1
            continue
        ours = x.numpy()
        out["checked"] += 1
        if not (np.array_equal(front, ours, equal_nan=True) and front.dtype == ours.dtype):
            d = float(np.nanmax(np.abs(front.astype(np.float64) - ours.astype(np.float64))))
            out["differ"].append(f"{i}: max_abs {d:.3e}")
    print(json.dumps(out))


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]))
