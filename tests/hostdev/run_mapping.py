"""Rendered kernels of the default mode's thread mappings on the host test
device (TEST INFRASTRUCTURE; run in a subprocess by
tests/test_hostdev_front.py): warp-per-output and block-per-32-outputs
reductions (f32 and i32, ragged shapes), a multi-axis reduction, a rendered
contraction, and the 128-bit elementwise path (f32, bool output, aligned
and unaligned narrow views, the fused relu(a*b+c)*0.5 chain).

argv: output .npz.
"""
import os
import sys

import numpy as np

os.environ["FG_FRONT_EXACT"] = "0"
_BUILD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(_BUILD, "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, _BUILD)
import _front as F  # noqa: E402


def main(dst):
    rng = np.random.default_rng(9)
    out = {}
    x = rng.standard_normal((300, 100), dtype=np.float32)
    c = rng.standard_normal((257, 40), dtype=np.float32)
    xi = rng.integers(-1000, 1001, (100, 333)).astype(np.int32)
    ci = rng.integers(-1000, 1001, (333, 50)).astype(np.int32)
    m3 = rng.standard_normal((20, 50, 3), dtype=np.float32)
    a = rng.standard_normal((24, 40), dtype=np.float32)
    b = rng.standard_normal((40, 36), dtype=np.float32)
    e1, e2, e3 = (rng.standard_normal((64, 128), dtype=np.float32) for _ in range(3))
    out.update(x=x, c=c, xi=xi, ci=ci, m3=m3, a=a, b=b, e1=e1, e2=e2, e3=e3)
    T = F.Tensor.new
    F.reset_stats()
    out["x_sum1"] = T(x).sum([1]).numpy()
    out["x_max1"] = T(x).max([1]).numpy()
    out["c_sum0"] = T(c).sum([0]).numpy()
    out["c_max0"] = T(c).max([0]).numpy()
    out["xi_sum1"] = T(xi).sum([1]).numpy()
    out["xi_max1"] = T(xi).max([1]).numpy()
    out["ci_sum0"] = T(ci).sum([0]).numpy()
    out["m3_sum01"] = T(m3).sum([0, 1]).numpy()
    v = rng.standard_normal((33, 1024), dtype=np.float32)
    out["v"] = v
    tv = T(v)
    out["v_sq_sum1"] = tv.mul(tv).sum([1]).numpy()  # 128-bit lane loads
    out["v_sum1_narrow"] = tv.narrow(1, 4, 512).sum([1]).numpy()
    out["ab"] = T(a).matmul(T(b)).numpy()
    half = F.Tensor.scalar(0.5)
    hand = F.stats()["hand_reduce"]
    ta, tb, tc = T(e1), T(e2), T(e3)
    F.reset_stats()
    out["chain"] = ta.mul(tb).add(tc).relu().mul(half).numpy()
    out["chain_kernels"] = np.array(F.stats()["kernels"])
    F.reset_stats()
    # relu's mask is shared by the forward and the gradient: a bool kernel
    xr = T(e1).with_requires_grad(True)
    y = xr.relu()
    (g,) = y.mul(T(e2)).sum([0, 1]).gradient([xr])
    F.Tensor.realize_many([y, g])
    out["relu"], out["relu_grad"] = y.numpy(), g.numpy()
    t1 = T(e1)
    out["narrow_rows"] = t1.narrow(0, 3, 10).add(t1.narrow(0, 20, 10)).numpy()
    out["narrow_cols"] = t1.narrow(1, 1, 64).mul(t1.narrow(1, 8, 64)).numpy()
    st = F.stats()
    out["hand_reduce"] = np.array(st["hand_reduce"] + hand)
    np.savez(dst, **out)


if __name__ == "__main__":
    main(sys.argv[1])
