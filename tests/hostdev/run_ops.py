"""Routed single operations of the front end on the host test device (TEST
INFRASTRUCTURE; run in a subprocess by tests/test_hostdev_front.py): a
Tensor-API matmul (routed to the GEMM contract) and large row/column
reductions (routed to the HBM reduction contracts), default (routed) mode.

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
    rng = np.random.default_rng(5)
    a = rng.standard_normal((384, 256), dtype=np.float32)
    b = rng.standard_normal((256, 320), dtype=np.float32)
    F.reset_stats()
    c = F.Tensor.new(a).matmul(F.Tensor.new(b)).numpy()
    gemm = F.stats()["gemm"]
    x = rng.standard_normal((2048, 1024), dtype=np.float32)
    t = F.Tensor.new(x)
    F.reset_stats()
    s_rows = t.sum([1]).numpy().ravel()
    m_rows = t.max([1]).numpy().ravel()
    s_cols = t.sum([0]).numpy().ravel()
    np.savez(dst, a=a, b=b, c=c, x=x, s_rows=s_rows, m_rows=m_rows, s_cols=s_cols,
             gemm=np.array(gemm), hand_reduce=np.array(F.stats()["hand_reduce"]))


if __name__ == "__main__":
    main(sys.argv[1])
