"""Regenerate tests/golden/c1_small_step.npz, a regression pin of the oracle.

It records one C1-shaped training step (Linear(784,128) -> ReLU ->
Linear(128,10), reference init with seed 42, lr 0.01) on a 32-row seeded
batch.  Run from the repo root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle  # noqa: E402


def main():
    rng = np.random.default_rng(1)
    x = rng.random((32, 784), dtype=np.float32)
    t = np.eye(10, dtype=np.float32)[np.random.default_rng(2).integers(0, 10, 32)]
    init = oracle.InitRng()
    W1, b1 = init.linear(784, 128)
    W2, b2 = init.linear(128, 10)
    loss, Ws, bs, dWs, dbs, _ = oracle.mlp_step([W1, W2], [b1, b2], x, t, 0.01)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "c1_small_step.npz")
    np.savez_compressed(out, x=x, t=t, W1_head=W1[:2, :8], loss=np.float32(loss),
                        db2=dbs[1], W2_new=Ws[1])
    print("wrote", out, "loss", loss)


if __name__ == "__main__":
    main()
