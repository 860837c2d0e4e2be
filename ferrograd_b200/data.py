"""Seeded synthetic inputs with the shapes and distributions of the five
benchmark configurations (MNIST itself is not available offline; the
reference's data loader is not on the measured path).

All generators use numpy's PCG64 (``np.random.default_rng(seed)``) in float32.
"""
from __future__ import annotations

import numpy as np


def uniform(shape, seed: int, low: float = 0.0, high: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.random(shape, dtype=np.float32)
    if low != 0.0 or high != 1.0:
        x = (x * np.float32(high - low) + np.float32(low)).astype(np.float32)
    return x


def normal(shape, seed: int, std: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return x


def one_hot(labels: np.ndarray, classes: int) -> np.ndarray:
    """examples/mnist.rs:18-25: dense one-hot targets."""
    out = np.zeros((labels.shape[0], classes), dtype=np.float32)
    out[np.arange(labels.shape[0]), labels] = 1.0
    return out


def labels(n: int, classes: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, classes, n)


def mlp_batch(batch: int, in_features: int, classes: int, x_seed: int, label_seed: int):
    """x uniform in [0,1) and one-hot targets of labels uniform over classes."""
    return uniform((batch, in_features), x_seed), one_hot(labels(batch, classes, label_seed), classes)


# Configuration constants (BASELINE configs 1..5).
C1 = dict(dims=(784, 128, 10), batch=256, lr=0.01, x_seed=1, label_seed=2)
C5 = dict(dims=(4096, 4096, 4096, 10), batch=8192, lr=0.01, x_seed=13, label_seed=14)
C2_N = 64 * 1024 * 1024
C2_X = (4096, 4096)
C3_N = 4096
C4 = (65536, 1000)
