"""IDX parsing of the MNIST loader (src/dataset.rs:108-162), on the host."""
import os
import struct

import numpy as np
import pytest

from ferrograd_b200 import dataset as D


def synth(tmp_path, n_train=64, n_test=16, seed=0):
    rng = np.random.default_rng(seed)
    tr = rng.integers(0, 256, (n_train, 784), dtype=np.uint8)
    te = rng.integers(0, 256, (n_test, 784), dtype=np.uint8)
    trl = rng.integers(0, 10, n_train, dtype=np.uint8)
    tel = rng.integers(0, 10, n_test, dtype=np.uint8)
    D.write_idx(str(tmp_path), tr, trl, te, tel)
    return tr, trl, te, tel


def test_idx_round_trip(tmp_path):
    tr, trl, te, tel = synth(tmp_path)
    px, count = D.parse_image_bytes(os.path.join(tmp_path, D.FILES[0]))
    assert count == 64 and np.array_equal(px, tr)
    assert np.array_equal(D.parse_labels(os.path.join(tmp_path, D.FILES[1])), trl)
    px, count = D.parse_image_bytes(os.path.join(tmp_path, D.FILES[2]))
    assert count == 16 and np.array_equal(px, te)


def test_bad_magic_and_dims_are_format_errors(tmp_path):
    p = tmp_path / "x"
    p.write_bytes(struct.pack(">IIII", 2049, 1, 28, 28) + bytes(784))
    with pytest.raises(D.DatasetError, match="expected IDX image magic 2051, got 2049"):
        D.parse_image_bytes(str(p))
    p.write_bytes(struct.pack(">IIII", 2051, 1, 32, 32) + bytes(1024))
    with pytest.raises(D.DatasetError, match="expected 28x28 images, got 32x32"):
        D.parse_image_bytes(str(p))
    p.write_bytes(struct.pack(">II", 2051, 3) + bytes(3))
    with pytest.raises(D.DatasetError, match="expected IDX label magic 2049, got 2051"):
        D.parse_labels(str(p))
    p.write_bytes(struct.pack(">IIII", 2051, 2, 28, 28) + bytes(784))
    with pytest.raises(D.DatasetError, match="truncated"):
        D.parse_image_bytes(str(p))


def test_missing_files_name_the_file(tmp_path):
    with pytest.raises(FileNotFoundError, match="train-images-idx3-ubyte"):
        D.MNISTDataset.load(str(tmp_path))
