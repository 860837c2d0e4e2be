"""MNIST IDX loader for the front end (the reference's src/dataset.rs).

The IDX files are parsed on the host exactly as ``parse_images`` /
``parse_labels`` do (big-endian u32 header, magic 2051 / 2049, 28x28 images);
the pixel bytes are then uploaded once (47 MB for the training set) and
converted on the GPU to ``f32(b) / 255.0`` -- the same values the reference
computes on the host -- so the whole dataset stays resident in HBM and
``narrow(0, start, batch)`` batches are zero-copy views (a Shrink whose start
is a kernel argument).  ``one_hot`` builds the dense targets of
examples/mnist.rs:7-14 on the GPU from the label bytes.

The reference downloads missing files (``download_if_missing``); this
environment has no network, so ``MNISTDataset.load`` requires the four
decompressed IDX files to be present and says which one is missing.
"""
from __future__ import annotations

import os
import struct

import numpy as np

from . import front as F

IMAGE_MAGIC = 2051
LABEL_MAGIC = 2049
FILES = ("train-images-idx3-ubyte", "train-labels-idx1-ubyte", "t10k-images-idx3-ubyte",
         "t10k-labels-idx1-ubyte")


class DatasetError(ValueError):
    """DatasetError::BadFormat (src/dataset.rs:10-19)."""


def _read_u32(f) -> int:
    b = f.read(4)
    if len(b) != 4:
        raise DatasetError("bad IDX format: truncated header")
    return struct.unpack(">I", b)[0]


def parse_image_bytes(path: str):
    """parse_images (src/dataset.rs:116-140) up to the pixel bytes:
    returns (uint8 array [count, 784], count)."""
    with open(path, "rb") as f:
        magic = _read_u32(f)
        if magic != IMAGE_MAGIC:
            raise DatasetError(f"bad IDX format: expected IDX image magic {IMAGE_MAGIC}, "
                               f"got {magic}")
        count, rows, cols = _read_u32(f), _read_u32(f), _read_u32(f)
        if (rows, cols) != (28, 28):
            raise DatasetError(f"bad IDX format: expected 28x28 images, got {rows}x{cols}")
        data = f.read(count * rows * cols)
        if len(data) != count * rows * cols:
            raise DatasetError("bad IDX format: truncated pixel data")
    return np.frombuffer(data, np.uint8).reshape(count, rows * cols), count


def parse_labels(path: str) -> np.ndarray:
    """parse_labels (src/dataset.rs:142-155)."""
    with open(path, "rb") as f:
        magic = _read_u32(f)
        if magic != LABEL_MAGIC:
            raise DatasetError(f"bad IDX format: expected IDX label magic {LABEL_MAGIC}, "
                               f"got {magic}")
        count = _read_u32(f)
        data = f.read(count)
        if len(data) != count:
            raise DatasetError("bad IDX format: truncated label data")
    return np.frombuffer(data, np.uint8).copy()


def images_tensor(pixels: np.ndarray) -> "F.Tensor":
    """[count, 784] f32 tensor of pixels / 255, converted on the GPU."""
    return F.Tensor.from_u8(np.ascontiguousarray(pixels, np.uint8), 255.0)


def one_hot(labels, num_classes: int) -> "F.Tensor":
    """Dense one-hot targets [n, num_classes] (examples/mnist.rs:7-14), built
    on the GPU from the label bytes."""
    return F.Tensor.one_hot_u8(np.ascontiguousarray(labels, np.uint8), int(num_classes))


class MNISTDataset:
    """MNISTDataset (src/dataset.rs:21-106): images resident on the GPU as
    f32 tensors, labels on the host as bytes."""

    def __init__(self, train_images, train_labels, test_images, test_labels, num_classes=10):
        self.train_images = train_images
        self.train_labels = train_labels
        self.test_images = test_images
        self.test_labels = test_labels
        self.num_classes = num_classes

    @classmethod
    def load(cls, directory: str = "data/mnist") -> "MNISTDataset":
        for name in FILES:
            path = os.path.join(directory, name)
            if not os.path.exists(path):
                raise FileNotFoundError(
                    f"{path} is missing (no download here: place the decompressed IDX files "
                    f"in {directory})")
        tr, _ = parse_image_bytes(os.path.join(directory, FILES[0]))
        trl = parse_labels(os.path.join(directory, FILES[1]))
        te, _ = parse_image_bytes(os.path.join(directory, FILES[2]))
        tel = parse_labels(os.path.join(directory, FILES[3]))
        return cls(images_tensor(tr), trl, images_tensor(te), tel)

    def train_len(self) -> int:
        return len(self.train_labels)

    def test_len(self) -> int:
        return len(self.test_labels)


def write_idx(directory: str, train_pixels, train_labels, test_pixels, test_labels) -> None:
    """Write the four IDX files (for synthetic datasets in tests and benches)."""
    os.makedirs(directory, exist_ok=True)

    def images(path, px):
        px = np.ascontiguousarray(px, np.uint8).reshape(-1, 784)
        with open(path, "wb") as f:
            f.write(struct.pack(">IIII", IMAGE_MAGIC, px.shape[0], 28, 28))
            f.write(px.tobytes())

    def labels(path, lb):
        lb = np.ascontiguousarray(lb, np.uint8).ravel()
        with open(path, "wb") as f:
            f.write(struct.pack(">II", LABEL_MAGIC, lb.size))
            f.write(lb.tobytes())

    images(os.path.join(directory, FILES[0]), train_pixels)
    labels(os.path.join(directory, FILES[1]), train_labels)
    images(os.path.join(directory, FILES[2]), test_pixels)
    labels(os.path.join(directory, FILES[3]), test_labels)
