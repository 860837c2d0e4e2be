"""The MNIST data path on the GPU: IDX bytes uploaded once and converted on
the device (bit-exact with the reference's f32::from(b) / 255.0), one-hot
targets, and the examples/mnist.rs training loop over narrow() batches of
the resident dataset."""
import ctypes

import numpy as np
import pytest
import torch

from ferrograd_b200 import dataset as D
from ferrograd_b200 import front as F
from ferrograd_b200._lib import call

pytestmark = pytest.mark.gpu


def test_u8_to_f32_div_is_bit_exact_including_unaligned_tails():
    rng = np.random.default_rng(1)
    raw = torch.from_numpy(rng.integers(0, 256, 1_000_037, dtype=np.uint8)).cuda()
    out = torch.empty(1_000_037, dtype=torch.float32, device="cuda")
    for off in (0, 3):  # 16-byte vector path and the scalar path
        n = raw.numel() - off
        call("fg_u8_to_f32_div", ctypes.c_void_p(raw.data_ptr() + off),
             ctypes.c_void_p(out.data_ptr()), n, ctypes.c_float(255.0), None)
        torch.cuda.synchronize()
        ref = raw[off:].cpu().numpy().astype(np.float32) / np.float32(255.0)
        assert np.array_equal(out[:n].cpu().numpy(), ref)


def test_dataset_tensors_match_the_reference_conversion(tmp_path):
    rng = np.random.default_rng(2)
    tr = rng.integers(0, 256, (300, 784), dtype=np.uint8)
    trl = rng.integers(0, 10, 300, dtype=np.uint8)
    D.write_idx(str(tmp_path), tr, trl, tr[:50], trl[:50])
    ds = D.MNISTDataset.load(str(tmp_path))
    assert ds.train_len() == 300 and ds.test_len() == 50
    assert ds.train_images.shape == (300, 784) and ds.train_images.is_realized()
    assert np.array_equal(ds.train_images.numpy(), tr.astype(np.float32) / np.float32(255.0))
    t = D.one_hot(trl, 10).numpy()
    ref = np.zeros((300, 10), np.float32)
    ref[np.arange(300), trl] = 1.0
    assert np.array_equal(t, ref)
    with pytest.raises(RuntimeError, match="out of range"):
        D.one_hot(np.array([3, 12], np.uint8), 10)


def test_mnist_example_loop_on_a_resident_synthetic_dataset(tmp_path):
    """examples/mnist.rs:60-124 on 2048 synthetic images: batches are narrow()
    views of the resident tensors, the loss falls, and the evaluation pass
    reads the test logits back."""
    rng = np.random.default_rng(3)
    n = 2048
    labels = rng.integers(0, 10, n, dtype=np.uint8)
    # class-dependent pixel intensities so the model has something to learn
    base = rng.integers(0, 256, (10, 784), dtype=np.uint8)
    noise = rng.integers(0, 64, (n, 784), dtype=np.uint8)
    px = np.clip(base[labels].astype(np.int32) // 2 + noise, 0, 255).astype(np.uint8)
    D.write_idx(str(tmp_path), px, labels, px[:256], labels[:256])
    ds = D.MNISTDataset.load(str(tmp_path))
    targets = D.one_hot(ds.train_labels, ds.num_classes)
    F.reset_init_seed(42)
    model = F.Mlp((784, 128, 10))
    opt = F.Sgd(model.parameters(), 0.01)
    batch = 256
    losses = []
    compiled = []
    for epoch in range(2):
        for b in range(ds.train_len() // batch):
            xb = ds.train_images.narrow(0, b * batch, batch)
            tb = targets.narrow(0, b * batch, batch)
            losses.append(F.train_step(model, opt, xb, tb))
            compiled.append(F.stats()["compiled"])
    assert np.mean(losses[-4:]) < np.mean(losses[:4])
    assert compiled[-1] == compiled[8]  # later batches reuse the programs
    logits = np.asarray(model.forward(ds.test_images).to_vec(), np.float32).reshape(256, 10)
    acc = float(np.mean(np.argmax(logits, 1) == ds.test_labels))
    assert 0.0 <= acc <= 1.0
