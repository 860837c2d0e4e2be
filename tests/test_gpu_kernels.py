"""Parity of the HBM-bound kernels against the CPU oracle (same seeded inputs).

Tolerances: elementwise and SGD are bit-exact (the kernels round each op
separately, like the reference's one-op-per-statement C); i32 reductions are
bit-exact; f32 reductions and the cross-entropy loss / gradient are checked
norm-relative, max|gpu - ref| / max|ref| <= 1e-4 (loss: relative 1e-5).
"""
import json
import os

import numpy as np
import pytest
import torch

from ferrograd_b200 import data, kernels
from ferrograd_b200._lib import REDUCE_MAX, REDUCE_SUM

pytestmark = pytest.mark.gpu

KAT = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))
RED_TOL = 1e-4


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def normrel(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30)


# --------------------------------------------------------------------------- elementwise
@pytest.mark.parametrize("n", [1, 3, 4, 1023, 1 << 20, (1 << 20) + 5])
def test_ew_bit_exact_vs_oracle(oracle, n):
    a, b, c = (data.normal(n, s) for s in (3, 4, 5))
    ref = oracle.ew_fma_relu_scale(a, b, c, 0.5)
    got = kernels.ew_fma_relu_scale(cuda(a), cuda(b), cuda(c), 0.5).cpu().numpy()
    assert np.array_equal(got, ref)


def test_ew_unaligned_tail(oracle):
    a, b, c = (data.normal(1001, s) for s in (3, 4, 5))
    ta, tb, tc = cuda(a), cuda(b), cuda(c)
    out = kernels.ew_fma_relu_scale(ta[1:], tb[1:], tc[1:], 0.5)   # 4-byte offset
    assert np.array_equal(out.cpu().numpy(), oracle.ew_fma_relu_scale(a[1:], b[1:], c[1:], 0.5))


def test_ew_full_size_property():
    """64M elements (config 2): compared with torch on the device."""
    n = data.C2_N
    g = torch.Generator(device="cuda").manual_seed(3)
    a, b, c = (torch.randn(n, device="cuda", generator=g) for _ in range(3))
    got = kernels.ew_fma_relu_scale(a, b, c, 0.5)
    ref = torch.relu(a * b + c) * 0.5
    torch.cuda.synchronize()
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)
    assert bool((got >= 0).all())


# --------------------------------------------------------------------------- reductions
@pytest.mark.parametrize("shape", [(1, 1), (3, 10), (64, 1000), (33, 4096), (257, 7)])
def test_reduce_rows_f32(oracle, shape):
    x = data.normal(shape, 6)
    for op, oop in ((REDUCE_SUM, oracle.SUM), (REDUCE_MAX, oracle.MAX)):
        got = kernels.reduce_rows(cuda(x), op).cpu().numpy().ravel()
        ref = oracle.reduce_last(x, oop)
        if op == REDUCE_MAX:
            assert np.array_equal(got, ref)
        else:
            assert normrel(got, ref) <= RED_TOL


@pytest.mark.parametrize("shape", [(1, 1), (2, 3), (10, 1000), (4096, 64), (1000, 257)])
def test_reduce_cols_f32(oracle, shape):
    x = data.normal(shape, 6)
    for op, oop in ((REDUCE_SUM, oracle.SUM), (REDUCE_MAX, oracle.MAX)):
        got = kernels.reduce_cols(cuda(x), op).cpu().numpy().ravel()
        ref = oracle.reduce_axis0(x, oop)
        if op == REDUCE_MAX:
            assert np.array_equal(got, ref)
        else:
            assert normrel(got, ref) <= RED_TOL


def test_reduce_known_answers():
    k = KAT["sum_axis0"]
    got = kernels.reduce_cols(cuda(np.array(k["input"], np.float32))).cpu().numpy().ravel()
    assert got.tolist() == k["expected"]
    k = KAT["max_reduce"]
    got = kernels.reduce_rows(cuda(np.array(k["input"], np.float32)), REDUCE_MAX).cpu().numpy()
    assert got.ravel().tolist() == k["expected"]


@pytest.mark.parametrize("shape", [(1, 1), (5, 3), (4096, 4096), (100, 1001)])
def test_reduce_i32_bit_exact(oracle, shape):
    x = np.random.default_rng(7).integers(-1000, 1001, size=shape, dtype=np.int32)
    tx = cuda(x)
    for op, oop in ((REDUCE_SUM, oracle.SUM), (REDUCE_MAX, oracle.MAX)):
        assert np.array_equal(kernels.reduce_rows(tx, op).cpu().numpy().ravel(), oracle.reduce_last(x, oop))
        assert np.array_equal(kernels.reduce_cols(tx, op).cpu().numpy().ravel(), oracle.reduce_axis0(x, oop))


def test_reduce_full_size_f32(oracle):
    """Config 2: X[4096,4096] N(0,1); sum and max over the last axis, sum over axis 0."""
    x = data.normal(data.C2_X, 6)
    tx = cuda(x)
    assert normrel(kernels.reduce_rows(tx, REDUCE_SUM).cpu().numpy().ravel(),
                   oracle.reduce_last(x, oracle.SUM)) <= RED_TOL
    assert np.array_equal(kernels.reduce_rows(tx, REDUCE_MAX).cpu().numpy().ravel(),
                          oracle.reduce_last(x, oracle.MAX))
    assert normrel(kernels.reduce_cols(tx, REDUCE_SUM).cpu().numpy().ravel(),
                   oracle.reduce_axis0(x, oracle.SUM)) <= RED_TOL


def test_reduce_rows_empty_columns():
    x = torch.zeros((3, 0), dtype=torch.int32, device="cuda")
    got = kernels.reduce_rows(x, REDUCE_MAX).cpu().numpy().ravel()
    assert got.tolist() == [np.iinfo(np.int32).min] * 3


# --------------------------------------------------------------------------- cross-entropy
def test_xent_known_answers():
    k = KAT["cross_entropy"]
    loss, dx = kernels.xent_fwd_bwd(cuda(np.array(k["logits"], np.float32)),
                                    cuda(np.array(k["targets"], np.float32)))
    assert abs(loss.item() - k["expected"]) < k["tol"]


@pytest.mark.parametrize("shape", [(1, 2), (256, 10), (8192, 10), (512, 1000), (96, 1001),
                                   (64, 2048), (33, 7)])
def test_xent_vs_oracle(oracle, shape):
    B, C = shape
    x = data.normal(shape, 11, std=2.0)
    t = data.one_hot(data.labels(B, C, 12), C)
    ref_loss, ref_dx = oracle.xent_fwd_bwd(x, t)
    loss, dx = kernels.xent_fwd_bwd(cuda(x), cuda(t))
    assert abs(loss.item() - ref_loss) <= 1e-5 * abs(ref_loss)
    assert normrel(dx.cpu().numpy(), ref_dx) <= 1e-4


def test_xent_ties_in_max():
    """Rows with repeated maxima exercise the tie-split mask of the max gradient."""
    x = np.array([[1.0, 3.0, 3.0, 0.0], [2.0, 2.0, 2.0, 2.0]], np.float32)
    t = np.array([[0, 1, 0, 0], [1, 0, 0, 0]], np.float32)
    from oracle import oracle as orc
    ref_loss, ref_dx = orc.xent_fwd_bwd(x, t)
    loss, dx = kernels.xent_fwd_bwd(cuda(x), cuda(t))
    assert abs(loss.item() - ref_loss) <= 1e-6
    assert np.max(np.abs(dx.cpu().numpy() - ref_dx)) <= 1e-6


def test_xent_full_size(oracle):
    """Config 4 shape [65536,1000], checked against the oracle on a row slice and
    through size-independent properties on the whole tensor."""
    B, C = data.C4
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((B, C), device="cuda", generator=g) * 2
    lab = torch.randint(0, C, (B,), device="cuda", generator=g)
    t = torch.nn.functional.one_hot(lab, C).float()
    loss, dx = kernels.xent_fwd_bwd(x, t)
    ref = torch.nn.functional.cross_entropy(x.double(), lab)
    assert abs(loss.item() - ref.item()) <= 1e-5 * abs(ref.item())
    # d loss / d logits rows sum to zero and equal (softmax - onehot) / B
    sm = torch.softmax(x.double(), 1)
    assert torch.max(torch.abs(dx.double() - (sm - t.double()) / B)).item() <= 1e-4 * (1.0 / B)
    xs, ts = x[:512].cpu().numpy(), t[:512].cpu().numpy()
    _, ref_dx = oracle.xent_fwd_bwd(xs, ts)
    assert normrel(dx[:512].cpu().numpy() * (B / 512), ref_dx) <= 1e-4


# --------------------------------------------------------------------------- SGD / split
@pytest.mark.parametrize("n", [1, 7, 101770, 1 << 20])
def test_sgd_bit_exact(oracle, n):
    p = data.normal(n, 1)
    g = data.normal(n, 2)
    ref = oracle.sgd(p, g, 0.01)
    tp = cuda(p)
    kernels.sgd_(tp, cuda(g), 0.01)
    assert np.array_equal(tp.cpu().numpy(), ref)


def test_sgd_writes_tf32_residual():
    p = cuda(data.normal(1000, 1))
    g = cuda(data.normal(1000, 2))
    lo = torch.empty_like(p)
    kernels.sgd_(p, g, 0.1, param_lo=lo)
    hi = (p.view(torch.int32) & -8192).view(torch.float32)
    assert torch.equal(hi + lo, p)


def test_split_lo_is_exact_residual():
    x = cuda(data.normal(4097, 5) * 100)
    lo = kernels.split_lo(x)
    hi = (x.view(torch.int32) & -8192).view(torch.float32)
    assert torch.equal(hi + lo, x)
    assert bool((lo.abs() <= x.abs() * 2.0 ** -10).all())
