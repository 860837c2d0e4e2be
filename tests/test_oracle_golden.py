"""Pin the CPU oracle against the reference's own known-answer tests.

Every expected value below is copied from a test in the reference crate
(ferrograd, Rust) and cites it as file:line.  The reference cannot be built on
this machine (no Rust toolchain, no clang), so these known answers -- plus the
float64 cross-checks further down -- are what pins the oracle.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")


def load_kat():
    with open(GOLDEN) as f:
        return json.load(f)


def test_log_softmax_known_values(oracle):
    # src/tensor.rs:1171-1179
    kat = load_kat()["log_softmax"]
    got = oracle.log_softmax(np.array(kat["input"], dtype=np.float32))
    assert np.all(np.abs(got.ravel() - np.array(kat["expected"], dtype=np.float32)) < kat["tol"])


def test_cross_entropy_one_hot_mean_loss(oracle):
    # src/tensor.rs:1181-1189
    kat = load_kat()["cross_entropy"]
    loss, _ = oracle.xent_fwd_bwd(np.array(kat["logits"], np.float32),
                                  np.array(kat["targets"], np.float32), need_grad=False)
    assert abs(loss - kat["expected"]) < kat["tol"]


def test_sum_axis0_known_values(oracle):
    # src/tensor.rs:1191-1196
    kat = load_kat()["sum_axis0"]
    got = oracle.reduce_axis0(np.array(kat["input"], np.float32), oracle.SUM)
    assert got.tolist() == kat["expected"]


def test_relu_known_values(oracle):
    # src/tensor.rs:1165-1169
    kat = load_kat()["relu"]
    assert oracle.relu(np.array(kat["input"], np.float32)).tolist() == kat["expected"]


def test_max_reduce_known_values(oracle):
    # src/codegen/clang.rs:646-665 (rows [1,5,3] and [-1,0,7])
    kat = load_kat()["max_reduce"]
    got = oracle.reduce_last(np.array(kat["input"], np.float32), oracle.MAX)
    assert got.tolist() == kat["expected"]


def test_narrow_matmul_weight_gradient(oracle):
    # src/tensor.rs:1219-1227: x = [[1,2],[3,4]].narrow(0,1,1); w = [[10],[20]];
    # loss = x.matmul(w).sum([0,1]); d loss / d w = [3, 4].
    kat = load_kat()["narrow_matmul_grad"]
    x = np.array(kat["x"], np.float32)[1:2]
    w = np.array(kat["w"], np.float32)          # [K=2, N=1]
    g = np.ones((1, 1), np.float32)             # d sum / d C
    dwt = oracle.gemm_dw(x, g)                  # [N, K]
    assert dwt.T.ravel().tolist() == kat["expected"]
    c = oracle.gemm_fwd(x, np.ascontiguousarray(w.T))
    assert c.ravel().tolist() == [3 * 10 + 4 * 20]


def test_backward_of_product(oracle):
    # src/tensor.rs:1268-1276: loss = (x*y).sum, x=3, y=5 -> dx=5, dy=3
    kat = load_kat()["mul_backward"]
    x = np.array([[kat["x"]]], np.float32)
    y = np.array([[kat["y"]]], np.float32)
    g = np.ones((1, 1), np.float32)
    assert oracle.gemm_dx(g, y).item() == kat["dx"]
    assert oracle.gemm_dw(x, g).item() == kat["dy"]


def test_sgd_step_decreases_parameter(oracle):
    # src/optim.rs:80-94: p=3, target=2, loss=sum((p-t)*(p-t)), lr=0.1
    kat = load_kat()["sgd"]
    p = np.array([kat["param"]], np.float32)
    d = p - np.float32(kat["target"])
    grad = d * 1.0 + d * 1.0  # Mul rule, two contributions of (p - t) * 1
    new = oracle.sgd(p, grad.astype(np.float32), kat["lr"])
    assert new[0] < kat["param"]
    assert new[0] == np.float32(3.0) + (-(np.float32(2.0) * np.float32(0.1)))


def test_linear_init_shapes_and_zero_bias(oracle):
    # src/nn.rs:134-148
    w, b = oracle.InitRng().linear(4, 5)
    assert w.shape == (5, 4) and w.dtype == np.float32
    assert b.tolist() == [0.0] * 5


# ---------------------------------------------------------------------------
# Cross-checks of the restatement itself (not reference known answers).
# ---------------------------------------------------------------------------

def _lcg_numpy(numel, fan_in, state):
    """Second, independent restatement of src/nn.rs:17-47 in numpy float32."""
    f = np.float32
    out = []
    std = np.sqrt(f(2.0) / f(fan_in), dtype=np.float32)
    mask = (1 << 64) - 1
    while len(out) < numel:
        state = (state * 6364136223846793005 + 1) & mask
        u1 = f(state >> 33) / f(1 << 31)
        state = (state * 6364136223846793005 + 1) & mask
        u2 = f(state >> 33) / f(1 << 31)
        u1 = max(u1, np.finfo(np.float32).tiny)
        r = np.sqrt(f(-2.0) * np.log(u1), dtype=np.float32) * std
        th = f(2.0) * f(np.pi) * u2
        out.append(r * np.cos(th, dtype=np.float32))
        if len(out) < numel:
            out.append(r * np.sin(th, dtype=np.float32))
    return np.array(out, np.float32), state


def test_kaiming_lcg_matches_independent_restatement(oracle):
    rng = oracle.InitRng(42)
    a = rng.kaiming_normal((7, 9), 9)          # odd numel: last sin dropped
    b = rng.kaiming_normal((4, 3), 3)          # seed continues across layers
    ref_a, st = _lcg_numpy(63, 9, 42)
    ref_b, _ = _lcg_numpy(12, 3, st)
    # libm vs numpy transcendental functions may differ by an ulp or two
    np.testing.assert_allclose(a.ravel(), ref_a, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(b.ravel(), ref_b, rtol=2e-6, atol=1e-7)
    # Box-Muller of the first pair, worked in float64 from the raw LCG draws
    s1 = (42 * 6364136223846793005 + 1) % 2**64
    s2 = (s1 * 6364136223846793005 + 1) % 2**64
    u1, u2 = (s1 >> 33) / 2**31, (s2 >> 33) / 2**31
    w0 = np.sqrt(-2 * np.log(u1)) * np.sqrt(2 / 9) * np.cos(2 * np.pi * u2)
    assert abs(a.ravel()[0] - w0) < 1e-5


def test_reduce_blocking_rule(oracle):
    # 8 elements -> blocked ((v0+v1)+v2)+v3 per group; 10 -> sequential
    x = np.array([[1e8, 1.0, -1e8, 1.0, 3.0, 0.5, 0.25, 0.125]], np.float32)
    f = np.float32
    g0 = ((f(1e8) + f(1.0)) + f(-1e8)) + f(1.0)
    g1 = ((f(3.0) + f(0.5)) + f(0.25)) + f(0.125)
    assert oracle.reduce_last(x, oracle.SUM)[0] == (f(0) + g0) + g1
    y = np.arange(10, dtype=np.float32).reshape(1, 10)
    acc = f(0)
    for v in y.ravel():
        acc = acc + v
    assert oracle.reduce_last(y, oracle.SUM)[0] == acc


def test_reduce_i32_bit_exact(oracle):
    rng = np.random.default_rng(7)
    x = rng.integers(-1000, 1001, size=(33, 68), dtype=np.int32)
    assert np.array_equal(oracle.reduce_last(x, oracle.SUM), x.sum(axis=1, dtype=np.int64).astype(np.int32))
    assert np.array_equal(oracle.reduce_last(x, oracle.MAX), x.max(axis=1))
    assert np.array_equal(oracle.reduce_axis0(x, oracle.SUM), x.sum(axis=0, dtype=np.int64).astype(np.int32))
    assert np.array_equal(oracle.reduce_axis0(x, oracle.MAX), x.max(axis=0))
    # empty rows reduce to the identity (INT32_MIN for max, 0 for sum)
    e = np.zeros((3, 0), np.int32)
    assert oracle.reduce_last(e, oracle.MAX).tolist() == [np.iinfo(np.int32).min] * 3
    assert oracle.reduce_last(e, oracle.SUM).tolist() == [0] * 3


def test_xent_gradient_matches_float64(oracle):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 37)) * 2).astype(np.float32)
    lab = rng.integers(0, 37, 64)
    t = np.eye(37, dtype=np.float32)[lab]
    loss, dx = oracle.xent_fwd_bwd(x, t)
    xd = x.astype(np.float64)
    lse = np.log(np.exp(xd - xd.max(1, keepdims=True)).sum(1, keepdims=True)) + xd.max(1, keepdims=True)
    ref_loss = -(t * (xd - lse)).sum() / 64
    sm = np.exp(xd - lse)
    ref_dx = (sm * t.sum(1, keepdims=True) - t) / 64
    assert abs(loss - ref_loss) <= 1e-5 * abs(ref_loss)
    assert np.max(np.abs(dx - ref_dx)) <= 1e-5 * np.max(np.abs(ref_dx))


def test_gemm_family_matches_float64(oracle):
    rng = np.random.default_rng(3)
    A = rng.uniform(-1, 1, (24, 36)).astype(np.float32)
    B = rng.uniform(-1, 1, (20, 36)).astype(np.float32)
    G = rng.standard_normal((24, 20)).astype(np.float32)
    bias = rng.standard_normal(20).astype(np.float32)
    Ad, Bd, Gd = A.astype(np.float64), B.astype(np.float64), G.astype(np.float64)
    np.testing.assert_allclose(oracle.gemm_fwd(A, B, bias), Ad @ Bd.T + bias, rtol=0, atol=1e-5)
    np.testing.assert_allclose(oracle.gemm_dx(G, B), Gd @ Bd, rtol=0, atol=1e-5)
    np.testing.assert_allclose(oracle.gemm_dw(A, G), Gd.T @ Ad, rtol=0, atol=1e-5)


def test_mlp_step_matches_float64(oracle):
    rng = np.random.default_rng(5)
    init = oracle.InitRng()
    W1, b1 = init.linear(32, 16)
    W2, b2 = init.linear(16, 10)
    x = rng.uniform(0, 1, (8, 32)).astype(np.float32)
    t = np.eye(10, dtype=np.float32)[rng.integers(0, 10, 8)]
    loss, Ws, bs, dWs, dbs, logits = oracle.mlp_step([W1, W2], [b1, b2], x, t, 0.01)
    # float64 reference of the same maths
    xd = x.astype(np.float64)
    z1 = xd @ W1.T.astype(np.float64) + b1
    h = np.maximum(z1, 0)
    z2 = h @ W2.T.astype(np.float64) + b2
    lse = np.log(np.exp(z2 - z2.max(1, keepdims=True)).sum(1, keepdims=True)) + z2.max(1, keepdims=True)
    ref_loss = -(t * (z2 - lse)).sum() / 8
    g2 = (np.exp(z2 - lse) - t) / 8
    dW2 = g2.T @ h
    dh = g2 @ W2.astype(np.float64)
    g1 = dh * (z1 > 0)
    dW1 = g1.T @ xd
    assert abs(loss - ref_loss) < 1e-5
    np.testing.assert_allclose(dWs[1], dW2, atol=1e-5)
    np.testing.assert_allclose(dWs[0], dW1, atol=1e-5)
    np.testing.assert_allclose(dbs[1], g2.sum(0), atol=1e-5)
    np.testing.assert_allclose(Ws[0], W1 - 0.01 * dW1, atol=1e-6)
    assert np.array_equal(logits, oracle.gemm_fwd(oracle.relu(oracle.gemm_fwd(x, W1, b1)), W2, b2))


def test_oracle_regression_fixture(oracle):
    """The committed C1-shaped fixture (tests/golden/make_golden.py) still reproduces."""
    path = os.path.join(os.path.dirname(__file__), "golden", "c1_small_step.npz")
    fx = np.load(path)
    init = oracle.InitRng()
    W1, b1 = init.linear(784, 128)
    W2, b2 = init.linear(128, 10)
    assert np.array_equal(W1[:2, :8], fx["W1_head"])
    loss, Ws, bs, dWs, dbs, _ = oracle.mlp_step([W1, W2], [b1, b2], fx["x"], fx["t"], 0.01)
    assert np.float32(loss) == fx["loss"]
    assert np.array_equal(dbs[1], fx["db2"])
    assert np.array_equal(Ws[1], fx["W2_new"])
