"""Edge cases of the lazy-Tensor front end on the GPU, checked against the
reference's arithmetic: in FG_FRONT_EXACT=1 mode every kernel is rendered
with the reference's op semantics and reduction order, so results must equal
a float32 evaluation in that order bit for bit (reductions: the last reduced
axis in 4-lane blocks when R > 4 and R % 4 == 0, src/optimize/unroll.rs:
41-113; everything else one rounding per op)."""
import numpy as np
import pytest

from ferrograd_b200 import front as F

pytestmark = pytest.mark.gpu


@pytest.fixture
def exact(monkeypatch):
    monkeypatch.setenv("FG_FRONT_EXACT", "1")


def ref_reduce(x, axes, op="sum"):
    """The reference's reduction order in float32: reduced axes walked in
    axis order with one accumulator; the last reduced axis in blocks of four
    folded left to right when R > 4 and R % 4 == 0."""
    x = np.asarray(x, np.float32)
    axes = sorted(set(axes))
    keep = [a for a in range(x.ndim) if a not in axes]
    xt = np.transpose(x, keep + axes)
    out_shape = [x.shape[a] for a in keep]
    red = xt.reshape(int(np.prod(out_shape, dtype=np.int64)), -1) if axes else xt.reshape(-1, 1)
    R_last = x.shape[axes[-1]] if axes else 1
    f = (lambda a, b: np.float32(a + b)) if op == "sum" else (lambda a, b: a if a > b else b)
    init = np.float32(0.0) if op == "sum" else np.float32(-np.inf)
    res = np.empty(red.shape[0], np.float32)
    for i in range(red.shape[0]):
        row = red[i]
        acc = init
        if R_last > 4 and R_last % 4 == 0:
            for j in range(0, row.size, 4):
                h = f(f(f(row[j], row[j + 1]), row[j + 2]), row[j + 3])
                acc = f(acc, h)
        else:
            for v in row:
                acc = f(acc, v)
        res[i] = acc
    full = [1 if a in axes else x.shape[a] for a in range(x.ndim)]
    return res.reshape(full)


def rng_f32(shape, seed, lo=-2.0, hi=2.0):
    return np.random.default_rng(seed).uniform(lo, hi, shape).astype(np.float32)


def test_broadcast_and_elementwise_are_exact(exact):
    a = rng_f32((4, 1, 3), 1)
    b = rng_f32((2, 3), 2)
    s = rng_f32((1,), 3)
    got = F.tensor(a).add(F.tensor(b)).mul(F.tensor(s)).sub(F.tensor(b)).numpy()
    ref = ((a + b) * s) + (-b)
    assert got.shape == (4, 2, 3) and np.array_equal(got, ref.astype(np.float32))


def test_transcendentals_round_like_the_reference(exact):
    x = rng_f32((1000,), 4, 0.01, 8.0)
    t = F.tensor(x)
    assert np.array_equal(t.exp2().numpy(), np.exp2(x.astype(np.float64)).astype(np.float32))
    assert np.array_equal(t.log2().numpy(), np.log2(x.astype(np.float64)).astype(np.float32))
    assert np.array_equal(t.sqrt().numpy(), np.sqrt(x))
    assert np.array_equal(t.reciprocal().numpy(), np.float32(1) / x)
    log2e = np.float32(1.44269504088896340736)
    assert np.array_equal(t.exp().numpy(),
                          np.exp2((x * log2e).astype(np.float64)).astype(np.float32))


@pytest.mark.parametrize("shape,axes", [((5, 8, 12), [2]), ((5, 8, 12), [0, 2]), ((6, 10), [1]),
                                        ((6, 10), [0]), ((3, 4, 5), [1]), ((7, 1), [0, 1]),
                                        ((2, 3, 16), [0, 1, 2])])
def test_reductions_follow_the_reference_order(exact, shape, axes):
    x = rng_f32(shape, 5)
    t = F.tensor(x)
    assert np.array_equal(t.sum(axes).numpy(), ref_reduce(x, axes, "sum"))
    assert np.array_equal(t.max(axes).numpy(), ref_reduce(x, axes, "max"))


def test_permute_reshape_narrow_views(exact):
    x = rng_f32((4, 6, 5), 6)
    t = F.tensor(x)
    p = t.permute([2, 0, 1])                  # (5, 4, 6)
    assert np.array_equal(p.contiguous().numpy(), np.transpose(x, (2, 0, 1)))
    r = p.reshape([20, 6])                    # merge of permuted dims: a general reshape
    assert np.array_equal(r.numpy(), np.transpose(x, (2, 0, 1)).reshape(20, 6))
    n = t.narrow(1, 2, 3).narrow(2, 1, 3)     # inner-dim narrows
    assert np.array_equal(n.numpy(), x[:, 2:5, 1:4])
    e = F.tensor(x[:, :1, :]).expand([4, 6, 5]).add(t)
    assert np.array_equal(e.numpy(), x[:, :1, :] + x)


def test_empty_tensors(exact):
    z = F.tensor(np.zeros((0, 3), np.float32))
    assert z.add(z).numpy().shape == (0, 3)
    assert np.array_equal(z.sum([0]).numpy(), np.zeros((1, 3), np.float32))
    assert np.all(z.max([0]).numpy() == -np.inf)


def test_i32_graphs_are_bit_exact(exact):
    a = np.random.default_rng(7).integers(-1000, 1000, (9, 12), dtype=np.int32)
    b = np.random.default_rng(8).integers(-1000, 1000, (9, 12), dtype=np.int32)
    ta, tb = F.tensor(a), F.tensor(b)
    assert np.array_equal(ta.add(tb).mul(tb).numpy(), (a + b) * b)
    assert np.array_equal(ta.sum([1]).numpy().ravel(), a.sum(1))
    assert np.array_equal(ta.max([0]).numpy().ravel(), a.max(0))
    assert np.array_equal(ta.neg().numpy(), -a)


def test_cross_entropy_with_tied_maxima_matches_oracle(exact, oracle):
    """Rows with repeated maxima exercise the ReduceAxis(Max) tie-split
    gradient (src/gradient.rs:186-198)."""
    x = rng_f32((64, 12), 9)
    x[::3, 4] = x[::3, 7] = x[::3].max(1) + 1.0   # two-way ties
    x[1::3, :] = 0.5                              # all-way ties
    t = np.zeros_like(x)
    t[np.arange(64), np.arange(64) % 12] = 1.0
    xt = F.tensor(x).with_requires_grad(True)
    loss = xt.cross_entropy(F.tensor(t))
    (g,) = loss.gradient([xt])
    oloss, odx = oracle.xent_fwd_bwd(x, t)
    assert np.float32(loss.to_vec()[0]) == np.float32(oloss)
    assert np.array_equal(g.numpy(), odx)


def test_odd_shape_matmul_is_routed_with_staged_operands():
    """K = 333 is not a multiple of 4, so neither operand can be passed in
    place: both are staged into padded layouts before the tensor-core GEMM."""
    a = rng_f32((300, 333), 10, -1, 1)
    b = rng_f32((333, 515), 11, -1, 1)
    F.reset_stats()
    c = F.tensor(a).matmul(F.tensor(b)).numpy()
    assert F.stats()["gemm"] == 1
    ref = a.astype(np.float64) @ b.astype(np.float64)
    bound = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)
    assert np.max(np.abs(c - ref) / bound) <= 1e-5


def test_gradients_of_elementwise_chains(exact):
    x = rng_f32((50,), 12, 0.5, 3.0)
    t = F.tensor(x).with_requires_grad(True)
    y = t.sqrt().mul(t.log()).add(t.reciprocal()).sum([0])
    (g,) = y.gradient([t])
    xd = x.astype(np.float64)
    ref = np.log(xd) / (2 * np.sqrt(xd)) + 1 / np.sqrt(xd) - 1 / xd ** 2
    assert np.max(np.abs(g.numpy() - ref) / np.abs(ref)) <= 1e-5


def test_backward_accumulates_across_calls(exact):
    p = F.tensor(rng_f32((8,), 13)).with_requires_grad(True)
    loss = p.mul(p).sum([0])
    loss.backward()
    g1 = p.grad().numpy()
    loss.backward()
    g2 = p.grad().numpy()
    assert np.array_equal(g2, np.float32(g1 + g1))
