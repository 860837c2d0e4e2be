"""The default mode's rendered-kernel thread mappings on the GPU.

Reductions the router leaves to the renderer run one warp per output
element (lanes split the innermost reduced axis, xor-shuffle fold) or 32
outputs per block (the 8 warps split an outer reduced axis and fold through
shared memory); elementwise chains over 16-byte aligned contiguous operands
load and store 4 elements per access; an elementwise node shared by
elementwise consumers of one kernel is recomputed there instead of
materialised (relu(a*b+c)*0.5 is one kernel).

Tolerances: f32 sums within 1e-5 of sum|x| per output (the fold order
differs from the reference's sequential one); max and every i32 result bit
for bit (max and wrap-around integer adds do not depend on the order);
elementwise results bit for bit (the same single-rounded ops).
"""
import numpy as np
import pytest

from ferrograd_b200 import front as F

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def default_mode(monkeypatch):
    monkeypatch.delenv("FG_FRONT_EXACT", raising=False)


def close_sums(got, x, axis):
    ref = x.astype(np.float64).sum(axis)
    scale = np.abs(x.astype(np.float64)).sum(axis)
    assert np.all(np.abs(got.ravel() - ref.ravel()) <= 1e-5 * scale.ravel() + 1e-30)


@pytest.mark.parametrize("shape", [(300, 100), (7, 4000), (1, 33)])
def test_warp_reductions(shape):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(shape, dtype=np.float32)
    t = F.tensor(x)
    close_sums(t.sum([1]).numpy(), x, 1)
    assert np.array_equal(t.max([1]).numpy().ravel(), x.max(1))
    xi = rng.integers(-1000, 1001, shape).astype(np.int32)
    ti = F.tensor(xi)
    assert np.array_equal(ti.sum([1]).numpy().ravel(), xi.sum(1, dtype=np.int32))
    assert np.array_equal(ti.max([1]).numpy().ravel(), xi.max(1))


@pytest.mark.parametrize("shape", [(33, 1024), (5, 4096), (3, 131072)])
def test_warp_reductions_with_128_bit_lane_loads(shape):
    rng = np.random.default_rng(7)
    x = rng.standard_normal(shape, dtype=np.float32)
    t = F.tensor(x)
    close_sums(t.mul(t).sum([1]).numpy(), x * x, 1)
    close_sums(t.narrow(1, 4, shape[1] - 8).sum([1]).numpy(), x[:, 4:-4], 1)
    assert np.array_equal(t.narrow(1, 8, shape[1] - 8).max([1]).numpy().ravel(),
                          x[:, 8:].max(1))


@pytest.mark.parametrize("shape", [(257, 40), (4000, 3), (64, 1000)])
def test_block_reductions(shape):
    rng = np.random.default_rng(2)
    x = rng.standard_normal(shape, dtype=np.float32)
    t = F.tensor(x)
    close_sums(t.sum([0]).numpy(), x, 0)
    assert np.array_equal(t.max([0]).numpy().ravel(), x.max(0))
    xi = rng.integers(-1000, 1001, shape).astype(np.int32)
    assert np.array_equal(F.tensor(xi).sum([0]).numpy().ravel(), xi.sum(0, dtype=np.int32))


def test_multi_axis_reduction_and_rendered_contraction():
    rng = np.random.default_rng(3)
    m3 = rng.standard_normal((20, 50, 3), dtype=np.float32)
    close_sums(F.tensor(m3).sum([0, 1]).numpy(), m3, (0, 1))
    a = rng.standard_normal((24, 40), dtype=np.float32)
    b = rng.standard_normal((40, 36), dtype=np.float32)
    F.reset_stats()
    got = F.tensor(a).matmul(F.tensor(b)).numpy()
    assert F.stats()["gemm"] == 0  # below the tensor-core size: rendered
    ref = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    assert np.all(np.abs(got - ref) <= 1e-5 * scale)


def test_large_i32_reductions_route_to_the_hand_kernels():
    rng = np.random.default_rng(4)
    xi = rng.integers(-1000, 1001, (1024, 1024)).astype(np.int32)
    t = F.tensor(xi)
    F.reset_stats()
    s, m, c = t.sum([1]).numpy(), t.max([1]).numpy(), t.sum([0]).numpy()
    assert F.stats()["hand_reduce"] == 3
    assert np.array_equal(s.ravel(), xi.sum(1, dtype=np.int32))
    assert np.array_equal(m.ravel(), xi.max(1))
    assert np.array_equal(c.ravel(), xi.sum(0, dtype=np.int32))


def test_elementwise_chain_is_one_128_bit_kernel():
    rng = np.random.default_rng(5)
    a, b, c = (rng.standard_normal((1000, 1024), dtype=np.float32) for _ in range(3))
    ta, tb, tc = F.tensor(a), F.tensor(b), F.tensor(c)
    F.reset_stats()
    got = ta.mul(tb).add(tc).relu().mul(F.Tensor.scalar(0.5)).numpy()
    assert F.stats()["kernels"] == 1
    assert "float4" in F.last_source()
    assert np.array_equal(got, np.maximum(a * b + c, np.float32(0)) * np.float32(0.5))


def test_128_bit_paths_with_views_and_bool_masks():
    rng = np.random.default_rng(6)
    e1, e2 = (rng.standard_normal((64, 128), dtype=np.float32) for _ in range(2))
    t1 = F.tensor(e1)
    assert np.array_equal(t1.narrow(0, 3, 10).add(t1.narrow(0, 20, 10)).numpy(),
                          e1[3:13] + e1[20:30])
    # unaligned column windows: gathered loads, 128-bit stores
    assert np.array_equal(t1.narrow(1, 1, 64).mul(t1.narrow(1, 8, 64)).numpy(),
                          e1[:, 1:65] * e1[:, 8:72])
    xr = F.tensor(e1).with_requires_grad(True)
    y = xr.relu()
    (g,) = y.mul(F.tensor(e2)).sum([0, 1]).gradient([xr])
    F.Tensor.realize_many([y, g])
    assert np.array_equal(y.numpy(), np.where(e1 > 0, e1, np.float32(0)))
    assert np.array_equal(g.numpy(), np.where(e1 > 0, e2, np.float32(0)))


def test_training_step_reaches_the_fused_kernels(oracle):
    """loss.backward(); optim.step() through the Tensor API: cross_entropy
    runs as one fg_xent_fwd_bwd pass (its loss reused by loss.to_vec()), the
    routed weight stores run on fg_sgd with the weights' TF32 residuals, and
    the step stays within 1e-4 of the oracle."""
    from ferrograd_b200 import data
    dims, batch, lr = (512, 256, 10), 256, 0.01
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 3, 4)
    F.reset_init_seed(42)
    model = F.Mlp(dims)
    ws = [layer.weight.numpy() for layer in model.layers]
    bs = [layer.bias.numpy() for layer in model.layers]
    opt = F.Sgd(model.parameters(), lr)
    F.reset_stats()
    loss = F.train_step(model, opt, F.tensor(x), F.tensor(t))
    st = F.stats()
    assert st["xent"] == 1 and st["xent_reused"] == 1
    assert st["sgd"] >= 1 and st["gemm"] >= 2
    oloss, ow, ob, _, _, _ = oracle.mlp_step(ws, bs, x, t, lr)
    assert abs(loss - oloss) <= 1e-4 * abs(oloss)
    for layer, w0, w1 in zip(model.layers, ws, ow):
        d_got, d_ref = layer.weight.numpy() - w0, w1 - w0
        assert np.max(np.abs(d_got - d_ref)) <= 1e-4 * np.max(np.abs(d_ref))
