"""The front end's schedule and rendered kernels executed on the CPU (a
host implementation of the device ABI, tests/hostdev/) -- an independent
second oracle for exact mode: whole training steps of Linear/relu/
cross_entropy/backward/Sgd must equal the C oracle bit for bit.  Runs
without a GPU; the kernels are the same CUDA C the GPU build compiles.
The default (routed) mode runs here too, its GEMM / reduction / residual
building blocks restated on the CPU from their C-ABI contracts, held to the
GPU tests' tolerance."""
import os
import subprocess
import sys

import numpy as np
import pytest

from ferrograd_b200 import data

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def hostdev():
    sys.path.insert(0, os.path.join(HERE, "hostdev"))
    try:
        import build as hb
        hb.build()
    finally:
        sys.path.pop(0)
    return os.path.join(HERE, "hostdev", "run_step.py")


def run(runner, tmp_path, dims, batch, steps, lr=0.01, seeds=(1, 2), opt=None, routed=False):
    x, t = data.mlp_batch(batch, dims[0], dims[-1], *seeds)
    src, dst = tmp_path / "in.npz", tmp_path / "out.npz"
    np.savez(src, x=x, t=t, dims=np.array(dims), lr=np.array(lr), steps=np.array(steps))
    env = dict(os.environ)
    env.pop("OPT", None)
    env["FG_FRONT_EXACT"] = "0" if routed else "1"
    if opt is not None:
        env["OPT"] = opt
    subprocess.run([sys.executable, runner, str(src), str(dst)], check=True, timeout=600, env=env)
    return x, t, dict(np.load(dst))


@pytest.mark.parametrize("dims,batch", [((64, 32, 10), 32), ((48, 40, 24, 10), 16)])
def test_host_executed_step_matches_oracle_bitwise(oracle, hostdev, tmp_path, dims, batch):
    x, t, r = run(hostdev, tmp_path, dims, batch, steps=1)
    nl = len(dims) - 1
    ws = [r[f"w0_{i}"] for i in range(nl)]
    bs = [r[f"b0_{i}"] for i in range(nl)]
    oloss, ow, ob, odw, odb, _ = oracle.mlp_step(ws, bs, x, t, 0.01)
    assert np.float32(r["loss"][0]) == np.float32(oloss)
    for i in range(nl):
        assert np.array_equal(r[f"dw_{i}"], odw[i])
        assert np.array_equal(r[f"db_{i}"], odb[i])
        assert np.array_equal(r[f"w_{i}"], ow[i]) and np.array_equal(r[f"b_{i}"], ob[i])


def test_host_executed_steps_track_oracle_and_reuse_programs(oracle, hostdev, tmp_path):
    dims = (32, 16, 10)
    x, t, r = run(hostdev, tmp_path, dims, 16, steps=3)
    ws, bs = [r["w0_0"], r["w0_1"]], [r["b0_0"], r["b0_1"]]
    for s in range(3):
        oloss, ws, bs, _, _, _ = oracle.mlp_step(ws, bs, x, t, 0.01)
        assert np.float32(r["loss"][s]) == np.float32(oloss)
    assert np.array_equal(r["w_0"], ws[0]) and np.array_equal(r["w_1"], ws[1])


@pytest.mark.parametrize("opt,unroll", [("0", False), ("symbolic,upcast", False),
                                        ("unroll", True), ("symbolic, unroll ,upcast", True)])
def test_host_executed_step_follows_the_reference_opt_setting(oracle, hostdev, tmp_path, opt,
                                                              unroll):
    """OPT (src/optimize/mod.rs:80-112) changes the arithmetic: without the
    unroll pass every reduction (the contractions over K and the batch, the
    row sums of log_softmax) is one sequential chain instead of 4-lane
    blocks.  The step must equal the oracle run with the same reduction
    order, bit for bit; with symbolic off nothing is folded, which leaves
    this step's values unchanged."""
    dims, batch = (64, 32, 10), 32
    x, t, r = run(hostdev, tmp_path, dims, batch, steps=1, opt=opt)
    ws, bs = [r["w0_0"], r["w0_1"]], [r["b0_0"], r["b0_1"]]
    oracle.set_unroll(unroll)
    try:
        oloss, ow, ob, odw, odb, _ = oracle.mlp_step(ws, bs, x, t, 0.01)
    finally:
        oracle.set_unroll(True)
    assert np.float32(r["loss"][0]) == np.float32(oloss)
    for i in range(2):
        assert np.array_equal(r[f"dw_{i}"], odw[i]), i
        assert np.array_equal(r[f"w_{i}"], ow[i]) and np.array_equal(r[f"b_{i}"], ob[i]), i
    if not unroll:
        # the sequential order is a different computation: it must not
        # coincide with the default (4-lane) one
        _, _, _, ddw, _, _ = oracle.mlp_step(ws, bs, x, t, 0.01)
        assert not np.array_equal(odw[0], ddw[0])


@pytest.mark.parametrize("level", [1, 2, 3, 4])
def test_debug_levels_follow_the_reference(hostdev, tmp_path, level):
    """DEBUG (src/tensor.rs:62-67): >= 1 one line per launch, "(compiled)"
    on a program-cache miss from 2 on (:870-874), >= 2 each launch's exec
    time (:1017-1028), >= 3 each kernel's graph (:855-869), >= 4 the
    rendered source (:852-854)."""
    x, t = data.mlp_batch(8, 16, 10, 1, 2)
    src, dst = tmp_path / "in.npz", tmp_path / "out.npz"
    np.savez(src, x=x, t=t, dims=np.array((16, 16, 10)), lr=np.array(0.01), steps=np.array(1))
    env = dict(os.environ, DEBUG=str(level))
    env.pop("OPT", None)
    r = subprocess.run([sys.executable, hostdev, str(src), str(dst)], env=env, timeout=600,
                       capture_output=True, text=True, check=True)
    lines = r.stderr.splitlines()
    launches = [l for l in lines if l.startswith("*** CUDA ")]
    assert launches
    compiled = [l for l in launches if "kernel_" in l]
    assert compiled and all(l.endswith("(compiled)") == (level >= 2) for l in compiled)
    times = [l for l in lines if l.strip().startswith("exec time=")]
    assert len(times) == (len(launches) if level >= 2 else 0)
    dumps = [l for l in lines if "[schedule]" in l]
    assert (len(dumps) > 0) == (level >= 3)
    assert any("extern \"C\" __global__" in l for l in lines) == (level >= 4)


def test_host_routed_step_matches_oracle_within_tolerance(oracle, hostdev, tmp_path):
    """The default (routed) mode on the host test device: contractions go to
    the GEMM contract (operands in place or staged, TF32 residuals made or
    reused), the rest is rendered.  Held to the GPU tests' 1e-4 and
    ReLU-tie-aware check (tests/mlp_check.py)."""
    from mlp_check import check_step
    dims, batch = (512, 256, 256, 10), 64
    x, t, r = run(hostdev, tmp_path, dims, batch, steps=1, routed=True)
    assert int(r["gemm"]) >= 4  # both forward contractions, both dW, the dX of layer 1
    # the fused routes: one cross-entropy pass whose loss to_vec() reuses,
    # SGD stores for the routed dW, the ReLU-masked dX as a GEMM epilogue
    # (a zero-initialised bias takes the plain product on the first step)
    assert int(r["xent"]) == 1 and int(r["xent_reused"]) == 1
    assert int(r["sgd"]) >= 2 and int(r["gemm_mask"]) == 1
    nl = len(dims) - 1
    ws = [r[f"w0_{i}"] for i in range(nl)]
    bs = [r[f"b0_{i}"] for i in range(nl)]
    oacts = []
    out = oracle.mlp_step(ws, bs, x, t, 0.01, acts=oacts)
    assert abs(float(r["loss"][0]) - out[0]) <= 1e-4 * abs(out[0])
    gacts = [r[f"act_{i}"] for i in range(nl - 1)]
    grads = ([r[f"dw_{i}"] for i in range(nl)], [r[f"db_{i}"] for i in range(nl)])
    params = ([r[f"w_{i}"] for i in range(nl)], [r[f"b_{i}"] for i in range(nl)])
    check_step(ws, bs, x, t, 0.01, gacts, grads, params, out, oacts, tol=1e-4)


def test_host_routed_steps_track_oracle(oracle, hostdev, tmp_path):
    """Three routed steps: the TF32 residual of each parameter is cached per
    version of its contents, so after every SGD store it must be remade; a
    stale residual would drift from the oracle here."""
    dims, batch = (512, 256, 256, 10), 64
    x, t, r = run(hostdev, tmp_path, dims, batch, steps=3, routed=True, seeds=(7, 8))
    # steps 2 and 3 add the updated biases in the forward GEMMs' epilogue
    assert int(r["gemm_bias"]) >= 4 and int(r["schedule_hits"]) >= 4
    ws = [r[f"w0_{i}"] for i in range(3)]
    bs = [r[f"b0_{i}"] for i in range(3)]
    w0 = [w.copy() for w in ws]
    for s in range(3):
        oloss, ws, bs, _, _, _ = oracle.mlp_step(ws, bs, x, t, 0.01, want_grads=False)
        assert abs(float(r["loss"][s]) - oloss) <= 1e-4 * abs(oloss), s
    for i in range(3):
        d_got, d_ref = r[f"w_{i}"] - w0[i], ws[i] - w0[i]
        assert np.max(np.abs(d_got - d_ref)) <= 3e-4 * np.max(np.abs(d_ref)), i


def test_host_routed_matmul_and_big_reductions(oracle, hostdev, tmp_path):
    runner = os.path.join(os.path.dirname(hostdev), "run_ops.py")
    dst = tmp_path / "ops.npz"
    subprocess.run([sys.executable, runner, str(dst)], check=True, timeout=600)
    r = dict(np.load(dst))
    assert int(r["gemm"]) == 1 and int(r["hand_reduce"]) == 3
    ref = r["a"].astype(np.float64) @ r["b"].astype(np.float64)
    assert np.max(np.abs(r["c"] - ref)) <= 1e-5 * np.max(np.abs(ref))
    x = r["x"]
    s_ref = oracle.reduce_last(x, oracle.SUM)
    assert np.max(np.abs(r["s_rows"] - s_ref)) <= 1e-4 * np.max(np.abs(s_ref))
    assert np.array_equal(r["m_rows"], oracle.reduce_last(x, oracle.MAX))
    c_ref = oracle.reduce_axis0(x, oracle.SUM)
    assert np.max(np.abs(r["s_cols"] - c_ref)) <= 1e-4 * np.max(np.abs(c_ref))


@pytest.mark.parametrize("routed", [False, True])
def test_host_narrow_batch_loop_tracks_oracle(oracle, hostdev, tmp_path, routed):
    """examples/mnist.rs's loop over narrow() batches of one resident tensor:
    each batch start is a kernel argument, so later batches reuse the
    programs.  Exact mode equals the oracle run on the same slices bit
    for bit; the routed mode (narrowed inputs reach the GEMM as strided
    views) stays within the per-step 1e-4."""
    dims, batch, nb = (512, 256, 10), 32, 4
    x, t = data.mlp_batch(batch * nb, dims[0], dims[-1], 5, 6)
    src, dst = tmp_path / "in.npz", tmp_path / "out.npz"
    np.savez(src, x=x, t=t, dims=np.array(dims), lr=np.array(0.01), batch=np.array(batch))
    env = dict(os.environ, FG_FRONT_EXACT="0" if routed else "1")
    env.pop("OPT", None)
    runner = os.path.join(os.path.dirname(hostdev), "run_narrow.py")
    subprocess.run([sys.executable, runner, str(src), str(dst)], check=True, timeout=600, env=env)
    r = dict(np.load(dst))
    assert (int(r["gemm"]) > 0) == routed
    # the first step reads the zero biases as literal zeros (never-written
    # buffers); from the second batch on every program is reused
    assert r["compiled"][-1] == r["compiled"][1]
    ws, bs = [r["w0_0"], r["w0_1"]], [r["b0_0"], r["b0_1"]]
    w0 = [w.copy() for w in ws]
    for b in range(nb):
        sl = slice(b * batch, (b + 1) * batch)
        oloss, ws, bs, _, _, _ = oracle.mlp_step(ws, bs, x[sl], t[sl], 0.01, want_grads=False)
        if routed:
            assert abs(float(r["loss"][b]) - oloss) <= 1e-4 * abs(oloss), b
        else:
            assert np.float32(r["loss"][b]) == np.float32(oloss), b
    for i in range(2):
        if routed:
            d_got, d_ref = r[f"w_{i}"] - w0[i], ws[i] - w0[i]
            assert np.max(np.abs(d_got - d_ref)) <= nb * 1e-4 * np.max(np.abs(d_ref)), i
        else:
            assert np.array_equal(r[f"w_{i}"], ws[i]) and np.array_equal(r[f"b_{i}"], bs[i]), i


def test_host_thread_mappings_and_128_bit_kernels(oracle, hostdev, tmp_path):
    """Default mode's rendered kernels (tests/hostdev/run_mapping.py):
    warp-per-output and block reductions within 1e-5 of sum|x| (f32 sums),
    bit-exact for max and for i32; the 128-bit elementwise kernels bit-exact
    (same single-rounded ops); relu(a*b+c)*0.5 in one kernel."""
    runner = os.path.join(os.path.dirname(hostdev), "run_mapping.py")
    dst = tmp_path / "map.npz"
    subprocess.run([sys.executable, runner, str(dst)], check=True, timeout=600)
    r = dict(np.load(dst))
    assert int(r["hand_reduce"]) == 0  # every case below the hand-kernel size: rendered

    def close(got, x, axis):
        ref = x.astype(np.float64).sum(axis)
        scale = np.abs(x.astype(np.float64)).sum(axis)
        assert np.all(np.abs(got.ravel() - ref.ravel()) <= 1e-5 * scale.ravel() + 1e-30)

    close(r["x_sum1"], r["x"], 1)
    close(r["c_sum0"], r["c"], 0)
    close(r["m3_sum01"], r["m3"], (0, 1))
    close(r["v_sq_sum1"], r["v"] * r["v"], 1)
    close(r["v_sum1_narrow"], r["v"][:, 4:516], 1)
    assert np.array_equal(r["x_max1"].ravel(), r["x"].max(1))
    assert np.array_equal(r["c_max0"].ravel(), r["c"].max(0))
    xi, ci = r["xi"], r["ci"]
    assert np.array_equal(r["xi_sum1"].ravel(), xi.sum(1, dtype=np.int32))
    assert np.array_equal(r["xi_max1"].ravel(), xi.max(1))
    assert np.array_equal(r["ci_sum0"].ravel(), ci.sum(0, dtype=np.int32))
    ab = r["a"].astype(np.float64) @ r["b"].astype(np.float64)
    sab = np.abs(r["a"].astype(np.float64)) @ np.abs(r["b"].astype(np.float64))
    assert np.all(np.abs(r["ab"] - ab) <= 1e-5 * sab)
    e1, e2, e3 = r["e1"], r["e2"], r["e3"]
    chain = np.maximum(e1 * e2 + e3, np.float32(0)) * np.float32(0.5)
    assert np.array_equal(r["chain"], chain)
    assert int(r["chain_kernels"]) == 1  # t = a*b+c is recomputed, not materialised
    assert np.array_equal(r["relu"], np.where(e1 > 0, e1, np.float32(0)))
    assert np.array_equal(r["relu_grad"], np.where(e1 > 0, e2, np.float32(0)))
    assert np.array_equal(r["narrow_rows"], e1[3:13] + e1[20:30])
    assert np.array_equal(r["narrow_cols"], e1[:, 1:65] * e1[:, 8:72])


@pytest.mark.parametrize("routed", [False, True])
def test_schedule_cache_replays_the_same_kernels(hostdev, tmp_path, routed, monkeypatch):
    """Steps 2.. of a training loop have the graph structure of step 1: their
    realizes reuse its schedule (leaves renamed), and every output is bit for
    bit the one the uncached scheduler gives."""
    dims, batch, steps = (48, 40, 24, 10), 16, 3
    monkeypatch.setenv("FG_SCHEDULE_CACHE", "0")
    _, _, off = run(hostdev, tmp_path, dims, batch, steps, routed=routed)
    monkeypatch.delenv("FG_SCHEDULE_CACHE")
    _, _, on = run(hostdev, tmp_path, dims, batch, steps, routed=routed)
    assert int(off["schedule_hits"]) == 0
    # per step: Sgd::step's realize and loss.to_vec()'s, all but the first
    assert int(on["schedule_hits"]) >= 2 * (steps - 1)
    for k in off:
        if k not in ("schedule_hits",):
            assert np.array_equal(off[k], on[k]), k


def test_host_fused_route_edge_cases(hostdev, tmp_path):
    """Default mode's fused routes on their edges (tests/hostdev/run_front_edges.py):
    targets needing a gradient keep the reference's decomposed graph; a loss
    read before its gradient costs a second fused pass but gives the same
    values; a scaled loss scales the fused gradient; graphs of alternating
    shapes miss and hit the schedule cache correctly; an SGD store whose
    gradient is not contiguous falls back to a rendered kernel; an axis
    expanded from 1 to 0 gets a zero gradient of the source's shape."""
    runner = os.path.join(os.path.dirname(hostdev), "run_front_edges.py")
    dst = tmp_path / "edges.npz"
    subprocess.run([sys.executable, runner, str(dst)], check=True, timeout=600)
    r = dict(np.load(dst))
    x, t, soft = (r[k].astype(np.float64) for k in ("x", "t", "soft"))
    B = x.shape[0]
    lse = np.log(np.exp(x - x.max(1, keepdims=True)).sum(1, keepdims=True)) + x.max(1, keepdims=True)
    logp = x - lse
    p = np.exp(logp)

    def near(got, ref, tol=1e-5):
        got, ref = np.asarray(got, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
        assert np.max(np.abs(got - ref)) <= tol * max(np.max(np.abs(ref)), 1e-30), (got, ref)

    assert int(r["dec_xent"]) == 0
    near(r["dec_loss"], -(soft * logp).sum() / B)
    near(r["dec_dl"], (p * soft.sum(1, keepdims=True) - soft) / B)
    near(r["dec_dt"], -logp / B)
    assert int(r["first_xent"]) == 2 and int(r["first_reused"]) == 0
    near(r["first_loss"], -(t * logp).sum() / B)
    dl = (p * t.sum(1, keepdims=True) - t) / B
    near(r["first_dl"], dl)
    near(r["scaled_dl"], 3.0 * dl)
    for i in range(4):
        assert np.array_equal(r[f"alt{i}"], np.full(5 if i % 2 == 0 else 6, 8.0 * (i + 1) ** 2))
    assert int(r["alt_hits"]) >= 2
    w0 = r["w0"].astype(np.float64)
    grad = np.arange(24, dtype=np.float64).reshape(4, 6).T
    assert np.array_equal(r["w1"], (w0 - 0.5 * grad).astype(np.float32))
    assert int(r["sgd_count"]) == 0
    assert np.array_equal(r["zero_expand_grad"], np.zeros((1, 64), np.float32))


@pytest.mark.parametrize("kind", ["fwd", "grad", "i32"])
def test_random_graphs_agree_across_modes(hostdev, tmp_path, kind):
    """Random Tensor-API graphs (tests/hostdev/run_fuzz.py): forward values of
    exact and default mode within 1e-4 of float64 (relative to the magnitude
    of the terms that make each element), gradients of the default
    mode within 1e-4 of exact mode's; gradients the reference leaves
    undefined raise in both modes; integer graphs exact in both modes."""
    runner = os.path.join(os.path.dirname(hostdev), "run_fuzz.py")
    dst = tmp_path / f"fuzz_{kind}.npz"
    subprocess.run([sys.executable, runner, "3", "30", kind, str(dst)], check=True, timeout=900)
    r = np.load(dst)
    assert list(r["failures"]) == []
    assert int(r["checked"]) >= 20
