"""Data-parallel training step on 2 GPUs versus the oracle's full-batch step,
with either gradient exchange: the NCCL all-reduce inside the step, or the
peer-sharded exchange (copy-engine reduce-scatter into the owning rank, its
fused reduce + SGD, copy-engine all-gather of the updated shard).  Needs two
GPUs; skipped otherwise.

Tolerance: loss relative 1e-4, gradients and parameter deltas norm-relative
1e-4 (ReLU-tie aware, tests/mlp_check.py); the two ranks' parameters must be
bit-identical after the step.  The batch (seeds 21/22) deliberately contains
pre-activations within rounding of zero.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mlp_check import check_step, normrel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

DIMS, BATCH, LR = (512, 256, 256, 10), 512, 0.01


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _make_dp_trainer(mode, rank, world, dist, lo, hi, ws, bs, graph):
    from ferrograd_b200 import Communicator, CudaDevice, MlpTrainer, dp
    if mode == "nccl":
        uid = dp.exchange_unique_id(dist, rank, Communicator.unique_id)
        comm = Communicator(rank, world, uid, timeout_ms=60000)
        return MlpTrainer(CudaDevice(rank), DIMS, hi - lo, LR, ws, bs, comm=comm,
                          use_graph=graph), comm
    tr = MlpTrainer(CudaDevice(rank), DIMS, hi - lo, LR, ws, bs, use_graph=graph)
    tr.shard_over_peers(rank, world, lambda h: dp.all_gather_bytes(dist, h, world), dist.barrier)
    return tr, None


def _worker(rank, world, port, q, graph=True, mode="nccl"):
    sys.path.insert(0, ROOT)
    try:
        import datetime

        import torch.distributed as dist

        from ferrograd_b200 import CudaDevice, MlpTrainer, data, dp, mlp_init
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 21, 22)
        lo, hi = dp.shard_rows(BATCH, rank, world)
        ws, bs = mlp_init(DIMS)
        # local (un-averaged) gradients of this shard, for the diagnostics below
        solo = MlpTrainer(CudaDevice(rank), DIMS, hi - lo, LR, ws, bs, use_graph=False)
        solo.step_host(np.ascontiguousarray(x[lo:hi]), np.ascontiguousarray(t[lo:hi]))
        local_gw, _ = solo.grads()
        solo.close()
        tr, comm = _make_dp_trainer(mode, rank, world, dist, lo, hi, ws, bs, graph)
        loss = tr.step_host(np.ascontiguousarray(x[lo:hi]), np.ascontiguousarray(t[lo:hi]))
        pw, pb = tr.params()
        gw, gb = tr.grads()
        acts = [tr.activations(l) for l in range(len(DIMS) - 2)]
        same = dp.digests_agree(dist, dp.params_digest(pw + pb), world)
        tr.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
        q.put((rank, loss, (pw, pb), same, None, (gw, gb), acts, local_gw))
    except Exception as e:
        q.put((rank, None, None, False, repr(e), None, None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer"])
@pytest.mark.parametrize("graph", [False, True])
def test_dp_step_matches_full_batch_oracle(oracle, graph, mode):
    from ferrograd_b200 import data, mlp_init
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, graph, mode)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=60)
    for r in res:
        assert r[4] is None, r[4]
        assert r[3], "parameters differ across ranks"
    x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 21, 22)
    ws, bs = mlp_init(DIMS)
    oacts = []
    out = oracle.mlp_step(ws, bs, x, t, LR, acts=oacts)
    # the all-reduced loss is the full-batch mean
    assert abs(res[0][1] - out[0]) <= 1e-4 * abs(out[0])
    # the full batch's activations are the ranks' shards stacked in rank order
    gacts = [np.concatenate([res[0][6][l], res[1][6][l]]) for l in range(len(DIMS) - 2)]
    check_step(ws, bs, x, t, LR, gacts, res[0][5], res[0][2], out, oacts)
    # averaging itself: all-reduced gradients = mean of the ranks' local ones
    for l in range(len(DIMS) - 1):
        mean_local = (res[0][7][l] + res[1][7][l]) / 2
        assert normrel(res[0][5][0][l], mean_local) <= 1e-6, l


def _steps_worker(rank, world, port, q, steps, graph, mode, push_lo=True):
    sys.path.insert(0, ROOT)
    os.environ["FG_PEER_PUSH_LO"] = "1" if push_lo else "0"
    try:
        import datetime

        import torch.distributed as dist

        from ferrograd_b200 import data, dp, mlp_init
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 23, 24)
        lo, hi = dp.shard_rows(BATCH, rank, world)
        ws, bs = mlp_init(DIMS)
        tr, comm = _make_dp_trainer(mode, rank, world, dist, lo, hi, ws, bs, graph)
        xs, ts = np.ascontiguousarray(x[lo:hi]), np.ascontiguousarray(t[lo:hi])
        losses = [tr.step_host(xs, ts) for _ in range(steps)]
        pw, pb = tr.params()
        same = dp.digests_agree(dist, dp.params_digest(pw + pb), world)
        tr.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
        q.put((rank, losses, (pw, pb), same, None))
    except Exception as e:
        q.put((rank, None, None, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("push_lo", [True, False])
@pytest.mark.parametrize("graph", [False, True])
def test_peer_sharded_steps_track_the_full_batch_oracle(oracle, graph, push_lo):
    """Five steps: both parameter buffers are read and written (even and odd
    steps), and with graphs each parity's graph is captured then replayed.
    push_lo: the all-gather carries the TF32 residuals, or each rank
    recomputes them for the arriving chunks (FG_PEER_PUSH_LO=0)."""
    from ferrograd_b200 import data, mlp_init
    world, port, steps = 2, _port(), 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_steps_worker, args=(r, world, port, q, steps, graph, "peer", push_lo))
          for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=60)
    for r in res:
        assert r[4] is None, r[4]
        assert r[3], "parameters differ across ranks"
    x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 23, 24)
    ws, bs = mlp_init(DIMS)
    w0 = [w.copy() for w in ws]
    for s in range(steps):
        oloss, ws, bs, _, _, _ = oracle.mlp_step(ws, bs, x, t, LR, want_grads=False)
        for r in res:  # every rank reports the global (full-batch) loss
            assert abs(r[1][s] - oloss) <= 1e-4 * abs(oloss), (s, r[1][s], oloss)
    # per-step tolerance 1e-4 (norm-relative), accumulated over the steps
    pw, pb = res[0][2]
    for l in range(len(DIMS) - 1):
        assert normrel(pw[l] - w0[l], ws[l] - w0[l]) <= steps * 1e-4, l
        assert normrel(pb[l], bs[l]) <= steps * 1e-4, l


@pytest.mark.parametrize("device", [0, 1])
@pytest.mark.parametrize("shard", [0, 1])
def test_shard_step_matches_oracle_on_each_device(oracle, device, shard):
    """Each rank's local step (no communicator) on its own device."""
    if device >= torch.cuda.device_count():
        pytest.skip("device not present")
    from ferrograd_b200 import CudaDevice, MlpTrainer, data, dp, mlp_init
    x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 21, 22)
    lo, hi = dp.shard_rows(BATCH, shard, 2)
    xs, ts = np.ascontiguousarray(x[lo:hi]), np.ascontiguousarray(t[lo:hi])
    ws, bs = mlp_init(DIMS)
    with torch.cuda.device(device):
        tr = MlpTrainer(CudaDevice(device), DIMS, hi - lo, LR, ws, bs)
        loss = tr.step_host(xs, ts)
        grads, params = tr.grads(), tr.params()
        gacts = [tr.activations(l) for l in range(len(DIMS) - 2)]
        tr.close()
    oacts = []
    out = oracle.mlp_step(ws, bs, xs, ts, LR, acts=oacts)
    assert abs(loss - out[0]) <= 1e-4 * abs(out[0])
    check_step(ws, bs, xs, ts, LR, gacts, grads, params, out, oacts)
