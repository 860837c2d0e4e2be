"""The headline configuration at its own shape: the config-5 training step
(Linear(4096,4096) -> ReLU -> Linear(4096,4096) -> ReLU -> Linear(4096,10),
cross_entropy, backward, Sgd lr=0.01; examples/mnist.rs:90-97 step order,
Linear::new init of src/nn.rs:77-85, x seed 13 / labels seed 14) on the GPU
versus the oracle's step on the same batch.

This is the step `bench.py` times: global batch 8192, 128x256 tensor-core
tiles, MN-major dW at K = 8192, the skinny 4096 -> 10 layer at B = 8192, CUDA
graph replay.  A 512-row case runs the same widths at a different tile count
(stream-K tail on), so a failure there and not at 8192 points at the tiling.

Tolerances (north star): loss relative <= 1e-4; gradients and one-step
parameter deltas norm-relative <= 1e-4, ReLU-tie aware (tests/mlp_check.py):
masks may differ from the oracle's only at pre-activations within fp32
rounding of zero, and in every case the step must match a float64 evaluation
with the GPU's masks.

The data-parallel variants (2 GPUs, and every GPU present when there are 4 or
more) run the same global batch split over the ranks with either gradient
exchange and compare with the same full-batch oracle step; the ranks'
parameters must be bit-identical afterwards.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mlp_check import check_step

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

DIMS, LR = (4096, 4096, 4096, 10), 0.01
X_SEED, LABEL_SEED = 13, 14
TOL = 1e-4

_ORACLE_CACHE = {}


def _oracle_step(oracle, batch):
    """(x, t, ws, bs, oracle output, oracle hidden activations), once per batch size."""
    if batch not in _ORACLE_CACHE:
        from ferrograd_b200 import data, mlp_init
        x, t = data.mlp_batch(batch, DIMS[0], DIMS[-1], X_SEED, LABEL_SEED)
        ws, bs = mlp_init(DIMS)
        oacts = []
        out = oracle.mlp_step(ws, bs, x, t, LR, acts=oacts)
        _ORACLE_CACHE.clear()
        _ORACLE_CACHE[batch] = (x, t, ws, bs, out, oacts)
    return _ORACLE_CACHE[batch]


@pytest.mark.parametrize("batch", [512, 8192])
def test_config5_step_at_full_width_matches_oracle(oracle, batch):
    from ferrograd_b200 import CudaDevice, MlpTrainer
    x, t, ws, bs, out, oacts = _oracle_step(oracle, batch)
    tr = MlpTrainer(CudaDevice(0), DIMS, batch, LR, ws, bs, use_graph=True)
    loss = tr.step_host(x, t)
    gacts = [tr.activations(l) for l in range(len(DIMS) - 2)]
    grads, params = tr.grads(), tr.params()
    logits = tr.logits()
    tr.close()
    assert abs(loss - out[0]) <= TOL * abs(out[0]), (loss, out[0])
    lref = out[5].astype(np.float64)
    assert np.max(np.abs(logits - lref)) / np.max(np.abs(lref)) <= TOL
    check_step(ws, bs, x, t, LR, gacts, grads, params, out, oacts, tol=TOL)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dp_worker(rank, world, port, outdir, mode, q):
    sys.path.insert(0, ROOT)
    try:
        import datetime

        import torch.distributed as dist

        from ferrograd_b200 import Communicator, CudaDevice, MlpTrainer, data, dp, mlp_init
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        x, t = data.mlp_batch(8192, DIMS[0], DIMS[-1], X_SEED, LABEL_SEED)
        lo, hi = dp.shard_rows(8192, rank, world)
        xs, ts = np.ascontiguousarray(x[lo:hi]), np.ascontiguousarray(t[lo:hi])
        del x, t
        ws, bs = mlp_init(DIMS)
        comm = None
        if mode == "nccl":
            uid = dp.exchange_unique_id(dist, rank, Communicator.unique_id)
            comm = Communicator(rank, world, uid, timeout_ms=60000)
            tr = MlpTrainer(CudaDevice(rank), DIMS, hi - lo, LR, ws, bs, comm=comm, use_graph=True)
        else:
            tr = MlpTrainer(CudaDevice(rank), DIMS, hi - lo, LR, ws, bs, use_graph=True)
            tr.shard_over_peers(rank, world, lambda h: dp.all_gather_bytes(dist, h, world),
                                dist.barrier)
        loss = tr.step_host(xs, ts)
        pw, pb = tr.params()
        same = dp.digests_agree(dist, dp.params_digest(pw + pb), world)
        acts = [tr.activations(l) for l in range(len(DIMS) - 2)]
        np.savez(os.path.join(outdir, f"acts{rank}.npz"), *acts)
        if rank == 0:
            # peer mode: each shard's averaged gradient is read from its
            # owner's region, so this is the whole averaged gradient too
            gw, gb = tr.grads()
            np.savez(os.path.join(outdir, "params.npz"), *pw, *pb)
            np.savez(os.path.join(outdir, "grads.npz"), *gw, *gb)
        dist.barrier()
        tr.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
        q.put((rank, loss, same, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, False, repr(e)))


def _run_dp(oracle, world, mode, tmp_path):
    x, t, ws, bs, out, oacts = _oracle_step(oracle, 8192)
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dp_worker, args=(r, world, port, str(tmp_path), mode, q))
          for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    for r in res:
        assert r[3] is None, r[3]
        assert r[2], "parameters differ across ranks"
    # every rank reports the global (full-batch) loss
    for r in res:
        assert abs(r[1] - out[0]) <= TOL * abs(out[0]), (r[0], r[1], out[0])
    nl = len(DIMS) - 1
    acts = [np.load(os.path.join(tmp_path, f"acts{r}.npz")) for r in range(world)]
    gacts = [np.concatenate([a[f"arr_{l}"] for a in acts]) for l in range(nl - 1)]
    p = np.load(os.path.join(tmp_path, "params.npz"))
    params = ([p[f"arr_{l}"] for l in range(nl)], [p[f"arr_{nl + l}"] for l in range(nl)])
    g = np.load(os.path.join(tmp_path, "grads.npz"))
    grads = ([g[f"arr_{l}"] for l in range(nl)], [g[f"arr_{nl + l}"] for l in range(nl)])
    check_step(ws, bs, x, t, LR, gacts, grads, params, out, oacts, tol=TOL)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_config5_dp2_step_matches_full_batch_oracle(oracle, mode, tmp_path):
    _run_dp(oracle, 2, mode, tmp_path)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 or more GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_config5_dp_all_gpus_step_matches_full_batch_oracle(oracle, mode, tmp_path):
    _run_dp(oracle, min(torch.cuda.device_count(), 8), mode, tmp_path)
