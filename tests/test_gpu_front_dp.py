"""Data parallelism through the Tensor API (Sgd with a communicator) on
B200s.

One GPU: a one-rank NCCL communicator attached to Sgd runs the step's
all-reduce path (gradients realized, averaged in place by
fg_allreduce_mean_f32 on the front end's stream, then the update), and the
mean over one rank is the value itself, so in exact mode the step still
equals the oracle bit for bit.  Two GPUs (skipped otherwise): each rank
trains its half of the batch in exact mode, NCCL averages the gradients and
the loss, and the result tracks the full-batch oracle step within 1e-4 with
the two ranks' parameters bit-identical."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

DIMS, BATCH, LR = (512, 256, 256, 10), 512, 0.01


def _train(F, dims, x, t, lr, comm_handle, steps=1):
    F.reset_init_seed(42)
    model = F.Mlp(dims)
    ws = [l.weight.numpy() for l in model.layers]
    bs = [l.bias.numpy().ravel() for l in model.layers]
    opt = F.Sgd(model.parameters(), lr)
    opt.set_comm(comm_handle)
    xt, tt = F.tensor(x), F.tensor(t)
    losses = []
    for _ in range(steps):
        loss = model(xt).cross_entropy(tt)
        opt.zero_grad()
        loss.backward()
        opt.step()
        loss.all_reduce_mean(comm_handle)
        losses.append(loss.to_vec()[0])
    opt.set_comm(0)
    pw = [l.weight.numpy() for l in model.layers]
    pb = [l.bias.numpy().ravel() for l in model.layers]
    return ws, bs, losses, pw, pb


def test_one_rank_communicator_keeps_the_exact_step(oracle, monkeypatch):
    from ferrograd_b200 import Communicator, data
    from ferrograd_b200 import front as F
    monkeypatch.setenv("FG_FRONT_EXACT", "1")
    dims, batch = (96, 64, 10), 64
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 1, 2)
    comm = Communicator(0, 1, Communicator.unique_id(), timeout_ms=60000)
    try:
        ws, bs, losses, pw, pb = _train(F, dims, x, t, LR, comm.handle)
        F.synchronize()
    finally:
        comm.close()
    oloss, ow, ob, _, _, _ = oracle.mlp_step(ws, bs, x, t, LR)
    assert np.float32(losses[0]) == np.float32(oloss)
    for i in range(len(dims) - 1):
        assert np.array_equal(pw[i], ow[i]) and np.array_equal(pb[i], ob[i].ravel())


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    try:
        import datetime

        import torch.distributed as dist

        from ferrograd_b200 import Communicator, data, dp
        from ferrograd_b200 import front as F
        os.environ["FG_FRONT_EXACT"] = "1"
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        torch.cuda.set_device(rank)
        F.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 21, 22)
        lo, hi = dp.shard_rows(BATCH, rank, world)
        uid = dp.exchange_unique_id(dist, rank, Communicator.unique_id)
        comm = Communicator(rank, world, uid, timeout_ms=60000)
        ws, bs, losses, pw, pb = _train(F, DIMS, np.ascontiguousarray(x[lo:hi]),
                                        np.ascontiguousarray(t[lo:hi]), LR, comm.handle)
        F.synchronize()
        same = dp.digests_agree(dist, dp.params_digest(pw + pb), world)
        comm.close()
        dist.destroy_process_group()
        q.put((rank, losses[0], ws, bs, pw, pb, same))
    except Exception as e:  # report, never hang the parent
        q.put((rank, repr(e), None, None, None, None, False))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_ranks_track_the_full_batch_step(oracle):
    from ferrograd_b200 import data
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    x, t = data.mlp_batch(BATCH, DIMS[0], DIMS[-1], 21, 22)
    for rank, loss, ws, bs, pw, pb, same in res:
        assert isinstance(loss, float), (rank, loss)
        assert same, rank
        oloss, ow, ob, _, _, _ = oracle.mlp_step(ws, bs, x, t, LR)
        assert abs(loss - oloss) <= 1e-4 * abs(oloss), (rank, loss, oloss)
        for i in range(len(DIMS) - 1):
            for got, p0, ref in ((pw[i], ws[i], ow[i]), (pb[i], bs[i], ob[i].ravel())):
                d_ref = ref - p0
                err = np.max(np.abs((got - p0) - d_ref)) / np.max(np.abs(d_ref))
                assert err <= 1e-4, (rank, i, err)
