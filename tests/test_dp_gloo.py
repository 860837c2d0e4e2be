"""Data-parallel host logic on CPU with world_size-2 gloo ranks.

The device math runs in the oracle here (CPU); what is tested is the
sharding, the mean of per-shard gradients equalling the full-batch gradient,
the communicator-id exchange, the cross-rank parameter digest, the
peer-sharded exchange's arithmetic over the product's chunk layout, and that
a rank which never joins a collective turns into an error on the others (not
a hang)."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _dp_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    try:
        import torch
        from ferrograd_b200 import data, dp
        from oracle import oracle as orc
        dist = _init(rank, world, port)
        dims, B, lr = (48, 32, 10), 16, 0.05
        x, t = data.mlp_batch(B, dims[0], dims[-1], 1, 2)
        rng = orc.InitRng()
        ws, bs = zip(*[rng.linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)])
        lo, hi = dp.shard_rows(B, rank, world)
        loss, _, _, dW, db, _ = orc.mlp_step(list(ws), list(bs), x[lo:hi], t[lo:hi], lr)
        flat = torch.from_numpy(np.concatenate([g.ravel() for g in dW + db] + [np.array([loss], np.float32)]))
        dist.all_reduce(flat)
        flat /= world
        full_loss, _, _, fdW, fdb, _ = orc.mlp_step(list(ws), list(bs), x, t, lr)
        ref = np.concatenate([g.ravel() for g in fdW + fdb] + [np.array([full_loss], np.float32)])
        err = np.max(np.abs(flat.numpy() - ref)) / np.max(np.abs(ref))
        uid = dp.exchange_unique_id(dist, rank, lambda: b"u" * 128)
        # SGD with the averaged gradient gives identical parameters on every rank
        off, new = 0, []
        for w in list(ws) + list(bs):
            g = flat.numpy()[off:off + w.size].reshape(w.shape)
            off += w.size
            new.append(orc.sgd(w, g, lr))
        agree = dp.digests_agree(dist, dp.params_digest(new), world)
        dist.destroy_process_group()
        q.put((rank, float(err), uid == b"u" * 128, agree))
    except Exception as e:  # report, never hang the parent
        q.put((rank, repr(e), False, False))


def test_dp_mean_of_shards_equals_full_batch():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, uid_ok, agree in res:
        assert isinstance(err, float), err
        assert err <= 1e-5, (rank, err)
        assert uid_ok and agree


def _absent_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import time

    import torch
    try:
        dist = _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left"))
            return  # leaves between steps, never joins the next collective
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(4))
            q.put((rank, "no error"))
        except Exception as e:
            q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    except Exception as e:
        q.put((rank, f"setup failed: {e!r}"))


def test_rank_that_never_joins_is_an_error():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_absent_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]


def _peer_worker(rank, world, port, q):
    """The peer-sharded exchange's arithmetic on the host: every rank lays its
    gradients out with fg_peer_layout (the product's layout), each chunk's
    shard r is summed by rank r over all ranks in rank order and updated with
    SGD (the loss slot carries the summed loss), and the updated shards are
    gathered back; the exchange itself goes over gloo instead of copy
    engines."""
    sys.path.insert(0, ROOT)
    try:
        import torch
        from ferrograd_b200 import data, dp, peer_layout
        from ferrograd_b200.mlp import peer_offsets
        from oracle import oracle as orc
        dist = _init(rank, world, port)
        dims, B, lr, chunks = (48, 64, 32, 10), 24, 0.05, 2
        x, t = data.mlp_batch(B, dims[0], dims[-1], 3, 4)
        rng = orc.InitRng()
        ws, bs = map(list, zip(*[rng.linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]))
        _, ch = peer_layout(dims, world, chunks)
        # where each layer's dW / db and the loss slot sit, from the product
        w_off, b_off, loss_off = peer_offsets(dims, world, chunks)
        G = max(o + n for o, n in ch)
        # this rank's local gradients, pre-scaled by 1/world like the step's
        lo, hi = dp.shard_rows(B, rank, world)
        loss, _, _, dW, db, _ = orc.mlp_step(ws, bs, x[lo:hi], t[lo:hi], lr)
        grad = np.zeros(G, np.float32)
        par = np.zeros(G, np.float32)
        for l in range(len(dims) - 1):
            grad[w_off[l]:w_off[l] + dW[l].size] = dW[l].ravel() / world
            grad[b_off[l]:b_off[l] + db[l].size] = db[l] / world
            par[w_off[l]:w_off[l] + ws[l].size] = ws[l].ravel()
            par[b_off[l]:b_off[l] + bs[l].size] = bs[l]
        grad[loss_off] = np.float32(np.float32(loss) / world)
        everyone = [torch.zeros(G) for _ in range(world)]
        dist.all_gather(everyone, torch.from_numpy(grad))
        parts = [e.numpy() for e in everyone]
        new = np.zeros(G, np.float32)
        for c_off, c_len in ch:
            S = c_len // world
            sl = slice(c_off + rank * S, c_off + (rank + 1) * S)
            g = parts[0][sl].copy()
            for j in range(1, world):
                g = (g + parts[j][sl]).astype(np.float32)
            upd = (par[sl] + (-(g * np.float32(lr)))).astype(np.float32)
            if c_off + rank * S <= loss_off < c_off + (rank + 1) * S:
                upd[loss_off - (c_off + rank * S)] = g[loss_off - (c_off + rank * S)]
            new[sl] = upd
        shards = [torch.zeros(G) for _ in range(world)]
        dist.all_gather(shards, torch.from_numpy(new))
        full = np.zeros(G, np.float32)
        for c_off, c_len in ch:
            S = c_len // world
            for j in range(world):
                sl = slice(c_off + j * S, c_off + (j + 1) * S)
                full[sl] = shards[j].numpy()[sl]
        pw = [full[w_off[l]:w_off[l] + ws[l].size].reshape(ws[l].shape) for l in range(len(ws))]
        pb = [full[b_off[l]:b_off[l] + bs[l].size] for l in range(len(bs))]
        agree = dp.digests_agree(dist, dp.params_digest(pw + pb), world)
        floss, fw, fb, _, _, _ = orc.mlp_step(ws, bs, x, t, lr)
        err = max(np.max(np.abs((pw[l] - ws[l]) - (fw[l] - ws[l]))) / np.max(np.abs(fw[l] - ws[l]))
                  for l in range(len(ws)))
        dist.destroy_process_group()
        q.put((rank, float(err), abs(float(full[loss_off]) - floss) / floss, agree, len(ch)))
    except Exception as e:  # report, never hang the parent
        q.put((rank, repr(e), None, False, 0))


@pytest.mark.parametrize("world", [2, 3])
def test_peer_sharded_exchange_arithmetic_on_gloo_ranks(world):
    port = free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, loss_err, agree, nchunks in res:
        assert isinstance(err, float), err
        # layer 0 (64 outputs) in 2 row blocks of 32 (a block's 32 x 48
        # floats split into 64-float shards for 2 and 3 ranks alike); layer 1
        # (32 outputs) whole, as blocks of 16 rows fall under the 32-row
        # rule; layer 2 whole
        assert nchunks == 4
        assert err <= 1e-5 and loss_err <= 1e-6, (rank, err, loss_err)
        assert agree


def test_shard_rows_partition():
    from ferrograd_b200 import dp
    spans = [dp.shard_rows(8192, r, 8) for r in range(8)]
    assert spans[0] == (0, 1024) and spans[-1] == (7168, 8192)
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        dp.shard_rows(10, 0, 3)
