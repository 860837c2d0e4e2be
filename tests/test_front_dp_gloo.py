"""Data parallelism through the Tensor API (Sgd with a communicator) on the
host test device, with gloo ranks on the CPU carrying the all-reduce.

Every rank builds the same seeded model, takes its shard of the batch, and
runs the reference training loop (examples/mnist.rs:90-97) with
`Sgd.set_comm`: `step()` realizes the gradients, replaces each by its mean
over the ranks (fg_allreduce_mean_f32, here a gloo sum of the host buffer
times 1/nranks), then updates.  The loss is averaged the same way
(`Tensor.all_reduce_mean`).  Checked: at two ranks in exact mode the
parameters equal, bit for bit, the oracle's per-shard gradients summed and
halved and applied by the oracle's SGD (a sum of two floats has one order);
every mode and rank count tracks the full-batch oracle step within 1e-4;
parameters are identical across ranks."""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from test_dp_gloo import _init, free_port

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "hostdev", "_build")


def _worker(rank, world, port, routed, x, t, dims, lr, steps, q):
    try:
        import ctypes

        import torch
        os.environ["FG_FRONT_EXACT"] = "0" if routed else "1"
        os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(BUILD, "kcache"))
        sys.path.insert(0, BUILD)
        import _front as F
        dist = _init(rank, world, port)
        lib = ctypes.CDLL(os.path.join(BUILD, "libferro_cuda.so"))
        cb_type = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_size_t)

        def allreduce_sum(ptr, n):
            try:
                dist.all_reduce(torch.from_numpy(np.ctypeslib.as_array(ptr, shape=(n,))))
                return 0
            except Exception:  # reported as FG_ERR_NCCL by the caller
                return 1

        cb = cb_type(allreduce_sum)
        lib.fg_hostdev_set_allreduce.argtypes = [cb_type]
        lib.fg_hostdev_set_allreduce(cb)
        lib.fg_comm_init.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_void_p)]
        comm = ctypes.c_void_p()
        assert lib.fg_comm_init(rank, world, b"\0" * 128, 10000, ctypes.byref(comm)) == 0

        per = x.shape[0] // world
        xs = F.Tensor.new(np.ascontiguousarray(x[rank * per:(rank + 1) * per]))
        ts = F.Tensor.new(np.ascontiguousarray(t[rank * per:(rank + 1) * per]))
        F.reset_init_seed(42)
        layers = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
        opt = F.Sgd([p for l in layers for p in l.parameters()], lr)
        opt.set_comm(comm.value)
        assert opt.comm == comm.value
        losses = []
        for _ in range(steps):
            h = xs
            for i, l in enumerate(layers):
                h = l.forward(h)
                if i + 1 < len(layers):
                    h = h.relu()
            loss = h.cross_entropy(ts)
            opt.zero_grad()
            loss.backward()
            opt.step()
            loss.all_reduce_mean(comm.value)
            losses.append(loss.to_vec()[0])
        ws = [l.weight.numpy() for l in layers]
        bs = [l.bias.numpy().ravel() for l in layers]
        dist.destroy_process_group()
        q.put((rank, losses, ws, bs))
    except Exception as e:  # report, never hang the parent
        q.put((rank, repr(e), None, None))


@pytest.fixture(scope="module")
def hostdev_build():
    sys.path.insert(0, os.path.join(HERE, "hostdev"))
    try:
        import build as hb
        hb.build()
    finally:
        sys.path.pop(0)


def run_ranks(world, routed, x, t, dims, lr, steps):
    port = free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, routed, x, t, dims, lr, steps, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, losses, _, _ in res:
        assert isinstance(losses, list), (rank, losses)
    return res


def oracle_init(oracle, dims):
    rng = oracle.InitRng()
    ws, bs = zip(*[rng.linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)])
    return list(ws), [b.ravel() for b in bs]


def batch(rows, dims, seed):
    rng = np.random.default_rng(seed)
    x = rng.random((rows, dims[0]), dtype=np.float32)
    t = np.zeros((rows, dims[-1]), np.float32)
    t[np.arange(rows), rng.integers(0, dims[-1], rows)] = 1
    return x, t


def test_two_ranks_exact_mode_is_the_mean_of_shard_gradients_bitwise(oracle, hostdev_build):
    dims, rows, lr, steps = (48, 32, 10), 16, 0.05, 2
    x, t = batch(rows, dims, 7)
    res = run_ranks(2, False, x, t, dims, lr, steps)
    ws, bs = oracle_init(oracle, dims)
    half = np.float32(0.5)
    losses = []
    for _ in range(steps):
        parts = [oracle.mlp_step(ws, bs, x[r * 8:(r + 1) * 8], t[r * 8:(r + 1) * 8], lr)
                 for r in range(2)]
        losses.append((np.float32(parts[0][0]) + np.float32(parts[1][0])) * half)
        gw = [(parts[0][3][i] + parts[1][3][i]) * half for i in range(len(ws))]
        gb = [(parts[0][4][i].ravel() + parts[1][4][i].ravel()) * half for i in range(len(bs))]
        ws = [oracle.sgd(w, g, lr) for w, g in zip(ws, gw)]
        bs = [oracle.sgd(b, g, lr).ravel() for b, g in zip(bs, gb)]
    for rank, rl, rw, rb in res:
        assert np.array_equal(np.float32(rl), np.float32(losses)), (rank, rl, losses)
        for i in range(len(ws)):
            assert np.array_equal(rw[i], ws[i]), (rank, "w", i)
            assert np.array_equal(rb[i], bs[i]), (rank, "b", i)


@pytest.mark.parametrize("world,routed", [(2, True), (3, False), (3, True)])
def test_ranks_track_the_full_batch_step(oracle, hostdev_build, world, routed):
    dims, rows, lr = (40, 24, 10), 24, 0.05
    x, t = batch(rows, dims, 11)
    res = run_ranks(world, routed, x, t, dims, lr, 1)
    ws, bs = oracle_init(oracle, dims)
    loss, ow, ob, _, _, _ = oracle.mlp_step(ws, bs, x, t, lr)
    for rank, rl, rw, rb in res:
        assert abs(rl[0] - loss) <= 1e-4 * abs(loss), (rank, rl[0], loss)
        for i in range(len(ws)):
            for got, w0, ref in ((rw[i], ws[i], ow[i]), (rb[i], bs[i], ob[i].ravel())):
                d_ref = ref - w0
                err = np.max(np.abs((got - w0) - d_ref)) / np.max(np.abs(d_ref))
                assert err <= 1e-4, (rank, i, err)
    # the same parameters on every rank
    for rank, _, rw, rb in res[1:]:
        for i in range(len(ws)):
            assert np.array_equal(rw[i], res[0][2][i]) and np.array_equal(rb[i], res[0][3][i])
