"""The peer-sharded exchange's owner pass (k_peer_wait + k_peer_reduce_sgd)
on one GPU, through fg_peer_reduce_sgd_local: every simulated sender's
contribution is placed in the staging area by the test instead of by a
peer's copy engine.

1. With every sender's flag already raised, the owned shard receives the
   rank-order sum of the contributions, the SGD update p + (-(g*lr))
   (src/optim.rs:60-71) with its TF32 residual, and the loss slot the summed
   value -- bit for bit what numpy computes with one rounding per operation;
   nothing outside the owned shard is written.
2. With a flag that nothing sets, the bounded wait gives up after its short
   limit, the call returns FG_ERR_DEVICE, nothing is written, and the device
   stays usable.
"""
import ctypes

import numpy as np
import pytest
import torch

from ferrograd_b200 import _lib

pytestmark = pytest.mark.gpu

FG_ERR_DEVICE = 5


def _call(grad, stage, p_cur, p_next, lo_next, shard, rank, nranks, lr, loss_idx, flags, val,
          wait_ms):
    return _lib.lib().fg_peer_reduce_sgd_local(
        grad.data_ptr(), stage.data_ptr(), p_cur.data_ptr(), p_next.data_ptr(), lo_next.data_ptr(),
        shard, rank, nranks, ctypes.c_float(lr), loss_idx, flags.data_ptr(), val, wait_ms,
        torch.cuda.current_stream().cuda_stream)


def _inputs(nranks, shard, seed):
    rng = np.random.default_rng(seed)
    n = nranks * shard
    grad = rng.standard_normal(n, dtype=np.float32) * np.float32(1e-2)
    stage = rng.standard_normal(n, dtype=np.float32) * np.float32(1e-2)
    p_cur = rng.standard_normal(n, dtype=np.float32) * np.float32(0.05)
    return grad, stage, p_cur


def _tf32_rest(v):
    hi = (v.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    return (v - hi).astype(np.float32)


@pytest.mark.parametrize("nranks,rank", [(2, 0), (4, 1), (8, 7)])
def test_owner_pass_matches_numpy_bit_for_bit(nranks, rank):
    shard, lr, val = 4096, np.float32(0.01), 3
    grad, stage, p_cur = _inputs(nranks, shard, 100 + nranks)
    base = rank * shard
    loss_idx = base + 5
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in
         (("grad", grad), ("stage", stage), ("p_cur", p_cur))}
    p_next = torch.full((nranks * shard,), float("nan"), device="cuda")
    lo_next = torch.full_like(p_next, float("nan"))
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    for j in range(nranks):
        if j != rank:
            flags[j] = val
    rc = _call(d["grad"], d["stage"], d["p_cur"], p_next, lo_next, shard, rank, nranks, lr,
               loss_idx, flags, val, 1000)
    assert rc == 0, _lib.lib().fg_last_error()

    own = slice(base, base + shard)
    acc = None
    for j in range(nranks):
        c = grad[own] if j == rank else stage[j * shard:(j + 1) * shard]
        acc = c.copy() if acc is None else (acc + c).astype(np.float32)
    pn = (p_cur[own] + (-(acc * lr).astype(np.float32))).astype(np.float32)
    pn[loss_idx - base] = acc[loss_idx - base]
    got_grad = d["grad"].cpu().numpy()
    got_p = p_next.cpu().numpy()
    got_lo = lo_next.cpu().numpy()
    assert np.array_equal(got_grad[own], acc)
    assert np.array_equal(got_p[own], pn)
    assert np.array_equal(got_lo[own], _tf32_rest(pn))
    # only the owned shard is written
    outside = np.ones(nranks * shard, bool)
    outside[own] = False
    assert np.array_equal(got_grad[outside], grad[outside])
    assert np.isnan(got_p[outside]).all() and np.isnan(got_lo[outside]).all()


def test_expired_wait_reports_the_device_error_and_writes_nothing():
    nranks, rank, shard, lr, val = 2, 0, 1024, 0.01, 1
    grad, stage, p_cur = _inputs(nranks, shard, 7)
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in
         (("grad", grad), ("stage", stage), ("p_cur", p_cur))}
    p_next = torch.full((nranks * shard,), float("nan"), device="cuda")
    lo_next = torch.full_like(p_next, float("nan"))
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")  # nothing raises rank 1's flag
    rc = _call(d["grad"], d["stage"], d["p_cur"], p_next, lo_next, shard, rank, nranks, lr, -1,
               flags, val, 50)
    assert rc == FG_ERR_DEVICE
    assert b"" != _lib.lib().fg_last_error()
    assert np.array_equal(d["grad"].cpu().numpy(), grad)
    assert torch.isnan(p_next).all() and torch.isnan(lo_next).all()
    # the error word was read and cleared; the context still works
    assert _lib.lib().fg_check_device_error() == 0
    flags[1] = val
    rc = _call(d["grad"], d["stage"], d["p_cur"], p_next, lo_next, shard, rank, nranks, lr, -1,
               flags, val, 1000)
    assert rc == 0, _lib.lib().fg_last_error()
    assert not torch.isnan(p_next[:shard]).any()
