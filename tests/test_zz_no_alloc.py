"""fg_xent_fwd_bwd_noalloc: cross-entropy for callers that may not allocate.

Callers that reserve their whole device-memory budget at start-up (serving
processes, runtimes with their own pool) cannot let a library call cudaMalloc
later: it can synchronise the device, fail under fragmentation mid-job and
escape the caller's accounting.  This entry point keeps its per-row scratch in
a static array inside the library (1 MiB per GPU, FG_XENT_NOALLOC_MAX_ROWS
rows) and must give the same result as the allocating entry point.

The file is named so pytest collects it last; it passes on its own in a
fresh process as well as after the other tests.
"""
import ctypes

import pytest
import torch

from ferrograd_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_ROWS = 262144


def _run(name, x, t, need_grad=True):
    loss = torch.full((1,), float("nan"), device="cuda")
    dx = torch.full_like(x, float("nan")) if need_grad else None
    rc = getattr(_lib.lib(), name)(x.data_ptr(), t.data_ptr(), x.shape[0], x.shape[1],
                                   loss.data_ptr(), None if dx is None else dx.data_ptr(),
                                   ctypes.c_float(1.0), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    return loss, dx


@pytest.mark.parametrize("shape", [(4096, 1000), (777, 10)])
def test_noalloc_matches_allocating_entry_point_twice(shape):
    g = torch.Generator(device="cuda").manual_seed(11)
    for call in range(2):  # two calls in a row share (and reuse) the static scratch
        rows, cols = shape[0] - 3 * call, shape[1]
        x = torch.randn((rows, cols), device="cuda", generator=g) * 2
        lab = torch.randint(0, cols, (rows,), device="cuda", generator=g)
        t = torch.nn.functional.one_hot(lab, cols).float()
        ref_loss, ref_dx = _run("fg_xent_fwd_bwd", x, t)
        loss, dx = _run("fg_xent_fwd_bwd_noalloc", x, t)
        # same tolerance as the cross-entropy parity tests: loss 1e-5 relative,
        # gradient 1e-4 norm-relative (the two paths run the same kernels)
        assert abs(loss.item() - ref_loss.item()) <= 1e-5 * abs(ref_loss.item())
        assert (torch.max(torch.abs(dx - ref_dx)) / torch.max(torch.abs(ref_dx))).item() <= 1e-4


def test_noalloc_rejects_rows_beyond_the_static_limit():
    x = torch.zeros((MAX_ROWS + 1, 4), device="cuda")
    t = torch.zeros_like(x)
    loss = torch.zeros(1, device="cuda")
    rc = _lib.lib().fg_xent_fwd_bwd_noalloc(x.data_ptr(), t.data_ptr(), MAX_ROWS + 1, 4,
                                            loss.data_ptr(), None, ctypes.c_float(1.0),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # FG_ERR_INVALID
    assert b"static scratch limit" in _lib.lib().fg_last_error()
