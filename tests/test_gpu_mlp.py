"""One MLP training step (examples/mnist.rs:90-97) on the GPU versus the oracle.

Tolerances (north star): loss relative <= 1e-4; gradients and one-step
parameter deltas norm-relative <= 1e-4 (max|gpu - ref| / max|ref|); logits
norm-relative <= 1e-5.  ReLU masks may differ from the oracle's only at
pre-activations within rounding of zero (tests/mlp_check.py).
"""
import numpy as np
import pytest

from ferrograd_b200 import CudaDevice, MlpTrainer, data, mlp_init
from mlp_check import check_step

pytestmark = pytest.mark.gpu

TOL = 1e-4


def normrel(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30)


def run_both(oracle, dims, batch, lr=0.01, seeds=(1, 2), graph=False, steps=1):
    x, t = data.mlp_batch(batch, dims[0], dims[-1], *seeds)
    ws, bs = mlp_init(dims)
    tr = MlpTrainer(CudaDevice(0), dims, batch, lr, ws, bs, use_graph=graph)
    ow, ob = [w.copy() for w in ws], [b.copy() for b in bs]
    for _ in range(steps):
        loss = tr.step_host(x, t)
        oloss, ow, ob, odw, odb, ologits = oracle.mlp_step(ow, ob, x, t, lr)
    return dict(tr=tr, x=x, t=t, ws=ws, bs=bs, loss=loss, oloss=oloss, ow=ow, ob=ob, odw=odw,
                odb=odb, ologits=ologits)


@pytest.mark.parametrize("dims,batch", [((784, 128, 10), 256),       # config 1
                                        ((512, 256, 256, 10), 384),   # config 5, scaled down
                                        ((512, 256, 256, 10), 256),
                                        ((64, 32), 64)])              # single tensor-core layer
def test_mlp_step_matches_oracle(oracle, dims, batch):
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 1, 2)
    ws, bs = mlp_init(dims)
    tr = MlpTrainer(CudaDevice(0), dims, batch, 0.01, ws, bs)
    loss = tr.step_host(x, t)
    oacts = []
    out = oracle.mlp_step(ws, bs, x, t, 0.01, acts=oacts)
    assert abs(loss - out[0]) <= TOL * abs(out[0])
    assert normrel(tr.logits(), out[5]) <= 1e-5
    gacts = [tr.activations(l) for l in range(len(dims) - 2)]
    check_step(ws, bs, x, t, 0.01, gacts, tr.grads(), tr.params(), out, oacts, tol=TOL)


def test_relu_ties_are_tolerated_but_checked(oracle):
    """A batch with ReLU pre-activations within fp32 rounding of zero (rows
    256..511 of seeds 21/22): masks may differ from the oracle's only there,
    and the step must match float64 evaluated with the GPU's masks."""
    dims = (512, 256, 256, 10)
    x, t = data.mlp_batch(512, dims[0], dims[-1], 21, 22)
    x, t = np.ascontiguousarray(x[256:]), np.ascontiguousarray(t[256:])
    ws, bs = mlp_init(dims)
    tr = MlpTrainer(CudaDevice(0), dims, 256, 0.01, ws, bs)
    loss = tr.step_host(x, t)
    oacts = []
    out = oracle.mlp_step(ws, bs, x, t, 0.01, acts=oacts)
    assert abs(loss - out[0]) <= TOL * abs(out[0])
    gacts = [tr.activations(l) for l in range(len(dims) - 2)]
    check_step(ws, bs, x, t, 0.01, gacts, tr.grads(), tr.params(), out, oacts, tol=TOL)


def test_mlp_config1_three_steps_track_oracle(oracle):
    r = run_both(oracle, (784, 128, 10), 256, steps=3)
    assert abs(r["loss"] - r["oloss"]) <= TOL * abs(r["oloss"])
    pw, _ = r["tr"].params()
    assert normrel(pw[0] - r["ws"][0], r["ow"][0] - r["ws"][0]) <= 3 * TOL


def test_graph_replay_matches_eager():
    dims, batch = (512, 256, 256, 10), 256
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 5, 6)
    ws, bs = mlp_init(dims)
    eager = MlpTrainer(CudaDevice(0), dims, batch, 0.01, ws, bs, use_graph=False)
    graph = MlpTrainer(CudaDevice(0), dims, batch, 0.01, ws, bs, use_graph=True)
    for _ in range(3):
        le = eager.step_host(x, t)
        lg = graph.step_host(x, t)
        assert le == lg
    for a, b in zip(eager.params()[0], graph.params()[0]):
        assert np.array_equal(a, b)
    assert graph.launches_per_step == eager.launches_per_step > 0


def test_loss_decreases_over_steps():
    """The integration check the reference's MNIST example makes: loss falls."""
    dims, batch = (784, 128, 10), 256
    x, t = data.mlp_batch(batch, dims[0], dims[-1], 1, 2)
    ws, bs = mlp_init(dims)
    tr = MlpTrainer(CudaDevice(0), dims, batch, 0.1, ws, bs, use_graph=True)
    losses = [tr.step_host(x, t) for _ in range(20)]
    assert losses[-1] < losses[0]


def test_unsupported_width_is_an_error():
    from ferrograd_b200 import FerroError
    with pytest.raises(FerroError):
        MlpTrainer(CudaDevice(0), (64, 40, 10), 32, 0.01, *mlp_init((64, 40, 10)))


@pytest.mark.parametrize("graph", [False, True])
def test_overlapped_upload_step_matches_plain_host_step(graph):
    """fg_mlp_step_host_next (batch i+1 uploaded while step i runs) gives
    bit-identical losses and parameters to fg_mlp_step_host over four steps
    that alternate two batches, including a call whose batch was not the
    staged one and a final call without a next batch."""
    dims, batch = (512, 256, 256, 10), 256
    xa, ta = data.mlp_batch(batch, dims[0], dims[-1], 5, 6)
    xb, tb = data.mlp_batch(batch, dims[0], dims[-1], 7, 8)
    ws, bs = mlp_init(dims)
    plain = MlpTrainer(CudaDevice(0), dims, batch, 0.01, ws, bs, use_graph=graph)
    piped = MlpTrainer(CudaDevice(0), dims, batch, 0.01, ws, bs, use_graph=graph)
    order = [(xa, ta), (xb, tb), (xa, ta), (xb, tb)]
    nexts = [(xb, tb), (xb, tb), (xb, tb), (None, None)]  # call 2 finds xa, not the staged xb
    for (x, t), (xn, tn) in zip(order, nexts):
        lp = plain.step_host(x, t)
        lq = piped.step_host_next(x, t, xn, tn)
        assert lp == lq
    for a, b in zip(plain.params()[0] + plain.params()[1], piped.params()[0] + piped.params()[1]):
        assert np.array_equal(a, b)
