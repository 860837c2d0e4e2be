"""Edge cases of the default mode's fused routes on the host test device
(TEST INFRASTRUCTURE; run in a subprocess by tests/test_hostdev_front.py).

argv: output .npz.
"""
import os
import sys

import numpy as np

os.environ["FG_FRONT_EXACT"] = "0"
_BUILD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(_BUILD, "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, _BUILD)
import _front as F  # noqa: E402


def main(dst):
    rng = np.random.default_rng(17)
    out = {}
    x = (rng.standard_normal((12, 7)) * 2).astype(np.float32)
    t = np.zeros((12, 7), np.float32)
    t[np.arange(12), rng.integers(0, 7, 12)] = 1
    soft = rng.random((12, 7)).astype(np.float32)
    soft /= soft.sum(1, keepdims=True)
    out.update(x=x, t=t, soft=soft)
    T = F.Tensor.new

    # 1. targets that need a gradient: the reference's decomposed graph
    F.reset_stats()
    lg = T(x).with_requires_grad(True)
    tg = T(soft).with_requires_grad(True)
    loss = lg.cross_entropy(tg)
    dl, dt = loss.gradient([lg, tg])
    F.Tensor.realize_many([dl, dt, loss])
    out["dec_loss"], out["dec_dl"], out["dec_dt"] = loss.numpy(), dl.numpy(), dt.numpy()
    out["dec_xent"] = np.array(F.stats()["xent"])

    # 2. the loss read before its gradient: two fused passes, same values
    F.reset_stats()
    lg = T(x).with_requires_grad(True)
    tt = T(t)
    loss = lg.cross_entropy(tt)
    (dl,) = loss.gradient([lg])  # built first: realizing loss drops its graph
    out["first_loss"] = loss.numpy()
    out["first_dl"] = dl.numpy()
    st = F.stats()
    out["first_xent"], out["first_reused"] = np.array(st["xent"]), np.array(st["xent_reused"])

    # 3. a scaled loss: the fused gradient times the incoming gradient
    lg = T(x).with_requires_grad(True)
    loss3 = lg.cross_entropy(tt).mul(F.Tensor.scalar(3.0))
    (dl3,) = loss3.gradient([lg])
    out["scaled_dl"] = dl3.numpy()

    # 4. alternating graph shapes through the schedule cache
    F.reset_stats()
    vals = []
    for i in range(4):
        n = 5 if i % 2 == 0 else 6
        a = T(np.full((n, 8), float(i + 1), np.float32))
        vals.append(a.mul(a).sum([1]).numpy().ravel())
    out["alt0"], out["alt1"], out["alt2"], out["alt3"] = vals
    out["alt_hits"] = np.array(F.stats()["schedule_hits"])

    # 5. an SGD store whose gradient is a non-contiguous view: rendered
    F.reset_stats()
    w0 = rng.standard_normal((6, 4)).astype(np.float32)
    w = T(w0).with_requires_grad(True)
    g = w.permute([1, 0]).mul(T(np.arange(24, dtype=np.float32).reshape(4, 6))).sum([0, 1])
    g.backward()
    opt = F.Sgd([w], 0.5)
    opt.step()
    out["w0"], out["w1"] = w0, w.numpy()
    out["sgd_count"] = np.array(F.stats()["sgd"])

    # 6. an axis of 1 expanded to 0: its gradient is the sum over nothing
    z = T(rng.standard_normal((1, 64)).astype(np.float32)).with_requires_grad(True)
    z.expand([0, 64]).relu().sum([0, 1]).backward()
    out["zero_expand_grad"] = z.grad().numpy()
    np.savez(dst, **out)


if __name__ == "__main__":
    main(sys.argv[1])
