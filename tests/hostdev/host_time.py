"""Host work per step of the front end, timed alone (TEST INFRASTRUCTURE; a
measurement, not a test): the config-1 training step (784-128-10, batch 256,
default mode) through the Tensor API on the host test device built with
FG_HOSTDEV_NOEXEC, where every launch and routed call returns without
computing, so what remains is graph building, scheduling, routing and launch
preparation.

    python tests/hostdev/host_time.py [steps]

Prints the mean host time per step, its parts, and the front end's counters.
"""
import importlib.util
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(steps):
    spec = importlib.util.spec_from_file_location("hostdev_build", os.path.join(HERE, "build.py"))
    hb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(hb)
    out = hb.build(noexec=True)
    os.environ["FG_FRONT_EXACT"] = "0"
    os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(out, "kcache"))
    os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
    sys.path.insert(0, out)
    import _front as F

    dims, batch = (784, 128, 10), 256
    rng = np.random.default_rng(0)
    x = rng.random((batch, dims[0]), dtype=np.float32)
    t = np.zeros((batch, dims[-1]), np.float32)
    t[np.arange(batch), rng.integers(0, dims[-1], batch)] = 1
    F.reset_init_seed(42)
    layers = [F.Linear(dims[i], dims[i + 1]) for i in range(len(dims) - 1)]
    opt = F.Sgd([p for l in layers for p in l.parameters()], 0.01)
    xt, tt = F.Tensor.new(x), F.Tensor.new(t)

    def step():
        t0 = time.perf_counter()
        h = xt
        for i, l in enumerate(layers):
            h = l.forward(h)
            if i + 1 < len(layers):
                h = h.relu()
        loss = h.cross_entropy(tt)
        opt.zero_grad()
        t1 = time.perf_counter()
        loss.backward()
        t2 = time.perf_counter()
        opt.step()
        t3 = time.perf_counter()
        loss.to_vec()
        t4 = time.perf_counter()
        return np.array([t1 - t0, t2 - t1, t3 - t2, t4 - t3])

    for _ in range(20):
        step()
    F.reset_stats()
    acc = np.zeros(4)
    t0 = time.perf_counter()
    for _ in range(steps):
        acc += step()
    total = (time.perf_counter() - t0) / steps * 1e6
    acc = acc / steps * 1e6
    print(f"host work per step {total:.1f} us: forward graph {acc[0]:.1f}, backward graph "
          f"{acc[1]:.1f}, Sgd::step {acc[2]:.1f}, loss read {acc[3]:.1f}")
    st = F.stats()
    print({k: (round(v / steps * 1e6, 1) if k.endswith("_s") else v / steps) for k, v in st.items()})


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 2000)
