"""Parity checks for a whole MLP training step, robust to ReLU ties.

ReLU's derivative jumps at 0.  Where a pre-activation lies within fp32
rounding of 0, two correct fp32 implementations that sum in different orders
(the GPU's tensor cores vs the reference's unrolled loops) can take different
branches, and a single flipped mask moves a whole row of dW by one sample's
contribution.  So the check is:

1. every element where the GPU's ReLU mask differs from the oracle's must be
   ill-conditioned: |z| / sum|terms| <= FLIP_MARGIN, with z recomputed in
   float64 from the GPU's own layer input;
2. if no mask differs, the GPU's gradients and one-step parameter deltas must
   match the oracle's (norm-relative <= tol);
3. in every case they must match a float64 evaluation of the same step that
   uses the GPU's masks (norm-relative <= tol).
"""
import numpy as np

FLIP_MARGIN = 1e-5


def normrel(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def f64_step(ws, bs, x, t, masks):
    """Loss and gradients in float64, with the hidden ReLU masks given."""
    nl = len(ws)
    acts = [x.astype(np.float64)]
    for l in range(nl):
        z = acts[-1] @ ws[l].astype(np.float64).T + bs[l].astype(np.float64)
        acts.append(z * masks[l] if l < nl - 1 else z)
    z = acts[-1]
    zmax = z.max(1, keepdims=True)
    lse = np.log(np.exp(z - zmax).sum(1, keepdims=True)) + zmax
    B = x.shape[0]
    loss = float(-(t * (z - lse)).sum() / B)
    g = (np.exp(z - lse) * t.sum(1, keepdims=True) - t) / B
    dws, dbs = [None] * nl, [None] * nl
    for l in range(nl - 1, -1, -1):
        dws[l] = g.T @ acts[l]
        dbs[l] = g.sum(0)
        if l > 0:
            g = (g @ ws[l].astype(np.float64)) * masks[l - 1]
    return loss, dws, dbs


def mask_flips_are_ties(ws, bs, x, gpu_acts, oracle_acts):
    """Return (n_flips, worst_margin) over all hidden layers; asserts item 1."""
    n, worst = 0, 0.0
    inp = x.astype(np.float64)
    for l, (ga, oa) in enumerate(zip(gpu_acts, oracle_acts)):
        flips = np.argwhere((ga > 0) != (oa > 0))
        if len(flips):
            w = ws[l].astype(np.float64)
            z = inp @ w.T + bs[l]
            scale = np.abs(inp) @ np.abs(w).T + np.abs(bs[l])
            margin = np.abs(z[flips[:, 0], flips[:, 1]]) / scale[flips[:, 0], flips[:, 1]]
            worst = max(worst, float(margin.max()))
            assert margin.max() <= FLIP_MARGIN, (l, flips[:8], margin[:8])
            n += len(flips)
        inp = ga.astype(np.float64)
    return n, worst


def check_step(ws, bs, x, t, lr, gpu_acts, gpu_grads, gpu_params, oracle_out, oracle_acts,
               tol=1e-4):
    """Items 1-3 above for one step.  oracle_out is oracle.mlp_step's tuple."""
    oloss, ow, ob, odw, odb, _ = oracle_out
    flips, _ = mask_flips_are_ties(ws, bs, x, gpu_acts, oracle_acts)
    gw, gb = gpu_grads
    pw, pb = gpu_params
    nl = len(ws)
    if flips == 0:
        for l in range(nl):
            assert normrel(gw[l], odw[l]) <= tol, ("dW vs oracle", l, normrel(gw[l], odw[l]))
            assert normrel(gb[l], odb[l]) <= tol, ("db vs oracle", l, normrel(gb[l], odb[l]))
            assert normrel(pw[l] - ws[l], ow[l] - ws[l]) <= tol, ("W delta vs oracle", l)
            assert normrel(pb[l] - bs[l], ob[l] - bs[l]) <= tol, ("b delta vs oracle", l)
    masks = [(a > 0).astype(np.float64) for a in gpu_acts]
    _, fdw, fdb = f64_step(ws, bs, x, t, masks)
    for l in range(nl):
        assert normrel(gw[l], fdw[l]) <= tol, ("dW vs float64", l, normrel(gw[l], fdw[l]))
        assert normrel(gb[l], fdb[l]) <= tol, ("db vs float64", l, normrel(gb[l], fdb[l]))
        assert normrel(pw[l] - ws[l], -lr * fdw[l]) <= tol, ("W delta vs float64", l)
    return flips
