"""Random Tensor-API graphs on the host test device (TEST INFRASTRUCTURE; run
in a subprocess by tests/test_hostdev_front.py).

Each graph is drawn from the ops the training path uses -- broadcast add and
mul, neg, relu, the fused chain relu(x*x+x), exp, log, reciprocal, sqrt,
sum / max over random axis sets, permute, reshape, expand, narrow,
contiguous, matmul, log_softmax, cross_entropy against one-hot targets --
over f32 leaves of ragged shapes (0 to 257 per axis, up to rank 3; a max
over an empty axis is -inf, the reference's identity).  Forward graphs are
realized in exact mode (every kernel rendered in the reference's order) and
in the default mode (routed GEMMs and reductions, warp/block reductions,
128-bit accesses, the fused cross-entropy) and both are held to float64
numpy within 1e-4 of the magnitude of the terms that make each element (a
sum's terms, not its possibly cancelled result).  Gradient graphs (loss =
sum of the graph times a random weight, backward to every leaf) compare the
default mode's gradients with exact mode's at the same tolerance, NaN where
the other mode has NaN (sqrt of 0 and the like); a gradient the reference
does not define (Shrink, src/gradient.rs:203) must raise in both modes.
Integer graphs (i32 leaves in -1000..1000; add, mul, neg, relu, sum, max and
the movement ops) must give the int64 result exactly in both modes.

argv: seed count fwd|grad|i32 output.npz
"""
import os
import sys

import numpy as np

_BUILD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")
os.environ.setdefault("FG_HOSTDEV_CACHE", os.path.join(_BUILD, "kcache"))
os.makedirs(os.environ["FG_HOSTDEV_CACHE"], exist_ok=True)
sys.path.insert(0, _BUILD)
import _front as F  # noqa: E402

SIZES = [0, 1, 3, 4, 7, 8, 16, 33, 40, 64, 100, 128, 257]
OPS = ["add", "mul", "neg", "relu", "sum", "max", "permute", "reshape", "expand", "narrow",
       "contig", "matmul", "exp", "log", "recip", "sqrt", "chain", "logsm", "xent"]


class Node:
    """A graph: build(env) makes its Tensor, ref is its float64 value and
    mag a bound on the magnitude of the terms that make each element (the
    graph over absolute values: a sum's terms, not its cancelled result), the
    scale its rounding error is measured against."""

    def __init__(self, build, ref, mag=None):
        self.build, self.ref = build, ref
        self.mag = np.abs(ref) if mag is None else mag

    @property
    def shape(self):
        return self.ref.shape


I32_OPS = ["add", "mul", "neg", "relu", "sum", "max", "permute", "reshape", "expand", "narrow",
           "contig"]


def leaf(rng, shape, i32=False):
    if i32:
        a = rng.integers(-1000, 1001, shape).astype(np.int32)
        return Node(lambda env, a=a: env.leaf(a), a.astype(np.int64))
    a = rng.standard_normal(shape).astype(np.float32)
    return Node(lambda env, a=a: env.leaf(a), a.astype(np.float64))


def rand_graph(rng, depth=0, i32=False):
    """A random graph over f32 leaves, or over i32 leaves with the integer
    ops (its float64 / int64 value alongside)."""
    if depth > 3 or rng.random() < 0.25:
        shape = tuple(int(rng.choice(SIZES)) for _ in range(int(rng.integers(1, 4))))
        if np.prod(shape) > 200000:
            shape = shape[:1]
        return leaf(rng, shape, i32)
    op = rng.choice(I32_OPS if i32 else OPS)
    x = rand_graph(rng, depth + 1, i32)
    s = x.shape
    if op in ("add", "mul"):
        y = leaf(rng, s if rng.random() < 0.5 else
                 tuple(d if rng.random() < 0.5 else 1 for d in s), i32)
        if op == "add":
            return Node(lambda env, x=x, y=y: x.build(env).add(y.build(env)), x.ref + y.ref,
                        x.mag + y.mag)
        return Node(lambda env, x=x, y=y: x.build(env).mul(y.build(env)), x.ref * y.ref,
                    x.mag * y.mag)
    if op == "neg":
        return Node(lambda env, x=x: x.build(env).neg(), -x.ref, x.mag)
    if op == "relu":
        return Node(lambda env, x=x: x.build(env).relu(),
                    np.where(x.ref > 0, x.ref, np.zeros_like(x.ref)), x.mag)
    if op == "chain":
        return Node(lambda env, x=x: x.build(env).mul(x.build(env)).add(x.build(env)).relu(),
                    np.maximum(x.ref * x.ref + x.ref, 0.0), x.mag * x.mag + x.mag)
    if op in ("sum", "max"):
        axes = sorted(rng.choice(len(s), int(rng.integers(1, len(s) + 1)), replace=False).tolist())
        if op == "sum":
            return Node(lambda env, x=x, a=axes: x.build(env).sum(a),
                        x.ref.sum(axis=tuple(axes), keepdims=True),
                        x.mag.sum(axis=tuple(axes), keepdims=True))
        ident = -np.inf if x.ref.dtype.kind == "f" else -(2**31)  # max over nothing
        return Node(lambda env, x=x, a=axes: x.build(env).max(a),
                    x.ref.max(axis=tuple(axes), keepdims=True, initial=ident),
                    x.mag.max(axis=tuple(axes), keepdims=True, initial=0))
    if op == "permute":
        order = rng.permutation(len(s)).tolist()
        return Node(lambda env, x=x, o=order: x.build(env).permute(o), np.transpose(x.ref, order),
                    np.transpose(x.mag, order))
    if op == "reshape":
        n = int(np.prod(s))
        if n == 0:
            return Node(lambda env, x=x: x.build(env).reshape([0, 3]), x.ref.reshape(0, 3),
                        x.mag.reshape(0, 3))
        d0 = int(rng.choice([d for d in range(1, n + 1) if n % d == 0]))
        return Node(lambda env, x=x, sh=[d0, n // d0]: x.build(env).reshape(sh),
                    x.ref.reshape(d0, n // d0), x.mag.reshape(d0, n // d0))
    if op == "expand":
        shape = tuple(int(rng.choice([2, 5, 32])) if d == 1 else d for d in s)
        if 1 not in s or np.prod(shape) > 300000:
            return x
        return Node(lambda env, x=x, sh=list(shape): x.build(env).expand(sh),
                    np.broadcast_to(x.ref, shape), np.broadcast_to(x.mag, shape))
    if op == "narrow":
        dim = int(rng.integers(0, len(s)))
        if s[dim] < 2:
            return x
        start = int(rng.integers(0, s[dim] - 1))
        ln = int(rng.integers(1, s[dim] - start + 1))
        sl = [slice(None)] * len(s)
        sl[dim] = slice(start, start + ln)
        return Node(lambda env, x=x, a=(dim, start, ln): x.build(env).narrow(*a), x.ref[tuple(sl)],
                    x.mag[tuple(sl)])
    if op == "contig":
        return Node(lambda env, x=x: x.build(env).contiguous(), x.ref, x.mag)
    if op == "matmul":
        if len(s) != 2:
            return x
        w = leaf(rng, (s[1], int(rng.choice([1, 5, 16, 40, 128]))))
        return Node(lambda env, x=x, w=w: x.build(env).matmul(w.build(env)), x.ref @ w.ref,
                    x.mag @ w.mag)
    if op == "logsm":
        axis = int(rng.integers(0, len(s)))
        m = x.ref.max(axis=axis, keepdims=True, initial=-np.inf)
        m = np.where(np.isfinite(m), m, 0.0)
        lse = np.log(np.exp(x.ref - m).sum(axis=axis, keepdims=True)) + m
        return Node(lambda env, x=x, a=axis: x.build(env).log_softmax(a), x.ref - lse,
                    np.abs(x.ref - lse) + 2 * x.mag.max(axis=axis, keepdims=True, initial=0))
    if op == "xent":
        if len(s) != 2 or s[0] == 0 or s[1] == 0:
            return x
        t = np.zeros(s, np.float32)
        t[np.arange(s[0]), rng.integers(0, s[1], s[0])] = 1
        m = x.ref.max(axis=1, keepdims=True)
        logp = x.ref - (np.log(np.exp(x.ref - m).sum(axis=1, keepdims=True)) + m)
        loss = -(t * logp).sum(keepdims=True) / s[0]
        mag = (np.abs(logp) + 2 * x.mag.max(axis=1, keepdims=True)).max(keepdims=True)
        return Node(lambda env, x=x, t=t: x.build(env).cross_entropy(F.Tensor.new(t)),
                    loss.reshape(1, 1), mag.reshape(1, 1))
    sq = lambda env, x: x.build(env).mul(x.build(env))  # noqa: E731
    if op == "exp":
        return Node(lambda env, x=x: x.build(env).mul(F.Tensor.scalar(0.25)).exp(),
                    np.exp(x.ref * 0.25), np.exp(x.mag * 0.25) * (1.0 + 0.25 * x.mag))
    if op == "log":
        return Node(lambda env, x=x: sq(env, x).add(F.Tensor.scalar(1.0)).log(),
                    np.log(x.ref * x.ref + 1.0), np.log(x.mag * x.mag + 1.0) + x.mag * x.mag)
    if op == "recip":
        return Node(lambda env, x=x: sq(env, x).add(F.Tensor.scalar(1.0)).reciprocal(),
                    1.0 / (x.ref * x.ref + 1.0), 1.0 + x.mag * x.mag)
    return Node(lambda env, x=x: sq(env, x).sqrt(), np.abs(x.ref), x.mag)  # sqrt


class Env:
    """One Tensor per leaf array per realization."""

    def __init__(self, grad):
        self.grad, self.tensors = grad, {}

    def leaf(self, a):
        if id(a) not in self.tensors:
            t = F.Tensor.new(np.ascontiguousarray(a))
            self.tensors[id(a)] = t.with_requires_grad(True) if self.grad else t
        return self.tensors[id(a)]


def scale_err(got, ref, mag=None):
    """Largest |got - ref| over the scale max(mag) (max |ref| by default);
    NaN must sit where ref has NaN."""
    if ref.size == 0:
        return 0.0
    both_nan = np.isnan(got) & np.isnan(ref)
    if np.any(np.isnan(got) != np.isnan(ref)):
        return float("inf")
    ref = np.where(both_nan, 0.0, ref)
    got = np.where(both_nan, 0.0, got.astype(np.float64))
    same = got == ref  # equal infinities too (a max over an empty axis is -inf)
    if np.any(~np.isfinite(ref) & ~same):
        return float("inf")
    diff = np.where(same, 0.0, np.abs(got - np.where(same, 0.0, ref)))
    scale = np.abs(ref) if mag is None else np.where(both_nan, 0.0, mag)
    scale = np.where(np.isfinite(scale), scale, 0.0)
    return float(np.max(diff) / max(np.max(scale), 1e-3))


def realize(node, mode, grad, wv):
    os.environ["FG_FRONT_EXACT"] = mode
    env = Env(grad)
    t = node.build(env)
    if not grad:
        return [t.numpy().reshape(node.shape)]
    nd = len(node.shape)
    t.mul(F.Tensor.new(wv)).sum(list(range(nd))).backward()
    grads = [env.tensors[k].grad() for k in sorted(env.tensors)]
    return [None if g is None else g.numpy() for g in grads]


def fits_i32(node):
    return node.ref.size == 0 or np.max(np.abs(node.ref)) <= 2**31


def main(seed, count, kind, dst):
    grad, i32 = kind == "grad", kind == "i32"
    failures, checked, undefined = [], 0, 0
    for i in range(count):
        rng = np.random.default_rng(seed * 100000 + i)
        node = rand_graph(rng, i32=i32)
        if i32 and not fits_i32(node):
            continue  # the int64 reference left the i32 range (a product of sums)
        wv = rng.standard_normal(node.shape).astype(np.float32)
        outs, errors = {}, {}
        for mode in ("1", "0"):
            try:
                outs[mode] = realize(node, mode, grad, wv)
            except RuntimeError as e:
                errors[mode] = str(e)
        if errors:
            if (grad and len(errors) == 2 and all("gradient not implemented" in m
                                                  for m in errors.values())):
                undefined += 1
                continue
            failures.append(f"{i}: {errors}")
            continue
        checked += 1
        if grad:
            for j, (a, b) in enumerate(zip(outs["1"], outs["0"])):
                if a is None or b is None:
                    if (a is None) != (b is None):
                        failures.append(f"{i}: leaf {j}: a gradient in one mode only")
                    continue
                e = scale_err(b, a.astype(np.float64))
                if not e <= 1e-4:
                    failures.append(f"{i}: leaf {j} {a.shape}: default vs exact {e:.2e}")
        elif i32:
            for mode in ("1", "0"):
                got = outs[mode][0]
                if got.dtype != np.int32 or not np.array_equal(got.astype(np.int64), node.ref):
                    failures.append(f"{i}: mode {mode} {node.shape}: i32 result differs")
        else:
            for mode in ("1", "0"):
                e = scale_err(outs[mode][0], node.ref, node.mag)
                if not e <= 1e-4:
                    failures.append(f"{i}: mode {mode} {node.shape}: vs float64 {e:.2e}")
    np.savez(dst, failures=np.array(failures, dtype=str), checked=np.array(checked),
             undefined=np.array(undefined))


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4])
