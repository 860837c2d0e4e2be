"""ctypes wrapper around ``oracle/libferro_oracle.so`` -- TEST INFRASTRUCTURE ONLY.

The oracle is a C restatement of ferrograd's clang CPU backend arithmetic for
the MLP training path (see ``ferro_oracle.c`` for the rules and the reference
file:line each one follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference legs may import this module; the
product path (``ferrograd_b200``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libferro_oracle.so")

SUM = 0
MAX = 1

_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_c_long = ctypes.c_long


def build() -> str:
    """Compile the oracle library with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    L.orc_set_threads.argtypes = [ctypes.c_int]
    L.orc_set_unroll.argtypes = [ctypes.c_int]
    L.orc_max_threads.restype = ctypes.c_int
    L.orc_kaiming_normal.argtypes = [_f32p, _c_long, _c_long, ctypes.POINTER(ctypes.c_uint64)]
    for name, p in (("orc_reduce_last_f32", _f32p), ("orc_reduce_axis0_f32", _f32p),
                    ("orc_reduce_last_i32", _i32p), ("orc_reduce_axis0_i32", _i32p)):
        getattr(L, name).argtypes = [p, _c_long, _c_long, ctypes.c_int, p]
    L.orc_ew_fma_relu_scale.argtypes = [_f32p, _f32p, _f32p, _f32p, _c_long, ctypes.c_float]
    L.orc_relu.argtypes = [_f32p, _f32p, _c_long]
    L.orc_gemm_fwd.argtypes = [_f32p, _f32p, ctypes.c_void_p, _c_long, _c_long, _c_long, _f32p]
    L.orc_gemm_dx.argtypes = [_f32p, _f32p, _c_long, _c_long, _c_long, _f32p]
    L.orc_gemm_dw.argtypes = [_f32p, _f32p, _c_long, _c_long, _c_long, _f32p]
    L.orc_log_softmax.argtypes = [_f32p, _c_long, _c_long, _f32p]
    L.orc_xent_fwd_bwd.argtypes = [_f32p, _f32p, _c_long, _c_long, ctypes.c_void_p]
    L.orc_xent_fwd_bwd.restype = ctypes.c_float
    L.orc_sgd.argtypes = [_f32p, _f32p, _c_long, ctypes.c_float]
    L.orc_mlp_step.argtypes = [ctypes.c_int, ctypes.POINTER(_c_long), _c_long, ctypes.c_float,
                               ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                               _f32p, _f32p, ctypes.POINTER(ctypes.c_void_p),
                               ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
    L.orc_mlp_step.restype = ctypes.c_float
    L.orc_mlp_step_acts.argtypes = L.orc_mlp_step.argtypes + [ctypes.POINTER(ctypes.c_void_p)]
    L.orc_mlp_step_acts.restype = ctypes.c_float
    _lib = L
    return L


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def set_unroll(on: bool) -> None:
    """The reference's OPT "unroll" pass (src/optimize/mod.rs:80-112): off
    makes every reduction sequential (process-wide; restore it after use)."""
    lib().orc_set_unroll(1 if on else 0)


def max_threads() -> int:
    return int(lib().orc_max_threads())


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


class InitRng:
    """The reference's thread-local init seed (src/nn.rs:12-14), starting at 42."""

    def __init__(self, seed: int = 42):
        self.state = ctypes.c_uint64(seed)

    def kaiming_normal(self, shape, fan_in: int) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), dtype=np.float32)
        lib().orc_kaiming_normal(out, out.size, int(fan_in), ctypes.byref(self.state))
        return out.reshape(shape)

    def linear(self, in_features: int, out_features: int):
        """Linear::new (src/nn.rs:77-85): Kaiming-normal weight, zero bias."""
        w = self.kaiming_normal((out_features, in_features), in_features)
        return w, np.zeros(out_features, dtype=np.float32)


def reduce_last(x, op):
    x = np.asarray(x)
    rows, cols = x.shape
    if x.dtype == np.int32:
        out = np.empty(rows, dtype=np.int32)
        lib().orc_reduce_last_i32(_c(x, np.int32), rows, cols, op, out)
    else:
        out = np.empty(rows, dtype=np.float32)
        lib().orc_reduce_last_f32(_c(x), rows, cols, op, out)
    return out


def reduce_axis0(x, op):
    x = np.asarray(x)
    rows, cols = x.shape
    if x.dtype == np.int32:
        out = np.empty(cols, dtype=np.int32)
        lib().orc_reduce_axis0_i32(_c(x, np.int32), rows, cols, op, out)
    else:
        out = np.empty(cols, dtype=np.float32)
        lib().orc_reduce_axis0_f32(_c(x), rows, cols, op, out)
    return out


def ew_fma_relu_scale(a, b, c, scale: float = 0.5):
    a, b, c = _c(a).ravel(), _c(b).ravel(), _c(c).ravel()
    out = np.empty_like(a)
    lib().orc_ew_fma_relu_scale(a, b, c, out, a.size, ctypes.c_float(scale))
    return out


def relu(x):
    x = _c(x)
    out = np.empty_like(x)
    lib().orc_relu(x.ravel(), out.ravel(), x.size)
    return out


def gemm_fwd(A, B, bias=None):
    """C = sum_k A[m,k] * B[n,k] (+ bias): Tensor::matmul with the rhs in [N,K] form."""
    A, B = _c(A), _c(B)
    M, K = A.shape
    N = B.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    bias_arr = None if bias is None else _c(bias)
    lib().orc_gemm_fwd(A, B, None if bias_arr is None else bias_arr.ctypes.data, M, N, K, out)
    return out


def gemm_dx(G, Bt):
    """dA[m,k] = sum_n Bt[n,k] * G[m,n]."""
    G, Bt = _c(G), _c(Bt)
    M, N = G.shape
    K = Bt.shape[1]
    out = np.empty((M, K), dtype=np.float32)
    lib().orc_gemm_dx(G, Bt, M, N, K, out)
    return out


def gemm_dw(A, G):
    """dBt[n,k] = sum_m A[m,k] * G[m,n]."""
    A, G = _c(A), _c(G)
    M, K = A.shape
    N = G.shape[1]
    out = np.empty((N, K), dtype=np.float32)
    lib().orc_gemm_dw(A, G, M, N, K, out)
    return out


def log_softmax(x):
    x = _c(x)
    B, C = x.shape
    out = np.empty_like(x)
    lib().orc_log_softmax(x, B, C, out)
    return out


def xent_fwd_bwd(x, t, need_grad: bool = True):
    x, t = _c(x), _c(t)
    B, C = x.shape
    dx = np.empty_like(x) if need_grad else None
    loss = lib().orc_xent_fwd_bwd(x, t, B, C, None if dx is None else dx.ctypes.data)
    return float(np.float32(loss)), dx


def sgd(p, g, lr: float):
    p = _c(p).copy()
    lib().orc_sgd(p.ravel(), _c(g).ravel(), p.size, ctypes.c_float(lr))
    return p


def mlp_step(weights, biases, x, t, lr: float, want_grads: bool = True, acts=None):
    """One training step; returns (loss, new_weights, new_biases, dW, db, logits).

    Inputs are not modified: parameters are copied before the in-place update.
    If `acts` is a list, it receives the hidden layers' post-ReLU activations.
    """
    nl = len(weights)
    dims = [weights[0].shape[1]] + [w.shape[0] for w in weights]
    B = x.shape[0]
    Ws = [_c(w).copy() for w in weights]
    bs = [_c(b).copy() for b in biases]
    dWs = [np.empty_like(w) for w in Ws] if want_grads else None
    dbs = [np.empty_like(b) for b in bs] if want_grads else None
    logits = np.empty((B, dims[-1]), dtype=np.float32)
    dims_c = (_c_long * (nl + 1))(*dims)
    Wp = (ctypes.c_void_p * nl)(*[w.ctypes.data for w in Ws])
    bp = (ctypes.c_void_p * nl)(*[b.ctypes.data for b in bs])
    dWp = (ctypes.c_void_p * nl)(*[w.ctypes.data for w in dWs]) if want_grads else None
    dbp = (ctypes.c_void_p * nl)(*[b.ctypes.data for b in dbs]) if want_grads else None
    hidden = [np.empty((B, dims[l + 1]), np.float32) for l in range(nl - 1)]
    ap = (ctypes.c_void_p * max(1, nl - 1))(*[h.ctypes.data for h in hidden])
    loss = lib().orc_mlp_step_acts(nl, dims_c, B, ctypes.c_float(lr), Wp, bp, _c(x), _c(t),
                                   dWp, dbp, logits.ctypes.data, ap)
    if acts is not None:
        acts.extend(hidden)
    return float(np.float32(loss)), Ws, bs, dWs, dbs, logits
