"""The MLP training path of ferrograd (examples/mnist.rs) on the B200 backend.

* :class:`InitRng` / :func:`linear_init` -- ``Linear::new`` (src/nn.rs:77-85):
  Kaiming-normal weight from the reference's thread-local LCG (seed 42,
  continuing across layers), zero bias.  Runs in the C library.
* :class:`MlpTrainer` -- one ``forward -> cross_entropy -> zero_grad ->
  backward -> Sgd::step -> loss.to_vec()`` step per call, planned once and
  replayed (optionally as a CUDA graph), data parallel when given a
  :class:`Communicator` or after :meth:`MlpTrainer.shard_over_peers`.
* :func:`peer_layout` -- the chunks of the peer-sharded gradient exchange.
"""
from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import call
from .device import CudaDevice


class InitRng:
    """The reference's init seed (``INIT_SEED``, src/nn.rs:12-14), starting at 42."""

    def __init__(self, seed: int = 42):
        self.state = ctypes.c_uint64(seed)

    def kaiming_normal(self, shape: Sequence[int], fan_in: int) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), dtype=np.float32)
        call("fg_kaiming_normal", out.ctypes.data, out.size, int(fan_in), ctypes.byref(self.state))
        return out.reshape(tuple(shape))


def linear_init(in_features: int, out_features: int, rng: InitRng) -> Tuple[np.ndarray, np.ndarray]:
    """``Linear::new(in, out)``: weight [out, in] Kaiming-normal, bias zeros."""
    w = rng.kaiming_normal((out_features, in_features), in_features)
    return w, np.zeros(out_features, dtype=np.float32)


def mlp_init(dims: Sequence[int], rng: Optional[InitRng] = None):
    """Parameters of ``Linear(dims[0], dims[1]) ... Linear(dims[-2], dims[-1])``."""
    rng = InitRng() if rng is None else rng
    ws, bs = [], []
    for i in range(len(dims) - 1):
        w, b = linear_init(dims[i], dims[i + 1], rng)
        ws.append(w)
        bs.append(b)
    return ws, bs


class Communicator:
    """NCCL communicator for the data-parallel step (no reference counterpart)."""

    def __init__(self, rank: int, nranks: int, unique_id: bytes, timeout_ms: int = 60000):
        h = ctypes.c_void_p()
        call("fg_comm_init", int(rank), int(nranks), bytes(unique_id), int(timeout_ms), ctypes.byref(h))
        self._h = h.value
        self.rank, self.nranks = rank, nranks

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(_lib.UNIQUE_ID_BYTES)
        call("fg_comm_unique_id", buf)
        return buf.raw

    @property
    def handle(self) -> int:
        """The fg_comm pointer, for the front end (``Sgd.set_comm``,
        ``Tensor.all_reduce_mean``)."""
        if not self._h:
            raise RuntimeError("communicator is closed")
        return int(self._h)

    def allreduce_mean_(self, ptr: int, count: int, stream: int) -> None:
        call("fg_allreduce_mean_f32", self._h, ptr, int(count), stream)

    def close(self) -> None:
        if self._h:
            call("fg_comm_destroy", self._h)
            self._h = None


class MlpTrainer:
    """Owns the device parameters and runs training steps through the C ABI."""

    def __init__(self, device: CudaDevice, dims: Sequence[int], batch: int, lr: float,
                 weights: Sequence[np.ndarray], biases: Sequence[np.ndarray],
                 comm: Optional[Communicator] = None, use_graph: bool = False):
        self.device = device
        self.dims = list(dims)
        self.batch = int(batch)
        self.lr = float(lr)
        self.n_layers = len(dims) - 1
        d = (ctypes.c_int * len(dims))(*[int(x) for x in dims])
        h = ctypes.c_void_p()
        call("fg_mlp_create", device.handle, self.n_layers, d, self.batch, ctypes.c_float(lr),
             ctypes.byref(h))
        self._h = h.value
        for l, (w, b) in enumerate(zip(weights, biases)):
            w = np.ascontiguousarray(w, dtype=np.float32)
            b = np.ascontiguousarray(b, dtype=np.float32)
            assert w.shape == (dims[l + 1], dims[l]) and b.shape == (dims[l + 1],)
            call("fg_mlp_set_params", self._h, l, w.ctypes.data, b.ctypes.data)
        self.comm = comm
        if comm is not None:
            call("fg_mlp_attach_comm", self._h, comm._h)
        call("fg_mlp_use_graph", self._h, 1 if use_graph else 0)

    def shard_over_peers(self, rank: int, world: int, all_gather: Callable[[bytes], List[bytes]],
                         barrier: Callable[[], None], chunks: int = 4) -> None:
        """Peer-sharded data parallelism instead of an NCCL communicator: the
        gradients move between the ranks' GPUs with the copy engines, each rank
        reduces and updates its shard of the parameters, and the updated shards
        are copied back to every rank (``fg_mlp_peer_prepare`` / ``_connect``).
        ``all_gather(handle)`` returns every rank's handle in rank order;
        ``barrier()`` is a host barrier over the same ranks (used at close)."""
        buf = ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
        call("fg_mlp_peer_prepare", self._h, int(rank), int(world), int(chunks), buf)
        handles = [bytes(h) for h in all_gather(buf.raw)]
        if len(handles) != world or any(len(h) != _lib.PEER_HANDLE_BYTES for h in handles):
            raise ValueError("shard_over_peers: expected one handle per rank")
        call("fg_mlp_peer_connect", self._h, b"".join(handles))
        self._peer_barrier = barrier

    def close(self) -> None:
        if getattr(self, "_h", None):
            barrier = getattr(self, "_peer_barrier", None)
            if barrier is not None:
                # unmap the peers' regions everywhere before any region is freed
                call("fg_mlp_peer_disconnect", self._h)
                barrier()
                self._peer_barrier = None
            call("fg_mlp_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def input_slots(self) -> Tuple[int, int]:
        x = ctypes.c_void_p()
        t = ctypes.c_void_p()
        call("fg_mlp_input_slots", self._h, ctypes.byref(x), ctypes.byref(t))
        return x.value, t.value

    def step_host(self, x: np.ndarray, targets: np.ndarray) -> float:
        """Copy the batch in, run one step, return the loss (blocking)."""
        assert x.shape == (self.batch, self.dims[0]) and targets.shape == (self.batch, self.dims[-1])
        assert x.dtype == np.float32 and targets.dtype == np.float32
        loss = ctypes.c_float()
        call("fg_mlp_step_host", self._h, x.ctypes.data, targets.ctypes.data, ctypes.byref(loss))
        return float(loss.value)

    def step_host_ptr(self, x_ptr: int, t_ptr: int, loss_ptr: int) -> None:
        """Step from raw (pinned) host pointers; the loss lands in loss_ptr."""
        call("fg_mlp_step_host", self._h, x_ptr, t_ptr, loss_ptr)

    def step_host_next(self, x: np.ndarray, targets: np.ndarray, x_next: Optional[np.ndarray],
                       targets_next: Optional[np.ndarray]) -> float:
        """One step on (x, targets) while (x_next, targets_next) is uploaded
        for the next call (``fg_mlp_step_host_next``); returns the loss.  The
        next batch's arrays must stay alive and unchanged until that call."""
        for a, cols in ((x, self.dims[0]), (targets, self.dims[-1]), (x_next, self.dims[0]),
                        (targets_next, self.dims[-1])):
            if a is not None:
                assert a.shape == (self.batch, cols) and a.dtype == np.float32
                assert a.flags["C_CONTIGUOUS"]
        loss = ctypes.c_float()
        call("fg_mlp_step_host_next", self._h, x.ctypes.data, targets.ctypes.data,
             None if x_next is None else x_next.ctypes.data,
             None if targets_next is None else targets_next.ctypes.data, ctypes.byref(loss))
        return float(loss.value)

    def step_host_next_ptr(self, x_ptr: int, t_ptr: int, xn_ptr: Optional[int],
                           tn_ptr: Optional[int], loss_ptr: int) -> None:
        """``step_host_next`` from raw (pinned) host pointers."""
        call("fg_mlp_step_host_next", self._h, x_ptr, t_ptr, xn_ptr, tn_ptr, loss_ptr)

    def step(self, loss_out_ptr: Optional[int] = None) -> None:
        """Step on inputs already in the device input slots (asynchronous)."""
        call("fg_mlp_step", self._h, loss_out_ptr)

    def params(self) -> Tuple[List[np.ndarray], List[np.ndarray]]:
        ws, bs = [], []
        for l in range(self.n_layers):
            w = np.empty((self.dims[l + 1], self.dims[l]), np.float32)
            b = np.empty(self.dims[l + 1], np.float32)
            call("fg_mlp_get_params", self._h, l, w.ctypes.data, b.ctypes.data)
            ws.append(w)
            bs.append(b)
        return ws, bs

    def grads(self) -> Tuple[List[np.ndarray], List[np.ndarray]]:
        ws, bs = [], []
        for l in range(self.n_layers):
            w = np.empty((self.dims[l + 1], self.dims[l]), np.float32)
            b = np.empty(self.dims[l + 1], np.float32)
            call("fg_mlp_get_grads", self._h, l, w.ctypes.data, b.ctypes.data)
            ws.append(w)
            bs.append(b)
        return ws, bs

    def activations(self, layer: int) -> np.ndarray:
        """Output of `layer` in the last forward pass (post-ReLU, or logits)."""
        out = np.empty((self.batch, self.dims[layer + 1]), np.float32)
        call("fg_mlp_get_activations", self._h, int(layer), out.ctypes.data)
        return out

    def logits(self) -> np.ndarray:
        out = np.empty((self.batch, self.dims[-1]), np.float32)
        call("fg_mlp_get_logits", self._h, out.ctypes.data)
        return out

    def enable_gemm_timing(self, enable: bool = True) -> None:
        call("fg_mlp_enable_gemm_timing", self._h, 1 if enable else 0)

    def gemm_times(self):
        """[(ms, flops)] of the tensor-core GEMM launches of the latest step."""
        cap = 3 * self.n_layers
        ms = (ctypes.c_float * cap)()
        fl = (ctypes.c_double * cap)()
        n = ctypes.c_int()
        call("fg_mlp_gemm_times", self._h, ms, fl, cap, ctypes.byref(n))
        return [(ms[i], fl[i]) for i in range(n.value)]

    def comm_times(self):
        """[(ms, bytes)] of the gradient all-reduces of the latest step."""
        cap = self.n_layers + 1
        ms = (ctypes.c_float * cap)()
        by = (ctypes.c_double * cap)()
        n = ctypes.c_int()
        call("fg_mlp_comm_times", self._h, ms, by, cap, ctypes.byref(n))
        return [(ms[i], by[i]) for i in range(n.value)]

    @property
    def launches_per_step(self) -> int:
        n = ctypes.c_int()
        call("fg_mlp_launch_count", self._h, ctypes.byref(n))
        return n.value


def peer_layout(dims: Sequence[int], nranks: int, chunks: int = 4):
    """(region floats, [(offset, length)] of the gradient chunks in exchange
    order) of the peer-sharded data-parallel step (host-only, no GPU)."""
    d = (ctypes.c_int * len(dims))(*[int(x) for x in dims])
    region = ctypes.c_size_t()
    cap = 64
    off = (ctypes.c_size_t * cap)()
    ln = (ctypes.c_size_t * cap)()
    n = ctypes.c_int()
    call("fg_peer_layout", len(dims) - 1, d, int(nranks), int(chunks), ctypes.byref(region), off, ln,
         cap, ctypes.byref(n))
    return region.value, [(off[i], ln[i]) for i in range(min(n.value, cap))]


def peer_offsets(dims: Sequence[int], nranks: int, chunks: int = 4):
    """([dW offset], [db offset], loss-slot offset) per layer in the gradient
    area of the peer-sharded step, in floats (host-only, no GPU)."""
    nl = len(dims) - 1
    d = (ctypes.c_int * len(dims))(*[int(x) for x in dims])
    w = (ctypes.c_size_t * nl)()
    b = (ctypes.c_size_t * nl)()
    loss = ctypes.c_size_t()
    call("fg_peer_layout_offsets", nl, d, int(nranks), int(chunks), w, b, ctypes.byref(loss))
    return list(w), list(b), loss.value
