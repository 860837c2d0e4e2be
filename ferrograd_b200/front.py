"""The lazy Tensor front end of ferrograd on the B200 backend.

``Tensor``, ``Linear`` and ``Sgd`` mirror the reference crate's API
(src/tensor.rs, src/nn.rs, src/optim.rs): operations build a lazy graph,
``realize``/``to_vec``/``numpy`` schedule it into kernels with the reference's
materialisation rules, and each kernel runs on the GPU through
``libferro_cuda.so`` -- contractions on the tcgen05 3xTF32 GEMM, large f32
reductions on the HBM reduction kernels, everything else as CUDA C rendered
with the reference's op semantics and compiled by NVRTC.  ``FG_FRONT_EXACT=1``
renders every kernel, reproducing the reference's arithmetic order.

The implementation is C++ (``csrc/front``, built into ``libferro_front.so``);
this module is its Python binding plus a few conveniences.
"""
from __future__ import annotations

import os

import numpy as np

from . import _lib  # noqa: F401  (loads libferro_cuda.so first)

try:
    from . import _front
except ImportError as e:  # pragma: no cover - build problem, fail loudly
    raise ImportError(
        "ferrograd_b200._front is not built; run python -m ferrograd_b200.build") from e

Tensor = _front.Tensor
Linear = _front.Linear
Sgd = _front.Sgd
UOp = _front.UOp
reset_init_seed = _front.reset_init_seed
init_seed = _front.init_seed
set_device = _front.set_device
synchronize = _front.synchronize
stream = _front.stream
schedule = _front.schedule
schedule_uops = _front.schedule_uops
stats = _front.stats
reset_stats = _front.reset_stats
last_source = _front.last_source
exact_mode = _front.exact_mode
interner_size = _front.interner_size

__all__ = ["Tensor", "Linear", "Sgd", "UOp", "Mlp", "reset_init_seed", "init_seed",
           "set_device", "synchronize", "stream", "schedule", "schedule_uops", "stats", "reset_stats",
           "last_source", "exact_mode", "interner_size", "tensor", "one_hot"]


def tensor(data, dtype=None) -> "Tensor":
    """Tensor::new from any array-like (float32 unless an int32/bool array)."""
    arr = np.asarray(data)
    if dtype is not None:
        arr = arr.astype(dtype)
    elif arr.dtype not in (np.float32, np.int32, np.bool_):
        arr = arr.astype(np.float32)
    return Tensor.new(np.ascontiguousarray(arr))


def one_hot(labels, num_classes: int) -> "Tensor":
    """Dense one-hot targets as examples/mnist.rs builds them."""
    labels = np.asarray(labels)
    out = np.zeros((labels.size, num_classes), np.float32)
    out[np.arange(labels.size), labels] = 1.0
    return Tensor.new(out)


class Mlp:
    """Linear layers with ReLU between them: the model of examples/mnist.rs,
    generalised to any widths (``dims = (in, hidden..., out)``)."""

    def __init__(self, dims):
        self.dims = tuple(int(d) for d in dims)
        self.layers = [Linear(self.dims[i], self.dims[i + 1])
                       for i in range(len(self.dims) - 1)]

    def forward(self, x: "Tensor") -> "Tensor":
        h = x
        for i, layer in enumerate(self.layers):
            h = layer.forward(h)
            if i + 1 < len(self.layers):
                h = h.relu()
        return h

    __call__ = forward

    def parameters(self):
        return [p for layer in self.layers for p in layer.parameters()]


def train_step(model: Mlp, optim: "Sgd", x: "Tensor", t: "Tensor") -> float:
    """One step of the reference training loop (examples/mnist.rs:90-97):
    forward, cross_entropy, zero_grad, backward, step, loss.to_vec()."""
    logits = model.forward(x)
    loss = logits.cross_entropy(t)
    optim.zero_grad()
    loss.backward()
    optim.step()
    return loss.to_vec()[0]


def debug_level() -> int:
    return int(os.environ.get("DEBUG", "0") or 0)
