"""ferrograd_b200: a B200 (sm_100a) execution backend for ferrograd's MLP
training path.  The compute lives in ``libferro_cuda.so`` (CUDA kernels and a
C ABI, ``include/ferro_cuda.h``); this package is the host-side binding.
"""
from ._lib import FerroError, lib  # noqa: F401
from .device import Buffer, CudaDevice, KernelArg, Program  # noqa: F401
from .mlp import Communicator, InitRng, MlpTrainer, linear_init, mlp_init, peer_layout  # noqa: F401

__all__ = ["FerroError", "lib", "Buffer", "CudaDevice", "KernelArg", "Program", "Communicator",
           "InitRng", "MlpTrainer", "linear_init", "mlp_init", "peer_layout"]
