"""Python entry points for the fused building blocks, on torch CUDA tensors.

torch only provides device memory and the current stream here; every call
lands in ``libferro_cuda.so``.  Each function names the reference computation
it implements.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import call


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream: Optional[int]) -> int:
    return torch.cuda.current_stream().cuda_stream if stream is None else stream


def _check_f32(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is None:
            continue
        if not (t.is_cuda and t.is_contiguous()):
            raise ValueError("expected a contiguous CUDA tensor")


def ew_fma_relu_scale(a, b, c, scale: float = 0.5, out=None, stream=None) -> torch.Tensor:
    """relu(a*b + c) * scale (Tensor::mul/add/relu, src/tensor.rs:471-491,519-531)."""
    _check_f32(a, b, c)
    out = torch.empty_like(a) if out is None else out
    call("fg_ew_fma_relu_scale", _p(a), _p(b), _p(c), _p(out), a.numel(), ctypes.c_float(scale),
         _stream(stream))
    return out


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return _lib.F32
    if t.dtype == torch.int32:
        return _lib.I32
    raise ValueError(f"unsupported dtype {t.dtype}")


def reduce_rows(x: torch.Tensor, op: int = _lib.REDUCE_SUM, stream=None) -> torch.Tensor:
    """Tensor::sum / Tensor::max over the last axis of a 2-D tensor (keepdim)."""
    _check_f32(x)
    rows, cols = x.shape
    out = torch.empty((rows, 1), dtype=x.dtype, device=x.device)
    call("fg_reduce_rows", _dtype_code(x), op, _p(x), _p(out), rows, cols, _stream(stream))
    return out


def reduce_cols(x: torch.Tensor, op: int = _lib.REDUCE_SUM, stream=None) -> torch.Tensor:
    """Tensor::sum / Tensor::max over axis 0 of a 2-D tensor (keepdim)."""
    _check_f32(x)
    rows, cols = x.shape
    out = torch.empty((1, cols), dtype=x.dtype, device=x.device)
    call("fg_reduce_cols", _dtype_code(x), op, _p(x), _p(out), rows, cols, _stream(stream))
    return out


def xent_fwd_bwd(logits: torch.Tensor, targets: torch.Tensor, need_grad: bool = True,
                 grad_scale: float = 1.0, stream=None):
    """Tensor::cross_entropy forward and d loss / d logits (src/tensor.rs:738-752)."""
    _check_f32(logits, targets)
    rows, cols = logits.shape
    loss = torch.empty(1, dtype=torch.float32, device=logits.device)
    dx = torch.empty_like(logits) if need_grad else None
    call("fg_xent_fwd_bwd", _p(logits), _p(targets), rows, cols, _p(loss), _p(dx),
         ctypes.c_float(grad_scale), _stream(stream))
    return loss, dx


def sgd_(param: torch.Tensor, grad: torch.Tensor, lr: float, param_lo=None, stream=None):
    """In-place Sgd::step update p <- p + (-(g*lr)) (src/optim.rs:60-71)."""
    _check_f32(param, grad)
    call("fg_sgd", _p(param), _p(grad), param.numel(), ctypes.c_float(lr), _p(param_lo),
         _stream(stream))
    return param


def split_lo(x: torch.Tensor, stream=None) -> torch.Tensor:
    """TF32 residual x - trunc_tf32(x) used by the 3xTF32 GEMM."""
    _check_f32(x)
    lo = torch.empty_like(x)
    call("fg_split_lo", _p(x), _p(lo), x.numel(), _stream(stream))
    return lo


def gemm(a, b, *, a_lo=None, b_lo=None, a_mn_major=False, b_mn_major=False, one_pass=False,
         epilogue=_lib.EPI_NONE, bias=None, mask=None, out=None, out_lo=None, stream=None):
    """C[m,n] = sum_k A(m,k) B(n,k) on the tcgen05 tensor cores (3xTF32).

    ``a`` is [M, K] (or [K, M] with ``a_mn_major``), ``b`` is [N, K] (or
    [K, N] with ``b_mn_major``).  Residuals are computed when not given.
    """
    _check_f32(a, b)
    M = a.shape[1] if a_mn_major else a.shape[0]
    K = a.shape[0] if a_mn_major else a.shape[1]
    N = b.shape[1] if b_mn_major else b.shape[0]
    if not one_pass:
        a_lo = split_lo(a, stream) if a_lo is None else a_lo
        b_lo = split_lo(b, stream) if b_lo is None else b_lo
    out = torch.empty((M, N), dtype=torch.float32, device=a.device) if out is None else out
    flags = ((_lib.GEMM_A_MN_MAJOR if a_mn_major else 0) | (_lib.GEMM_B_MN_MAJOR if b_mn_major else 0)
             | (_lib.GEMM_1XTF32 if one_pass else 0))
    call("fg_gemm_3xtf32", M, N, K, _p(a), _p(a_lo), a.stride(0), _p(b), _p(b_lo), b.stride(0),
         _p(out), _p(out_lo), out.stride(0), flags, epilogue, _p(bias), _p(mask),
         0 if mask is None else mask.stride(0), _stream(stream))
    return out


def check_device_error() -> None:
    call("fg_check_device_error")


def kernel_launches() -> int:
    return int(_lib.lib().fg_kernel_launches())
