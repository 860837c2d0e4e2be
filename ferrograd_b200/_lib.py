"""ctypes binding of ``libferro_cuda.so`` (declared in ``include/ferro_cuda.h``).

The library is the product: every call in this package goes through it.
Loading fails loudly when it is missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libferro_cuda.so")

FG_OK = 0
ERR_NAMES = {1: "FG_ERR_INVALID", 2: "FG_ERR_CUDA", 3: "FG_ERR_COMPILE", 4: "FG_ERR_NCCL",
             5: "FG_ERR_DEVICE", 6: "FG_ERR_UNSUPPORTED"}

F32, I32, BOOL = 0, 1, 2
REDUCE_SUM, REDUCE_MAX = 0, 1
EPI_NONE, EPI_BIAS, EPI_BIAS_RELU, EPI_RELU_MASK = 0, 1, 2, 3
GEMM_A_MN_MAJOR, GEMM_B_MN_MAJOR, GEMM_1XTF32 = 1, 2, 4
ARG_BUFFER, ARG_I32, ARG_F32, ARG_BOOL = 0, 1, 2, 3
UNIQUE_ID_BYTES = 128
PEER_HANDLE_BYTES = 96


class FerroError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class _ArgValue(ctypes.Union):
    _fields_ = [("buffer", ctypes.c_void_p), ("i32", ctypes.c_int32), ("f32", ctypes.c_float),
                ("b", ctypes.c_uint8)]


class KernelArgC(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("v", _ArgValue)]


# (name, restype, argtypes) for every exported entry point in include/ferro_cuda.h.
_vp, _sz, _i, _f = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
_pp = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = [
    ("fg_last_error", ctypes.c_char_p, []),
    ("fg_device_open", _i, [_i, _pp]),
    ("fg_device_close", _i, [_vp]),
    ("fg_device_stream", _i, [_vp, _pp]),
    ("fg_device_sync", _i, [_vp]),
    ("fg_event_create", _i, [_vp, _pp]),
    ("fg_event_record", _i, [_vp, _vp]),
    ("fg_event_elapsed_ms", _i, [_vp, _vp, ctypes.POINTER(ctypes.c_float)]),
    ("fg_event_destroy", _i, [_vp]),
    ("fg_alloc", _i, [_vp, _i, _sz, _pp]),
    ("fg_free", _i, [_vp]),
    ("fg_buffer_info", _i, [_vp, _pp, ctypes.POINTER(_i), ctypes.POINTER(_sz)]),
    ("fg_copy_h2d", _i, [_vp, _vp, _sz]),
    ("fg_copy_d2h", _i, [_vp, _vp, _sz]),
    ("fg_compile", _i, [_vp, ctypes.c_char_p, ctypes.c_char_p, _i, ctypes.POINTER(ctypes.c_uint32),
                        ctypes.POINTER(ctypes.c_uint32), _pp]),
    ("fg_program_free", _i, [_vp]),
    ("fg_execute", _i, [_vp, ctypes.POINTER(KernelArgC), _i]),
    ("fg_kaiming_normal", _i, [_vp, _sz, _sz, ctypes.POINTER(ctypes.c_uint64)]),
    ("fg_ew_fma_relu_scale", _i, [_vp, _vp, _vp, _vp, _sz, _f, _vp]),
    ("fg_reduce_rows", _i, [_i, _i, _vp, _vp, _sz, _sz, _vp]),
    ("fg_reduce_cols", _i, [_i, _i, _vp, _vp, _sz, _sz, _vp]),
    ("fg_xent_fwd_bwd", _i, [_vp, _vp, _sz, _sz, _vp, _vp, _f, _vp]),
    ("fg_xent_fwd_bwd_noalloc", _i, [_vp, _vp, _sz, _sz, _vp, _vp, _f, _vp]),
    ("fg_sgd", _i, [_vp, _vp, _sz, _f, _vp, _vp]),
    ("fg_split_lo", _i, [_vp, _vp, _sz, _vp]),
    ("fg_u8_to_f32_div", _i, [_vp, _vp, _sz, _f, _vp]),
    ("fg_one_hot_u8", _i, [_vp, _vp, _sz, _i, _vp]),
    ("fg_gemm_3xtf32", _i, [_i, _i, _i, _vp, _vp, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp, _vp,
                            _i, _vp]),
    ("fg_mlp_create", _i, [_vp, _i, ctypes.POINTER(_i), _i, _f, _pp]),
    ("fg_mlp_destroy", _i, [_vp]),
    ("fg_mlp_set_params", _i, [_vp, _i, _vp, _vp]),
    ("fg_mlp_get_params", _i, [_vp, _i, _vp, _vp]),
    ("fg_mlp_get_grads", _i, [_vp, _i, _vp, _vp]),
    ("fg_mlp_attach_comm", _i, [_vp, _vp]),
    ("fg_mlp_input_slots", _i, [_vp, _pp, _pp]),
    ("fg_mlp_step", _i, [_vp, _vp]),
    ("fg_mlp_step_host", _i, [_vp, _vp, _vp, _vp]),
    ("fg_mlp_step_host_next", _i, [_vp, _vp, _vp, _vp, _vp, _vp]),
    ("fg_mlp_use_graph", _i, [_vp, _i]),
    ("fg_mlp_get_logits", _i, [_vp, _vp]),
    ("fg_mlp_get_activations", _i, [_vp, _i, _vp]),
    ("fg_mlp_launch_count", _i, [_vp, ctypes.POINTER(_i)]),
    ("fg_mlp_enable_gemm_timing", _i, [_vp, _i]),
    ("fg_mlp_gemm_times", _i, [_vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double),
                               _i, ctypes.POINTER(_i)]),
    ("fg_mlp_comm_times", _i, [_vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double),
                               _i, ctypes.POINTER(_i)]),
    ("fg_mlp_peer_prepare", _i, [_vp, _i, _i, _i, ctypes.c_char_p]),
    ("fg_mlp_peer_connect", _i, [_vp, ctypes.c_char_p]),
    ("fg_mlp_peer_disconnect", _i, [_vp]),
    ("fg_peer_layout", _i, [_i, ctypes.POINTER(_i), _i, _i, ctypes.POINTER(_sz), ctypes.POINTER(_sz),
                            ctypes.POINTER(_sz), _i, ctypes.POINTER(_i)]),
    ("fg_peer_layout_offsets", _i, [_i, ctypes.POINTER(_i), _i, _i, ctypes.POINTER(_sz),
                                    ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    ("fg_peer_reduce_sgd_local", _i, [_vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _f, ctypes.c_longlong,
                                      _vp, ctypes.c_uint, _i, _vp]),
    ("fg_comm_unique_id", _i, [ctypes.c_char_p]),
    ("fg_comm_init", _i, [_i, _i, ctypes.c_char_p, _i, _pp]),
    ("fg_comm_destroy", _i, [_vp]),
    ("fg_comm_abort", _i, [_vp]),
    ("fg_allreduce_mean_f32", _i, [_vp, _vp, _sz, _vp]),
    ("fg_check_device_error", _i, []),
    ("fg_kernel_launches", ctypes.c_uint64, []),
    ("fg_kernel_arch", _i, [ctypes.POINTER(_i), ctypes.POINTER(_i)]),
]

_lib = None


def lib() -> ctypes.CDLL:
    """Load the library (RTLD_GLOBAL not needed) and declare every signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FerroError(2, f"{LIB_PATH} is missing: build it with `python -m ferrograd_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(code: int) -> None:
    if code != FG_OK:
        raise FerroError(code, lib().fg_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
