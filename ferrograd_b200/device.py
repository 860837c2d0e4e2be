"""The CUDA implementation of ferrograd's ``Device`` trait, over the C ABI.

Mirrors ``src/device.rs:275-332`` of the reference: ``allocate`` returns a
zero-initialised :class:`Buffer`, ``copy_from_host`` / ``copy_to_host`` move
raw bytes, ``compile`` turns CUDA C into a :class:`Program` (NVRTC, sm_100a
cubin), ``execute`` launches it with :class:`KernelArg` values in parameter
slot order, and ``cached_program`` / ``insert_program`` keep the program cache
the reference keys by the lowered kernel.  Errors raise
:class:`~ferrograd_b200._lib.FerroError` with the library's message (the
reference panics with the same texts, e.g. ``copy_from_host: expected 8
bytes, got 4``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any, Dict, Optional, Sequence, Union

from . import _lib
from ._lib import F32, I32, BOOL, call

DTYPE_SIZE = {F32: 4, I32: 4, BOOL: 1}


class Buffer:
    """Typed device memory (``Buffer``, src/device.rs:95-214); freed when dropped."""

    __slots__ = ("_h", "device", "dtype", "numel")

    def __init__(self, handle: int, device: "CudaDevice", dtype: int, numel: int):
        self._h = handle
        self.device = device
        self.dtype = dtype
        self.numel = numel

    @property
    def nbytes(self) -> int:
        return DTYPE_SIZE[self.dtype] * self.numel

    @property
    def ptr(self) -> int:
        p = ctypes.c_void_p()
        call("fg_buffer_info", self._h, ctypes.byref(p), None, None)
        return p.value or 0

    def __del__(self):
        if getattr(self, "_h", None):
            try:
                _lib.lib().fg_free(self._h)
            except Exception:
                pass
            self._h = None


@dataclass(frozen=True)
class KernelArg:
    """``KernelArg`` (src/device.rs:241-251): a buffer or an i32 / f32 / bool scalar."""

    kind: int
    value: Any

    @staticmethod
    def buffer(b: Buffer) -> "KernelArg":
        return KernelArg(_lib.ARG_BUFFER, b)

    @staticmethod
    def i32(v: int) -> "KernelArg":
        return KernelArg(_lib.ARG_I32, int(v))

    @staticmethod
    def f32(v: float) -> "KernelArg":
        return KernelArg(_lib.ARG_F32, float(v))

    @staticmethod
    def bool_(v: bool) -> "KernelArg":
        return KernelArg(_lib.ARG_BOOL, bool(v))


class Program:
    """A compiled kernel (``Program``, src/device.rs:258-268)."""

    def __init__(self, handle: int, name: str, num_args: int):
        self._h = handle
        self.name = name
        self.num_args = num_args

    def __del__(self):
        if getattr(self, "_h", None):
            try:
                _lib.lib().fg_program_free(self._h)
            except Exception:
                pass
            self._h = None


class Event:
    """A point on a device stream (``fg_event_*``); ``elapsed_ms(start, end)``
    waits for ``end`` and returns the device time between the two points."""

    def __init__(self, device: "CudaDevice"):
        h = ctypes.c_void_p()
        call("fg_event_create", device.handle, ctypes.byref(h))
        self._h = h.value

    def record(self, stream: Optional[int] = None) -> "Event":
        call("fg_event_record", self._h, stream)
        return self

    @staticmethod
    def elapsed_ms(start: "Event", end: "Event") -> float:
        ms = ctypes.c_float()
        call("fg_event_elapsed_ms", start._h, end._h, ctypes.byref(ms))
        return float(ms.value)

    def __del__(self):
        if getattr(self, "_h", None):
            try:
                _lib.lib().fg_event_destroy(self._h)
            except Exception:
                pass
            self._h = None


class CudaDevice:
    """``device::get(DeviceId::Cuda(ordinal))``: one per ordinal per process."""

    _open: Dict[int, "CudaDevice"] = {}

    def __new__(cls, ordinal: int = 0):
        if ordinal in cls._open:
            return cls._open[ordinal]
        self = super().__new__(cls)
        h = ctypes.c_void_p()
        call("fg_device_open", int(ordinal), ctypes.byref(h))
        self._h = h.value
        self.ordinal = ordinal
        self._programs: Dict[Any, Program] = {}
        cls._open[ordinal] = self
        return self

    def id(self) -> str:
        return f"cuda:{self.ordinal}"

    @property
    def handle(self) -> int:
        return self._h

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        call("fg_device_stream", self._h, ctypes.byref(s))
        return s.value or 0

    def synchronize(self) -> None:
        call("fg_device_sync", self._h)

    # -- Device trait ------------------------------------------------------
    def allocate(self, dtype: int, numel: int) -> Buffer:
        h = ctypes.c_void_p()
        call("fg_alloc", self._h, int(dtype), int(numel), ctypes.byref(h))
        return Buffer(h.value, self, dtype, int(numel))

    def copy_from_host(self, buffer: Buffer, src: Union[bytes, bytearray, memoryview]) -> None:
        data = bytes(src)
        call("fg_copy_h2d", buffer._h, data, len(data))

    def copy_to_host(self, buffer: Buffer) -> bytes:
        out = ctypes.create_string_buffer(buffer.nbytes)
        call("fg_copy_d2h", buffer._h, out, buffer.nbytes)
        return out.raw

    def compile(self, source: str, func_name: str, num_args: int,
                grid: Sequence[int] = (1, 1, 1), block: Sequence[int] = (1, 1, 1)) -> Program:
        g = (ctypes.c_uint32 * 3)(*(list(grid) + [1] * (3 - len(grid))))
        b = (ctypes.c_uint32 * 3)(*(list(block) + [1] * (3 - len(block))))
        h = ctypes.c_void_p()
        call("fg_compile", self._h, source.encode(), func_name.encode(), int(num_args), g, b,
             ctypes.byref(h))
        return Program(h.value, func_name, num_args)

    def execute(self, program: Program, args: Sequence[KernelArg]) -> None:
        arr = (_lib.KernelArgC * max(1, len(args)))()
        for i, a in enumerate(args):
            arr[i].kind = a.kind
            if a.kind == _lib.ARG_BUFFER:
                arr[i].v.buffer = a.value._h
            elif a.kind == _lib.ARG_I32:
                arr[i].v.i32 = a.value
            elif a.kind == _lib.ARG_F32:
                arr[i].v.f32 = a.value
            else:
                arr[i].v.b = 1 if a.value else 0
        call("fg_execute", program._h, arr, len(args))

    def cached_program(self, key) -> Optional[Program]:
        return self._programs.get(key)

    def insert_program(self, key, program: Program) -> None:
        self._programs[key] = program

    def clear_for_tests(self) -> None:
        self._programs.clear()
