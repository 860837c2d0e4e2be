"""The reference's device tests (src/device.rs:427-477, src/device/cpu.rs:518-649)
re-expressed against the CUDA device through the C ABI."""
import json
import os
import struct

import numpy as np
import pytest

from ferrograd_b200 import CudaDevice, FerroError, KernelArg
from ferrograd_b200._lib import BOOL, F32, I32

pytestmark = pytest.mark.gpu

KAT = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))


@pytest.fixture(scope="module")
def dev():
    return CudaDevice(0)


def f32_buffer(dev, data):
    buf = dev.allocate(F32, len(data))
    dev.copy_from_host(buf, np.asarray(data, np.float32).tobytes())
    return buf


def read_f32(dev, buf):
    return np.frombuffer(dev.copy_to_host(buf), dtype=np.float32).tolist()


def test_allocate_zeroed(dev):
    buf = dev.allocate(F32, 4)
    assert buf.numel == 4 and buf.nbytes == 16
    assert dev.copy_to_host(buf) == b"\x00" * 16


def test_f32_roundtrip(dev):
    buf = f32_buffer(dev, [1.0, 2.0, 3.0])
    assert read_f32(dev, buf) == [1.0, 2.0, 3.0]


def test_copyin_copyout_raw_i32(dev):
    buf = dev.allocate(I32, 2)
    src = bytes([1, 0, 0, 0, 2, 0, 0, 0])
    dev.copy_from_host(buf, src)
    assert dev.copy_to_host(buf) == src


def test_i32_and_bool_roundtrip(dev):
    # src/tensor.rs:1278-1313
    b = dev.allocate(I32, 3)
    dev.copy_from_host(b, struct.pack("<3i", *KAT["i32_roundtrip"]["input"]))
    assert list(struct.unpack("<3i", dev.copy_to_host(b))) == [1, 2, 3]
    bb = dev.allocate(BOOL, 3)
    dev.copy_from_host(bb, bytes([1, 0, 1]))
    assert dev.copy_to_host(bb) == bytes([1, 0, 1])


def test_copyin_wrong_size_fails(dev):
    buf = dev.allocate(F32, 2)
    with pytest.raises(FerroError) as e:
        dev.copy_from_host(buf, b"\x00" * 4)
    assert KAT["copyin_wrong_size"]["message"] in str(e.value)


def _compile(dev, src, name, nargs, n=32):
    return dev.compile(src, name, nargs, grid=(1, 1, 1), block=(n, 1, 1))


def test_device_add(dev):
    src = r'''extern "C" __global__ void add(float* out, float* a, float* b) {
        int i = threadIdx.x; if (i < 3) out[i] = a[i] + b[i]; }'''
    prog = _compile(dev, src, "add", 3)
    k = KAT["device_add"]
    out = dev.allocate(F32, 3)
    dev.execute(prog, [KernelArg.buffer(out), KernelArg.buffer(f32_buffer(dev, k["a"])),
                       KernelArg.buffer(f32_buffer(dev, k["b"]))])
    assert read_f32(dev, out) == k["expected"]


def test_device_mul(dev):
    src = r'''extern "C" __global__ void mul(float* out, float* a, float* b) {
        int i = threadIdx.x; if (i < 3) out[i] = a[i] * b[i]; }'''
    prog = _compile(dev, src, "mul", 3)
    k = KAT["device_mul"]
    out = dev.allocate(F32, 3)
    dev.execute(prog, [KernelArg.buffer(out), KernelArg.buffer(f32_buffer(dev, k["a"])),
                       KernelArg.buffer(f32_buffer(dev, k["b"]))])
    assert read_f32(dev, out) == k["expected"]


def test_device_unary(dev):
    src = r'''extern "C" __global__ void negate(float* output, float* input) {
        int i = threadIdx.x; if (i < 3) output[i] = -input[i]; }'''
    prog = _compile(dev, src, "negate", 2)
    k = KAT["device_unary"]
    out = dev.allocate(F32, 3)
    dev.execute(prog, [KernelArg.buffer(out), KernelArg.buffer(f32_buffer(dev, k["input"]))])
    assert read_f32(dev, out) == k["expected"]


def test_device_mixed_scalar_args(dev):
    src = r'''extern "C" __global__ void add_offset(float* out, float* input, int offset, float scale) {
        int i = threadIdx.x; if (i < 2) out[i] = (input[offset + i] * scale); }'''
    prog = _compile(dev, src, "add_offset", 4)
    k = KAT["device_mixed_scalar_args"]
    out = dev.allocate(F32, 2)
    dev.execute(prog, [KernelArg.buffer(out), KernelArg.buffer(f32_buffer(dev, k["input"])),
                       KernelArg.i32(k["offset"]), KernelArg.f32(k["scale"])])
    assert read_f32(dev, out) == k["expected"]


def test_device_compile_bad_source(dev):
    with pytest.raises(FerroError) as e:
        dev.compile("not valid CUDA!", "nope", 1)
    assert "nvrtc" in str(e.value).lower()


def test_execute_wrong_arg_count(dev):
    src = r'''extern "C" __global__ void one(float* out) { out[0] = 1.0f; }'''
    prog = _compile(dev, src, "one", 1, n=1)
    with pytest.raises(FerroError) as e:
        dev.execute(prog, [])
    assert "expected 1 kernel args, got 0" in str(e.value)


def test_program_cache(dev):
    src = r'''extern "C" __global__ void fill(float* out) { out[threadIdx.x] = 7.0f; }'''
    prog = _compile(dev, src, "fill", 1, n=4)
    dev.insert_program("fill-key", prog)
    assert dev.cached_program("fill-key") is prog
    out = dev.allocate(F32, 4)
    dev.execute(dev.cached_program("fill-key"), [KernelArg.buffer(out)])
    assert read_f32(dev, out) == [7.0] * 4
    dev.clear_for_tests()
    assert dev.cached_program("fill-key") is None


def test_event_elapsed_times_of_a_known_kernel_are_positive_and_ordered(dev):
    """fg_event_*: the device timing DEBUG >= 2 reports per kernel
    (src/tensor.rs:1017-1028).  Three events bracket two launches of a kernel
    that spins for a fixed number of global-timer nanoseconds, so the elapsed
    times must be positive, ordered (start->mid <= start->end) and at least
    the spin."""
    from ferrograd_b200.device import Event
    src = r'''extern "C" __global__ void spin(float* out, int ns) {
        unsigned long long t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        do { asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); } while (t - t0 < (unsigned long long)ns);
        out[0] = (float)(t - t0); }'''
    prog = _compile(dev, src, "spin", 2, n=1)
    out = dev.allocate(F32, 1)
    args = [KernelArg.buffer(out), KernelArg.i32(2_000_000)]  # 2 ms
    dev.execute(prog, args)  # first launch loads the module
    dev.synchronize()
    e0, e1, e2 = Event(dev), Event(dev), Event(dev)
    e0.record()
    dev.execute(prog, args)
    e1.record()
    dev.execute(prog, args)
    e2.record()
    t01 = Event.elapsed_ms(e0, e1)
    t02 = Event.elapsed_ms(e0, e2)
    t12 = Event.elapsed_ms(e1, e2)
    assert 2.0 <= t01 < 1000.0 and 2.0 <= t12 < 1000.0
    assert t01 <= t02 and t12 <= t02
    assert abs(t02 - (t01 + t12)) <= 0.05 * t02


def test_library_kernels_run_as_sm100a():
    """The kernels of libferro_cuda.so run from an sm_100a binary on this
    device (cudaFuncGetAttributes: binaryVersion 100), not from PTX JIT."""
    import ctypes

    from ferrograd_b200 import _lib
    bv, pv = ctypes.c_int(), ctypes.c_int()
    _lib.call("fg_kernel_arch", ctypes.byref(bv), ctypes.byref(pv))
    assert bv.value == 100, bv.value
