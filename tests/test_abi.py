"""CPU-side checks of the C ABI: the library loads, exports every entry point
``include/ferro_cuda.h`` declares, and its host-only parts behave (no GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ferro_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fg_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ("fg_device_open", "fg_alloc", "fg_copy_h2d", "fg_copy_d2h", "fg_compile",
                 "fg_execute", "fg_gemm_3xtf32", "fg_xent_fwd_bwd", "fg_mlp_step_host",
                 "fg_comm_init", "fg_allreduce_mean_f32"):
        assert must in syms


def test_library_exports_every_declared_symbol():
    from ferrograd_b200 import _lib
    L = _lib.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    # the Python binding declares a signature for every exported entry point
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert set(declared_symbols()) <= bound, set(declared_symbols()) - bound


def test_kaiming_init_matches_oracle_bit_exact(oracle):
    """Linear::new init in the product library equals the oracle's restatement."""
    from ferrograd_b200.mlp import InitRng, mlp_init
    ws, bs = mlp_init((784, 128, 10), InitRng())
    orng = oracle.InitRng()
    w1, b1 = orng.linear(784, 128)
    w2, b2 = orng.linear(128, 10)
    assert np.array_equal(ws[0], w1) and np.array_equal(ws[1], w2)
    assert np.array_equal(bs[0], b1) and bs[1].tolist() == [0.0] * 10


def test_errors_are_reported_not_raised_without_gpu():
    """Without a GPU, device calls fail with a status code and a message."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from ferrograd_b200 import _lib
    L = _lib.lib()
    h = ctypes.c_void_p()
    rc = L.fg_device_open(0, ctypes.byref(h))
    assert rc != 0
    assert L.fg_last_error().decode()


def test_invalid_arguments_rejected_before_any_device_work():
    from ferrograd_b200 import _lib
    L = _lib.lib()
    assert L.fg_gemm_3xtf32(0, 4, 4, None, None, 4, None, None, 4, None, None, 4, 0, 0,
                            None, None, 0, None) == 1
    assert b"positive" in L.fg_last_error()
    assert L.fg_reduce_rows(7, 0, None, None, 1, 1, None) == 1
    assert L.fg_kaiming_normal(None, 4, 1, None) == 1


def test_event_entry_points_reject_null_arguments_without_a_gpu():
    from ferrograd_b200 import _lib
    L = _lib.lib()
    out = ctypes.c_void_p()
    ms = ctypes.c_float()
    assert L.fg_event_create(None, ctypes.byref(out)) == 1  # FG_ERR_INVALID
    assert L.fg_event_record(None, None) == 1
    assert L.fg_event_elapsed_ms(None, None, ctypes.byref(ms)) == 1
    assert L.fg_event_destroy(None) == 0


def test_python_constants_match_the_header():
    """Sizes the binding allocates for handles must be the header's."""
    from ferrograd_b200 import _lib
    text = open(HEADER).read()
    defs = dict(re.findall(r"#define\s+(FG_[A-Z0-9_]+)\s+(\d+)", text))
    assert int(defs["FG_UNIQUE_ID_BYTES"]) == _lib.UNIQUE_ID_BYTES
    assert int(defs["FG_PEER_HANDLE_BYTES"]) == _lib.PEER_HANDLE_BYTES


def test_missing_library_fails_loudly(tmp_path):
    """No CPU fallback: without libferro_cuda.so the package refuses to load,
    naming the file and the build command; without the front-end extension
    the Tensor API refuses to import."""
    import subprocess
    import sys
    code = (
        "import ferrograd_b200._lib as L\n"
        f"L.LIB_PATH = {str(tmp_path / 'absent.so')!r}\n"
        "L._lib = None\n"
        "try:\n"
        "    L.lib()\n"
        "except L.FerroError as e:\n"
        "    assert 'absent.so is missing' in str(e) and 'ferrograd_b200.build' in str(e), e\n"
        "    print('ok')\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=120, cwd=ROOT)
    assert out.stdout.strip() == "ok", out.stderr
    code = (
        "import sys, builtins\n"
        "real = builtins.__import__\n"
        "def fake(name, *a, **k):\n"
        "    if name.endswith('_front') or (a and a[2] and '_front' in a[2]):\n"
        "        raise ImportError('no _front')\n"
        "    return real(name, *a, **k)\n"
        "builtins.__import__ = fake\n"
        "try:\n"
        "    import ferrograd_b200.front\n"
        "except ImportError as e:\n"
        "    assert 'not built' in str(e), e\n"
        "    print('ok')\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=120, cwd=ROOT)
    assert out.stdout.strip() == "ok", out.stderr
