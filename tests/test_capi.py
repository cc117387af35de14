"""CPU tests of the C ABI: the library loads, exports every symbol include/hayai_cuda.h
declares, and its host-side validation mirrors the reference (no compute, no GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

import hayai_b200
from hayai_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "hayai_cuda.h")


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(hc_[a-z0-9_]+)\s*\(", text))


def test_library_loads():
    assert os.path.exists(_lib.LIB_PATH)
    _lib.lib()


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in sorted(syms) if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_header():
    assert declared_symbols() == set(_lib.exported_symbols())


def test_rust_binding_covers_header():
    """The hayai-cuda crate (integration/hayai-cuda, not compiled here: no Rust toolchain on
    this image) declares exactly the header's entry points, with as many parameters each."""
    root = os.path.dirname(HEADER)
    ffi = open(os.path.join(root, "..", "integration", "hayai-cuda", "src", "ffi.rs")).read()
    rust = dict(re.findall(r"pub fn (hc_[a-z0-9_]+)\(([^)]*)\)", ffi, flags=re.S))
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    c = dict(re.findall(r"\b(hc_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text, flags=re.S))
    assert set(rust) == set(c) == declared_symbols()

    def nparams(args):
        args = args.strip()
        return 0 if args in ("", "void") else args.count(",") + 1

    for name in c:
        assert nparams(rust[name]) == nparams(c[name]), name


# gemv_row_bytes (crates/hayai-opencl/src/compute.rs:877-907) for the formats with a kernel here
@pytest.mark.parametrize("t,n,expect", [
    (hayai_b200.Q4_K, 4096, 16 * 144), (hayai_b200.Q6_K, 14336, 56 * 210), (hayai_b200.Q8_0, 4096, 128 * 34),
    (hayai_b200.IQ2_XXS, 256, 66), (hayai_b200.IQ2_XS, 512, 148), (hayai_b200.IQ2_S, 256, 82),
    (hayai_b200.IQ3_XXS, 256, 98), (hayai_b200.IQ3_S, 768, 330), (hayai_b200.F32, 7, 28)])
def test_row_bytes_table(t, n, expect):
    assert hayai_b200.row_bytes(t, n) == expect


def test_row_bytes_rejects_partial_block():
    with pytest.raises(hayai_b200.CudaError) as e:
        hayai_b200.row_bytes(hayai_b200.Q4_K, 576)
    assert e.value.code == _lib.HC_ERR_INVALID
    assert "not a valid column count" in str(e.value)


def test_unsupported_type_is_a_hard_error():
    with pytest.raises(hayai_b200.CudaError) as e:
        hayai_b200.row_bytes(19, 256)  # IQ1_S: no kernel (the reference hard-fails IQ1 too)
    assert e.value.code == _lib.HC_ERR_UNSUPPORTED


def test_engine_init_without_gpu_reports_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = _lib.lib().hc_engine_init(0, ctypes.byref(h))
    assert rc != 0 and not h.value
    assert _lib.lib().hc_last_error()


def test_null_arguments_rejected_before_any_device_call():
    L = _lib.lib()
    assert L.hc_engine_init(0, None) == _lib.HC_ERR_INVALID
    assert L.hc_weights_info(None, None, None, None, None) == _lib.HC_ERR_INVALID
    assert L.hc_pending_free(None) == 0 and L.hc_weights_free(None) == 0 and L.hc_engine_free(None) == 0


def test_error_message_is_thread_local():
    import threading

    L = _lib.lib()
    hayai_b200.engine._check  # noqa: B018  (import side effects)
    out = {}

    def worker():
        L.hc_gemv_row_bytes(12, 100, None)
        out["t"] = L.hc_last_error()

    L.hc_gemv_row_bytes(99, 256, None)
    main_msg = L.hc_last_error()
    th = threading.Thread(target=worker)
    th.start()
    th.join()
    assert b"type 99" in main_msg and b"n=100" in out["t"]
    assert L.hc_last_error() == main_msg


def test_python_wrappers_validate_shapes_without_gpu():
    eng = object.__new__(hayai_b200.CudaEngine)  # no device needed for argument checks
    eng.handle = ctypes.c_void_p(0)
    with pytest.raises(ValueError):
        eng.lut_matmul_q4(4, 3, np.zeros(6, np.uint8), np.zeros(16, np.float32), np.zeros(3, np.float32))
    with pytest.raises(ValueError):
        eng.ggml_gemv_dispatch(hayai_b200.Q4_K, 4, 256, np.zeros(4 * 144, np.uint8), np.zeros(255, np.float32))
