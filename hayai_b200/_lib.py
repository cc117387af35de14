"""Loader and ctypes declarations for libhayai_cuda.so (the C ABI of include/hayai_cuda.h).

The library is built in-tree (``hayai_b200/lib``) by ``__graft_entry__.build()``.  There is
no fallback: if the shared library is missing, every entry point of the package fails
with ``NativeLibraryMissing``.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libhayai_cuda.so")

HC_OK = 0
HC_ERR_INVALID = 1
HC_ERR_UNSUPPORTED = 2
HC_ERR_CUDA = 3
HC_ERR_RANGE = 4
HC_ERR_NCCL = 5
HC_ERR_TIMEOUT = 6


class NativeLibraryMissing(RuntimeError):
    pass


_P = ctypes.c_void_p
_S = ctypes.c_size_t
_I = ctypes.c_int
_F = ctypes.c_float
_PP = ctypes.POINTER(ctypes.c_void_p)

# name -> argtypes (all return int status except hc_last_error)
SIGNATURES: dict[str, list] = {
    "hc_device_count": [ctypes.POINTER(_I)],
    "hc_engine_init": [_I, _PP],
    "hc_engine_free": [_P],
    "hc_engine_set_stream": [_P, _P],
    "hc_engine_use_own_stream": [_P],
    "hc_engine_get_stream": [_P, _PP],
    "hc_sync": [_P],
    "hc_gemv_row_bytes": [_I, _S, ctypes.POINTER(_S)],
    "hc_weights_upload": [_P, _I, _S, _S, _P, _S, _PP],
    "hc_weights_from_device": [_P, _I, _S, _S, _P, _S, _PP],
    "hc_weights_free": [_P],
    "hc_weights_info": [_P, ctypes.POINTER(_I), ctypes.POINTER(_S), ctypes.POINTER(_S), ctypes.POINTER(_S)],
    "hc_ggml_gemv_dispatch": [_P, _I, _S, _S, _P, _S, _P, _P],
    "hc_ggml_gemv_bound": [_P, _P, _P, _P],
    "hc_ggml_gemv_batched": [_P, _P, _P, _P, _S],
    "hc_ggml_gemv_async": [_P, _P, _P, _PP],
    "hc_pending_wait": [_P, _P, _S],
    "hc_pending_free": [_P],
    "hc_gemv_dev": [_P, _P, _P, _S, _P, _S, _P, _S, _S],
    "hc_gemv_dev_noalloc": [_P, _P, _P, _S, _P, _S, _P, _S, _S],
    "hc_lut_matmul_q4": [_P, _S, _S, _P, _P, _P, _P],
    "hc_lut_matmul_q4_dev": [_P, _S, _S, _P, _P, _P, _P],
    "hc_ffn_swiglu": [_P, _P, _P, _P, _P, _P, _S],
    "hc_ffn_swiglu_dev": [_P, _P, _P, _P, _P, _P, _P, _P, _S],
    "hc_ffn_gateup_dev": [_P, _P, _P, _P, _P, _S, _P, _S, _F],
    "hc_ffn_stack_dev": [_P, _P, _P, _P, _P, _F, _S, _P, _S],
    "hc_ffn_stack": [_P, _P, _P, _P, _P, _F, _S, _P, _P, _S],
    "hc_ffn_stack_tp_dev": [_P, _P, _P, _P, _P, _F, _S, _P, _S],
    "hc_ffn_stack_tp": [_P, _P, _P, _P, _P, _F, _S, _P, _P, _S],
    "hc_peer_handle_bytes": [_P],
    "hc_peer_open": [_P, _I, _I, _S, _P],
    "hc_peer_connect": [_P, _P],
    "hc_peer_close": [_P],
    "hc_peer_region": [_P, _P, _P],
    "hc_route_experts_dev": [_P, _P, _P, _S, _S, _S, _S, _S, _I, _I, _F, _P, _P],
    "hc_router_scores_dev": [_P, _P, _S, _S, _P, _S, _P],
    "hc_moe_ffn_dev": [_P, _P, _S, _S, _I, _F, _P, _P, _P, _P, _S, _P, _P, _P],
    "hc_moe_ffn_ep_dev": [_P, _P, _S, _S, _I, _F, _P, _P, _P, _S, _S, _P, _S, _P, _P, _P],
    "hc_moe_stack_dev": [_P, _S, _P, _S, _S, _I, _F, _P, _P, _P, _P, _S],
    "hc_moe_stack_ep_dev": [_P, _S, _P, _S, _S, _I, _F, _P, _P, _P, _S, _S, _P, _S],
    "hc_synth_normal_dev": [_P, ctypes.c_uint64, _S, _F, _F, _P],
    "hc_quantize_dev": [_P, _I, _P, _S, _P],
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} is not built; run __graft_entry__.build() (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.hc_last_error.restype = ctypes.c_char_p
        L.hc_last_error.argtypes = []
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = _I
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return ["hc_last_error", *SIGNATURES.keys()]
