"""ctypes binding of the CPU oracle (``hayai_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` as the parity checker / timed CPU baseline.
The product path (``hayai_b200``) never imports this package.

Every function restates the reference's Rust CPU code; see the C file for the
file:line each one follows.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

# GgmlType ids (crates/hayai-model/src/gguf_types.rs:6-40)
F32, Q8_0, Q4_K, Q6_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ3_S, IQ2_S = 0, 8, 12, 14, 16, 17, 18, 21, 22
Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, IQ4_NL, IQ4_XS = 2, 3, 6, 7, 10, 11, 13, 20, 23
F16, Q8_1, Q8_K, BF16 = 1, 9, 15, 30

# (elements per block, bytes per block), crates/hayai-opencl/src/compute.rs:877-907; q5.rs:8-9,
# q5k.rs:8, q2k.rs:8, q3k.rs:8, iq4.rs:8-11
BLOCK = {
    F32: (1, 4), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), IQ2_XXS: (256, 66),
    IQ2_XS: (256, 74), IQ2_S: (256, 82), IQ3_XXS: (256, 98), IQ3_S: (256, 110),
    Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), Q2_K: (256, 84), Q3_K: (256, 110),
    Q5_K: (256, 176), IQ4_NL: (32, 18), IQ4_XS: (256, 136),
    F16: (1, 2), BF16: (1, 2), Q8_1: (32, 36), Q8_K: (256, 292),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"oracle library not built: {LIB_PATH} (run __graft_entry__.build())")
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_S = ctypes.c_size_t


def _declare(L: ctypes.CDLL) -> None:
    L.or_f16_to_f32.restype = ctypes.c_float
    L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.or_f32_to_f16.restype = ctypes.c_uint16
    L.or_f32_to_f16.argtypes = [ctypes.c_float]
    L.or_rng_u64.restype = ctypes.c_uint64
    L.or_rng_u64.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
    L.or_fill_normal.restype = None
    L.or_fill_normal.argtypes = [ctypes.c_uint64, _S, ctypes.c_float, ctypes.c_float, _P]
    L.or_fill_bytes.restype = None
    L.or_fill_bytes.argtypes = [ctypes.c_uint64, _S, _P]
    for name in ("or_quantize_q4_k", "or_quantize_q6_k", "or_quantize_q8_0"):
        f = getattr(L, name)
        f.restype = ctypes.c_int
        f.argtypes = [_P, _S, _P]
    L.or_dequant.restype = ctypes.c_int
    L.or_dequant.argtypes = [ctypes.c_int, _P, _S, _P]
    L.or_gemv.restype = ctypes.c_int
    L.or_gemv.argtypes = [ctypes.c_int, _S, _S, _P, _P, _P]
    L.or_lut_matmul_q4.restype = None
    L.or_lut_matmul_q4.argtypes = [_S, _S, _P, _P, _P, _P]
    L.or_fp32_matmul.restype = None
    L.or_fp32_matmul.argtypes = [_S, _S, _P, _P, _P]
    L.or_swiglu.restype = None
    L.or_swiglu.argtypes = [_P, _P, _P, _S]
    L.or_ffn_swiglu.restype = ctypes.c_int
    L.or_ffn_swiglu.argtypes = [ctypes.c_int, _P, ctypes.c_int, _P, ctypes.c_int, _P, _S, _S, _S, _P, _P]
    L.or_route_experts.restype = ctypes.c_int
    L.or_route_experts.argtypes = [_P, _P, _S, _S, _S, _S, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P, _P]
    L.or_moe_ffn.restype = ctypes.c_int
    L.or_moe_ffn.argtypes = [_P, _P, _S, _S, ctypes.c_int, ctypes.c_float,
                             ctypes.c_int, _P, _S, ctypes.c_int, _P, _S, ctypes.c_int, _P, _S,
                             _S, _S, _S, _P, _P, _P, _P]
    L.or_rms_norm.restype = None
    L.or_rms_norm.argtypes = [_P, _P, _S, ctypes.c_float, _P]
    L.or_set_threads.restype = None
    L.or_set_threads.argtypes = [ctypes.c_int]
    L.or_get_threads.restype = ctypes.c_int
    L.or_get_threads.argtypes = []


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def row_bytes(ggml_type: int, ncols: int) -> int:
    qk, nb = BLOCK[ggml_type]
    if ncols % qk:
        raise ValueError(f"ncols={ncols} not a multiple of {qk}")
    return ncols // qk * nb


# ---------------------------------------------------------------- data
def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def get_threads() -> int:
    return lib().or_get_threads()


def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def f32_to_f16(v: float) -> int:
    return lib().or_f32_to_f16(v)


def normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().or_fill_normal(seed & (2**64 - 1), n, mean, std, _ptr(out))
    return out


def random_bytes(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint8)
    lib().or_fill_bytes(seed & (2**64 - 1), n, _ptr(out))
    return out


def quantize(ggml_type: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    qk, nb = BLOCK[ggml_type]
    out = np.zeros(x.size // qk * nb, dtype=np.uint8)
    fn = {Q4_K: lib().or_quantize_q4_k, Q6_K: lib().or_quantize_q6_k, Q8_0: lib().or_quantize_q8_0}[ggml_type]
    if fn(_ptr(x), x.size, _ptr(out)) != 0:
        raise ValueError("quantize: size not a multiple of the block")
    return out


def dequant(ggml_type: int, w: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    rc = lib().or_dequant(ggml_type, _ptr(np.ascontiguousarray(w)), n, _ptr(out))
    if rc != 0:
        raise ValueError(f"dequant rc={rc}")
    return out


# ---------------------------------------------------------------- compute
def gemv(ggml_type: int, m: int, n: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    if w.dtype != np.uint8:  # F32 / F16 / BF16 element arrays: their bytes
        w = w.view(np.uint8)
    assert w.nbytes >= m * row_bytes(ggml_type, n), "weights too small"
    y = np.empty(m, dtype=np.float32)
    rc = lib().or_gemv(ggml_type, m, n, _ptr(w), _ptr(x), _ptr(y))
    if rc != 0:
        raise ValueError(f"gemv rc={rc}")
    return y


def lut_matmul_q4(m: int, n: int, w: np.ndarray, lut: np.ndarray, x: np.ndarray) -> np.ndarray:
    y = np.empty(m, dtype=np.float32)
    lib().or_lut_matmul_q4(m, n, _ptr(np.ascontiguousarray(w, dtype=np.uint8)),
                           _ptr(np.ascontiguousarray(lut, dtype=np.float32)),
                           _ptr(np.ascontiguousarray(x, dtype=np.float32)), _ptr(y))
    return y


def fp32_matmul(m: int, n: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
    y = np.empty(m, dtype=np.float32)
    lib().or_fp32_matmul(m, n, _ptr(np.ascontiguousarray(w, dtype=np.float32)),
                         _ptr(np.ascontiguousarray(x, dtype=np.float32)), _ptr(y))
    return y


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    h = np.empty_like(g)
    lib().or_swiglu(_ptr(g), _ptr(u), _ptr(h), g.size)
    return h


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rms_norm (crates/hayai-cpu/src/attention.rs:142-147), out of place."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    assert x.size == w.size
    out = np.empty_like(x)
    lib().or_rms_norm(_ptr(x), _ptr(w), x.size, eps, _ptr(out))
    return out


def ffn_swiglu(tg: int, wg: np.ndarray, tu: int, wu: np.ndarray, td: int, wd: np.ndarray,
               k_in: int, d_ff: int, n_out: int, x: np.ndarray) -> np.ndarray:
    y = np.empty(n_out, dtype=np.float32)
    rc = lib().or_ffn_swiglu(tg, _ptr(np.ascontiguousarray(wg)), tu, _ptr(np.ascontiguousarray(wu)),
                             td, _ptr(np.ascontiguousarray(wd)), k_in, d_ff, n_out,
                             _ptr(np.ascontiguousarray(x, dtype=np.float32)), _ptr(y))
    if rc != 0:
        raise ValueError(f"ffn rc={rc}")
    return y


def route_experts(scores: np.ndarray, top_k: int, bias: np.ndarray | None = None, n_group: int = 0,
                  topk_group: int = 0, gating: int = 0, norm_topk_prob: bool = False,
                  routed_scaling_factor: float = 1.0):
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    n = scores.size
    ids = np.zeros(max(n, 1), dtype=np.int32)
    w = np.zeros(max(n, 1), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    k = lib().or_route_experts(_ptr(scores), _ptr(b), n, top_k, n_group, topk_group, gating,
                               int(norm_topk_prob), routed_scaling_factor, _ptr(ids), _ptr(w))
    return ids[:k].copy(), w[:k].copy()


def moe_ffn(router_w: np.ndarray, n_expert: int, top_k: int, tg: int, wg: np.ndarray, tu: int, wu: np.ndarray,
            td: int, wd: np.ndarray, d_model: int, d_ff: int, x: np.ndarray, norm_topk_prob: bool = False,
            scaling: float = 1.0, router_bias: np.ndarray | None = None):
    """x: [n_tok, d_model]; expert e's matrices are wg[e], wu[e], wd[e] (2-D byte arrays)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, d_model)
    n_tok = x.shape[0]
    wg = np.ascontiguousarray(wg)
    wu = np.ascontiguousarray(wu)
    wd = np.ascontiguousarray(wd)
    y = np.empty_like(x)
    ids = np.empty((n_tok, top_k), dtype=np.int32)
    ws = np.empty((n_tok, top_k), dtype=np.float32)
    b = None if router_bias is None else np.ascontiguousarray(router_bias, dtype=np.float32)
    rc = lib().or_moe_ffn(_ptr(np.ascontiguousarray(router_w, dtype=np.float32)), _ptr(b), n_expert, top_k,
                          int(norm_topk_prob), scaling, tg, _ptr(wg), wg.shape[1] if wg.ndim == 2 else wg[0].nbytes,
                          tu, _ptr(wu), wu.shape[1] if wu.ndim == 2 else wu[0].nbytes,
                          td, _ptr(wd), wd.shape[1] if wd.ndim == 2 else wd[0].nbytes,
                          d_model, d_ff, n_tok, _ptr(x), _ptr(y), _ptr(ids), _ptr(ws))
    if rc != 0:
        raise ValueError(f"moe rc={rc}")
    return y, ids, ws
