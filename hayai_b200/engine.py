"""Host-side mirror of Hayai's GPU backend API, over the C ABI of libhayai_cuda.so.

``CudaEngine`` mirrors ``OpenClEngine``'s GEMV method set
(crates/hayai-opencl/src/compute.rs:45-461, async_gemv.rs:60-130): the same method
names, argument meaning (m = output rows, n = input columns, GGUF-layout weight bytes)
and error behaviour (validation failures and unsupported types raise, there is no
silent CPU fallback, orchestrator.rs:403-409).  ``QuantMatrix`` mirrors
crates/hayai-model/src/quant.rs:31-117; the orchestrator's dispatch is in
``hayai_b200.orchestrator``.

Device-memory entry points (``*_dev``) take torch CUDA tensors: torch is used for device
memory and streams only; all compute runs in the native library.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import lib

# GgmlType ids (crates/hayai-model/src/gguf_types.rs:6-40)
F32, Q8_0, Q4_K, Q6_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ3_S, IQ2_S = 0, 8, 12, 14, 16, 17, 18, 21, 22
Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, IQ4_NL, IQ4_XS = 2, 3, 6, 7, 10, 11, 13, 20, 23
F16, Q8_1, Q8_K, BF16 = 1, 9, 15, 30
TYPE_LABELS = {F32: "f32", Q8_0: "q8_0", Q4_K: "q4_k", Q6_K: "q6_k", IQ2_XXS: "iq2_xxs", IQ2_XS: "iq2_xs",
               IQ2_S: "iq2_s", IQ3_XXS: "iq3_xxs", IQ3_S: "iq3_s", Q4_0: "q4_0", Q4_1: "q4_1", Q5_0: "q5_0",
               Q5_1: "q5_1", Q2_K: "q2_k", Q3_K: "q3_k", Q5_K: "q5_k", IQ4_NL: "iq4_nl", IQ4_XS: "iq4_xs",
               F16: "f16", BF16: "bf16", Q8_1: "q8_1", Q8_K: "q8_k"}
LABEL_TYPES = {v: k for k, v in TYPE_LABELS.items()}
# (elements, bytes) per block: gemv_row_bytes (compute.rs:877-907)
BLOCK = {F32: (1, 4), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), IQ2_XXS: (256, 66), IQ2_XS: (256, 74),
         IQ2_S: (256, 82), IQ3_XXS: (256, 98), IQ3_S: (256, 110), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22),
         Q5_1: (32, 24), Q2_K: (256, 84), Q3_K: (256, 110), Q5_K: (256, 176), IQ4_NL: (32, 18), IQ4_XS: (256, 136),
         F16: (1, 2), BF16: (1, 2), Q8_1: (32, 36), Q8_K: (256, 292)}


class CudaError(RuntimeError):
    """Error returned by the native library (the OpenClError::ClError counterpart)."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def _check(rc: int) -> None:
    if rc != _lib.HC_OK:
        raise CudaError(rc, lib().hc_last_error().decode(errors="replace"))


def row_bytes(ggml_type: int, n: int) -> int:
    out = ctypes.c_size_t()
    _check(lib().hc_gemv_row_bytes(ggml_type, n, ctypes.byref(out)))
    return out.value


def device_count() -> int:
    n = ctypes.c_int()
    try:
        rc = lib().hc_device_count(ctypes.byref(n))
    except _lib.NativeLibraryMissing:
        raise
    return n.value if rc == 0 else 0


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    return a.view(np.uint8).reshape(-1)


def _tptr(t) -> int:
    """data_ptr of a CUDA torch tensor (or 0 for None)."""
    if t is None:
        return 0
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous CUDA tensor")
    return t.data_ptr()


class ResidentWeights:
    """A weight matrix uploaded once to HBM (GPU layout of its format)."""

    def __init__(self, engine: "CudaEngine", handle: int, ggml_type: int, m: int, n: int):
        self.engine = engine
        self.handle = ctypes.c_void_p(handle)
        self.ggml_type = ggml_type
        self.m = m
        self.n = n
        b = ctypes.c_size_t()
        _check(lib().hc_weights_info(self.handle, None, None, None, ctypes.byref(b)))
        self.nbytes = b.value

    def free(self) -> None:
        if self.handle:
            lib().hc_weights_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class PendingGemv:
    """In-flight GEMV (PendingGemv, async_gemv.rs:15-57): ``wait()`` returns the output;
    dropping it without waiting still blocks until the device is done."""

    def __init__(self, handle: int, m: int):
        self.handle = ctypes.c_void_p(handle)
        self.m = m

    def wait(self) -> np.ndarray:
        out = np.empty(self.m, dtype=np.float32)
        _check(lib().hc_pending_wait(self.handle, out.ctypes.data, self.m))
        self.free()
        return out

    def free(self) -> None:
        if self.handle:
            lib().hc_pending_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _handles(ws: Sequence[ResidentWeights]):
    arr = (ctypes.c_void_p * len(ws))(*[w.handle.value for w in ws])
    return arr


def _norm_ptrs(norms):
    """Array of device pointers of per-layer RMSNorm weights (torch CUDA tensors), or NULL."""
    if norms is None:
        return None
    return (ctypes.c_void_p * len(norms))(*[_tptr(t) for t in norms])


class BoundStack:
    """A layer stack bound once to an engine: its handle and norm-pointer arrays are built at
    binding, so a decode loop pays only the call (the bound-op pattern of the reference's
    orchestrator, crates/hayai-core/src/orchestrator.rs:276-392).  Holds references to the
    weights and norm tensors, which must stay alive and unchanged while it is used."""

    def __init__(self, engine, gates, ups, downs, norms=None, eps: float = 1e-5, tp: bool = False):
        if not (len(gates) == len(ups) == len(downs)) or not gates:
            raise ValueError("gates, ups and downs need the same, non-zero number of layers")
        self.engine = engine
        self._keep = (list(gates), list(ups), list(downs), None if norms is None else list(norms))
        self._g, self._u, self._d = _handles(gates), _handles(ups), _handles(downs)
        self._n = _norm_ptrs(norms)
        self.eps = float(eps)
        self.layers = len(gates)
        self._fn = lib().hc_ffn_stack_tp if tp else lib().hc_ffn_stack

    def run(self, x, out=None, nvec: int = 1) -> np.ndarray:
        """x <- x + FFN_l(rms_norm(x)) for every layer, host buffers (x float32 [nvec][d_model]);
        the result goes to ``out`` (a new array when None)."""
        xv = x if isinstance(x, np.ndarray) and x.dtype == np.float32 and x.flags.c_contiguous else _f32(x)
        if out is None:
            out = np.empty_like(xv)
        elif out.dtype != np.float32 or not out.flags.c_contiguous or out.size < xv.size:
            raise ValueError("out must be a contiguous float32 array at least the size of x")
        _check(self._fn(self.engine.handle, self._g, self._u, self._d, self._n, self.eps, self.layers,
                        xv.ctypes.data, out.ctypes.data, nvec))
        return out


class CudaEngine:
    """One GPU + stream (OpenClEngine, crates/hayai-opencl/src/context.rs:23)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().hc_engine_init(device, ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self) -> None:
        if self.handle:
            lib().hc_engine_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- streams
    def set_stream(self, stream) -> None:
        """Enqueue on a caller stream (a torch.cuda.Stream or a raw cudaStream_t handle; handle 0 is the
        legacy default stream), or on the engine's own stream when ``stream`` is None."""
        if stream is None:
            _check(lib().hc_engine_use_own_stream(self.handle))
            return
        ptr = stream if isinstance(stream, int) else stream.cuda_stream
        _check(lib().hc_engine_set_stream(self.handle, ctypes.c_void_p(ptr)))

    def stream_handle(self) -> int:
        s = ctypes.c_void_p()
        _check(lib().hc_engine_get_stream(self.handle, ctypes.byref(s)))
        return s.value or 0

    def sync(self) -> None:
        _check(lib().hc_sync(self.handle))

    # ---------------------------------------------------------------- weights
    def upload(self, ggml_type: int, m: int, n: int, weights) -> ResidentWeights:
        """One-time resident upload of GGUF-layout bytes (replaces the device mirror DMA)."""
        w = _u8(weights)
        h = ctypes.c_void_p()
        _check(lib().hc_weights_upload(self.handle, ggml_type, m, n, w.ctypes.data, w.nbytes, ctypes.byref(h)))
        return ResidentWeights(self, h.value, ggml_type, m, n)

    def upload_from_device(self, ggml_type: int, m: int, n: int, tensor) -> ResidentWeights:
        h = ctypes.c_void_p()
        nbytes = tensor.numel() * tensor.element_size()
        _check(lib().hc_weights_from_device(self.handle, ggml_type, m, n, ctypes.c_void_p(_tptr(tensor)), nbytes,
                                            ctypes.byref(h)))
        return ResidentWeights(self, h.value, ggml_type, m, n)

    # ---------------------------------------------------------------- GEMV (host buffers)
    def ggml_gemv_dispatch(self, ggml_type, m: int, n: int, weights, input, output=None) -> np.ndarray:
        """compute.rs:281-385 (``kernel``/``label`` are replaced by the ggml type id or label)."""
        t = LABEL_TYPES[ggml_type] if isinstance(ggml_type, str) else ggml_type
        x = _f32(input)
        if x.size != n:
            raise ValueError(f"input has {x.size} values, expected n={n}")
        w = _u8(weights)
        y = np.empty(m, dtype=np.float32) if output is None else output
        if y.dtype != np.float32 or y.size != m or not y.flags["C_CONTIGUOUS"]:
            raise ValueError("output must be a contiguous float32 array of m values")
        _check(lib().hc_ggml_gemv_dispatch(self.handle, t, m, n, w.ctypes.data, w.nbytes, x.ctypes.data,
                                           y.ctypes.data))
        return y

    def ggml_gemv_q4_k(self, m, n, weights, input, output=None):
        return self.ggml_gemv_dispatch(Q4_K, m, n, weights, input, output)

    def ggml_gemv_q6_k(self, m, n, weights, input, output=None):
        return self.ggml_gemv_dispatch(Q6_K, m, n, weights, input, output)

    def ggml_gemv_q8_0(self, m, n, weights, input, output=None):
        return self.ggml_gemv_dispatch(Q8_0, m, n, weights, input, output)

    def ggml_gemv_dispatch_bound(self, weights: ResidentWeights, input, output=None) -> np.ndarray:
        """compute.rs:388-461: resident weights, host input/output."""
        x = _f32(input)
        if x.size != weights.n:
            raise ValueError(f"input has {x.size} values, expected n={weights.n}")
        y = np.empty(weights.m, dtype=np.float32) if output is None else output
        _check(lib().hc_ggml_gemv_bound(self.handle, weights.handle, x.ctypes.data, y.ctypes.data))
        return y

    def ggml_gemv_batched(self, weights: ResidentWeights, inputs, batch: int, outputs=None) -> np.ndarray:
        """compute.rs:179-257 (any type): inputs [batch*n] -> outputs [batch*m]."""
        x = _f32(inputs)
        if x.size != batch * weights.n:
            raise ValueError("inputs must hold batch*n values")
        y = np.empty(batch * weights.m, dtype=np.float32) if outputs is None else outputs
        _check(lib().hc_ggml_gemv_batched(self.handle, weights.handle, x.ctypes.data, y.ctypes.data, batch))
        return y

    def ggml_gemv_batched_q4_k(self, m, n, weights, inputs, outputs, batch):
        rw = self.upload(Q4_K, m, n, weights)
        try:
            self.ggml_gemv_batched(rw, inputs, batch, outputs)
        finally:
            rw.free()
        return outputs

    def ggml_gemv_async(self, weights: ResidentWeights, input) -> PendingGemv:
        """async_gemv.rs:90-130: enqueue and return a PendingGemv."""
        x = _f32(input)
        if x.size != weights.n:
            raise ValueError(f"input has {x.size} values, expected n={weights.n}")
        h = ctypes.c_void_p()
        _check(lib().hc_ggml_gemv_async(self.handle, weights.handle, x.ctypes.data, ctypes.byref(h)))
        return PendingGemv(h.value, weights.m)

    def lut_matmul_q4(self, m: int, n: int, weights_q4, lut, input, output=None) -> np.ndarray:
        """compute.rs:45-128: toy 16-entry LUT matmul (two nibbles per byte, low first)."""
        if n % 2:
            raise ValueError("N must be even for packed Q4 weights")
        w = _u8(weights_q4)
        if w.size != m * (n // 2):
            raise ValueError("weights_q4 must hold m*n/2 bytes")
        lt = _f32(lut)
        x = _f32(input)
        if lt.size != 16 or x.size != n:
            raise ValueError("lut must hold 16 values and input n values")
        y = np.empty(m, dtype=np.float32) if output is None else output
        _check(lib().hc_lut_matmul_q4(self.handle, m, n, w.ctypes.data, lt.ctypes.data, x.ctypes.data,
                                      y.ctypes.data))
        return y

    # ---------------------------------------------------------------- FFN (host buffers)
    def ffn_swiglu(self, gate: ResidentWeights, up: ResidentWeights, down: ResidentWeights, x,
                   nvec: int = 1) -> np.ndarray:
        xv = _f32(x)
        y = np.empty(nvec * down.m, dtype=np.float32)
        _check(lib().hc_ffn_swiglu(self.handle, gate.handle, up.handle, down.handle, xv.ctypes.data,
                                   y.ctypes.data, nvec))
        return y

    def bind_ffn_stack(self, gates, ups, downs, norms=None, eps: float = 1e-5, tp: bool = False) -> BoundStack:
        """Bind a layer stack for repeated host-buffer calls (see BoundStack); tp: the
        tensor-parallel stack over this rank's d_ff shard (ffn_stack_tp)."""
        return BoundStack(self, gates, ups, downs, norms, eps, tp)

    def ffn_stack(self, gates, ups, downs, x, nvec: int = 1, norms=None, eps: float = 1e-5) -> np.ndarray:
        """x <- x + FFN_l(rms_norm(x, norms[l])) for every layer (host buffers in and out).
        ``norms`` is a list of float32 CUDA tensors (or None for no normalization)."""
        xv = _f32(x)
        out = np.empty_like(xv)
        _check(lib().hc_ffn_stack(self.handle, _handles(gates), _handles(ups), _handles(downs), _norm_ptrs(norms),
                                  eps, len(gates), xv.ctypes.data, out.ctypes.data, nvec))
        return out

    # ---------------------------------------------------------------- device tensors
    def gemv_dev(self, w: ResidentWeights, x, y, resid=None, nvec: int = 1) -> None:
        ldx = x.shape[-1]
        ldy = y.shape[-1]
        ldr = resid.shape[-1] if resid is not None else 0
        _check(lib().hc_gemv_dev(self.handle, w.handle, ctypes.c_void_p(_tptr(x)), ldx, ctypes.c_void_p(_tptr(y)),
                                 ldy, ctypes.c_void_p(_tptr(resid)), ldr, nvec))

    def lut_matmul_q4_dev(self, m, n, w, lut, x, y) -> None:
        _check(lib().hc_lut_matmul_q4_dev(self.handle, m, n, ctypes.c_void_p(_tptr(w)), ctypes.c_void_p(_tptr(lut)),
                                          ctypes.c_void_p(_tptr(x)), ctypes.c_void_p(_tptr(y))))

    def ffn_swiglu_dev(self, gate, up, down, x, y, resid=None, h_ws=None, nvec: int = 1) -> None:
        _check(lib().hc_ffn_swiglu_dev(self.handle, gate.handle, up.handle, down.handle, ctypes.c_void_p(_tptr(x)),
                                       ctypes.c_void_p(_tptr(y)), ctypes.c_void_p(_tptr(resid)),
                                       ctypes.c_void_p(_tptr(h_ws)), nvec))

    def ffn_gateup_dev(self, gate, up, x, h, nvec: int = 1, norm=None, norm_len: int = 0, eps: float = 1e-5) -> None:
        _check(lib().hc_ffn_gateup_dev(self.handle, gate.handle, up.handle, ctypes.c_void_p(_tptr(x)),
                                       ctypes.c_void_p(_tptr(h)), nvec, ctypes.c_void_p(_tptr(norm)),
                                       norm_len if norm is not None else 0, eps))

    def ffn_stack_dev(self, gates, ups, downs, x, nvec: int = 1, norms=None, eps: float = 1e-5) -> None:
        _check(lib().hc_ffn_stack_dev(self.handle, _handles(gates), _handles(ups), _handles(downs), _norm_ptrs(norms),
                                      eps, len(gates), ctypes.c_void_p(_tptr(x)), nvec))

    # ---------------------------------------------------------------- tensor parallelism
    def peer_open(self, rank: int, world: int, nbytes: int = 64 << 20) -> bytes:
        """Allocate this rank's exchange region; returns its IPC handle (to be gathered)."""
        n = ctypes.c_size_t()
        _check(lib().hc_peer_handle_bytes(ctypes.byref(n)))
        buf = (ctypes.c_ubyte * n.value)()
        _check(lib().hc_peer_open(self.handle, rank, world, nbytes, buf))
        return bytes(buf)

    def peer_connect(self, handles: Sequence[bytes]) -> None:
        """Map every rank's region (handles in rank order, this rank's included)."""
        blob = b"".join(handles)
        buf = (ctypes.c_ubyte * len(blob)).from_buffer_copy(blob)
        _check(lib().hc_peer_connect(self.handle, buf))

    def peer_close(self) -> None:
        _check(lib().hc_peer_close(self.handle))

    def peer_region(self) -> tuple[int, int]:
        """(device address, bytes) of this rank's exchange region."""
        p, n = ctypes.c_void_p(), ctypes.c_size_t()
        _check(lib().hc_peer_region(self.handle, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def ffn_stack_tp_dev(self, gates, ups, downs, x, nvec: int = 1, norms=None, eps: float = 1e-5) -> None:
        """Tensor-parallel stack over this rank's d_ff shard; x [nvec][d_model] replicated, in place."""
        _check(lib().hc_ffn_stack_tp_dev(self.handle, _handles(gates), _handles(ups), _handles(downs),
                                         _norm_ptrs(norms), eps, len(gates), ctypes.c_void_p(_tptr(x)), nvec))

    def ffn_stack_tp(self, gates, ups, downs, x, nvec: int = 1, norms=None, eps: float = 1e-5) -> np.ndarray:
        """Host-buffer version of ffn_stack_tp_dev (x copied in, the result copied out)."""
        xv = _f32(x)
        out = np.empty_like(xv)
        _check(lib().hc_ffn_stack_tp(self.handle, _handles(gates), _handles(ups), _handles(downs), _norm_ptrs(norms),
                                     eps, len(gates), xv.ctypes.data, out.ctypes.data, nvec))
        return out

    def synth_normal_dev(self, seed: int, out, mean: float = 0.0, std: float = 1.0) -> None:
        """Fill a float32 CUDA tensor with seeded N(mean, std^2) values."""
        _check(lib().hc_synth_normal_dev(self.handle, seed & (2**64 - 1), out.numel(), mean, std,
                                         ctypes.c_void_p(_tptr(out))))

    def quantize_dev(self, ggml_type: int, x, out) -> None:
        """Quantize a float32 CUDA tensor into GGUF blocks (uint8 CUDA tensor) on the device."""
        _check(lib().hc_quantize_dev(self.handle, ggml_type, ctypes.c_void_p(_tptr(x)), x.numel(),
                                     ctypes.c_void_p(_tptr(out))))

    def synth_weights(self, ggml_type: int, m: int, n: int, seed: int, std: float = 0.02,
                      scratch=None) -> ResidentWeights:
        """Seeded N(0, std^2) weights quantized on the device and made resident (bench data)."""
        import torch

        qk, bs = BLOCK[ggml_type]
        f = scratch if scratch is not None and scratch.numel() >= m * n else torch.empty(
            m * n, dtype=torch.float32, device=f"cuda:{self.device}")
        f = f[:m * n]
        q = torch.empty(m * n // qk * bs, dtype=torch.uint8, device=f"cuda:{self.device}")
        self.synth_normal_dev(seed, f, 0.0, std)
        self.quantize_dev(ggml_type, f, q)
        rw = self.upload_from_device(ggml_type, m, n, q)
        del q
        return rw

    def router_scores_dev(self, router_w, x, scores, n_tok: int) -> None:
        E, D = router_w.shape
        _check(lib().hc_router_scores_dev(self.handle, ctypes.c_void_p(_tptr(router_w)), E, D,
                                          ctypes.c_void_p(_tptr(x)), n_tok, ctypes.c_void_p(_tptr(scores))))

    def route_experts_dev(self, scores, ids, weights, top_k: int, bias=None, n_group: int = 0,
                          topk_group: int = 0, gating: int = 0, norm_topk_prob: bool = False,
                          routed_scaling_factor: float = 1.0) -> None:
        T, E = scores.shape
        _check(lib().hc_route_experts_dev(self.handle, ctypes.c_void_p(_tptr(scores)), ctypes.c_void_p(_tptr(bias)),
                                          T, E, top_k, n_group, topk_group, gating, int(norm_topk_prob),
                                          routed_scaling_factor, ctypes.c_void_p(_tptr(ids)),
                                          ctypes.c_void_p(_tptr(weights))))

    def moe_ffn_dev(self, router_w, top_k: int, gates, ups, downs, x, y, ids=None, weights=None,
                    norm_topk_prob: bool = False, routed_scaling_factor: float = 1.0) -> None:
        E = router_w.shape[0]
        n_tok = x.shape[0]
        _check(lib().hc_moe_ffn_dev(self.handle, ctypes.c_void_p(_tptr(router_w)), E, top_k, int(norm_topk_prob),
                                    routed_scaling_factor, _handles(gates), _handles(ups), _handles(downs),
                                    ctypes.c_void_p(_tptr(x)), n_tok, ctypes.c_void_p(_tptr(y)),
                                    ctypes.c_void_p(_tptr(ids)), ctypes.c_void_p(_tptr(weights))))

    def moe_ffn_ep_dev(self, router_w, top_k: int, gates, ups, downs, expert_lo: int, x, y, ids=None, weights=None,
                       norm_topk_prob: bool = False, routed_scaling_factor: float = 1.0) -> None:
        """Expert-parallel MoE: this rank holds experts [expert_lo, expert_lo + len(gates)); collective."""
        E = router_w.shape[0]
        n_tok = x.shape[0]
        _check(lib().hc_moe_ffn_ep_dev(self.handle, ctypes.c_void_p(_tptr(router_w)), E, top_k, int(norm_topk_prob),
                                       routed_scaling_factor, _handles(gates), _handles(ups), _handles(downs),
                                       expert_lo, len(gates), ctypes.c_void_p(_tptr(x)), n_tok,
                                       ctypes.c_void_p(_tptr(y)), ctypes.c_void_p(_tptr(ids)),
                                       ctypes.c_void_p(_tptr(weights))))

    def moe_stack_dev(self, routers, top_k: int, gates, ups, downs, x, expert_lo: int = 0, ep: bool = False,
                      norm_topk_prob: bool = False, routed_scaling_factor: float = 1.0) -> None:
        """x <- x + MoE_l(x) for every layer, in place (one graph launch).  routers: per-layer
        [E][d_model] CUDA tensors; gates/ups/downs: per-layer lists of the experts held here
        (all E, or [expert_lo, expert_lo + n) with ep=True, collective)."""
        L = len(routers)
        E = routers[0].shape[0]
        n = len(gates[0])
        flat = lambda ws: _handles([w for layer in ws for w in layer])  # noqa: E731
        rp = (ctypes.c_void_p * L)(*[_tptr(r) for r in routers])
        n_tok = x.shape[0]
        if ep:
            _check(lib().hc_moe_stack_ep_dev(self.handle, L, rp, E, top_k, int(norm_topk_prob), routed_scaling_factor,
                                             flat(gates), flat(ups), flat(downs), expert_lo, n,
                                             ctypes.c_void_p(_tptr(x)), n_tok))
        else:
            _check(lib().hc_moe_stack_dev(self.handle, L, rp, E, top_k, int(norm_topk_prob), routed_scaling_factor,
                                          flat(gates), flat(ups), flat(downs), ctypes.c_void_p(_tptr(x)), n_tok))


# ---------------------------------------------------------------------------- QuantMatrix
@dataclass
class QuantMatrix:
    """GGUF-layout matrix (quant.rs:31-37): ``ncols`` contiguous, y[nrows] = W x[ncols].

    ``data`` holds the GGUF bytes: an owned copy (``owned``), or a view of the caller's buffer
    (``view``, quant.rs:97-117: the caller keeps the buffer alive, no copy is made).  The GEMV
    runs on the GPU through ``hayai_b200.orchestrator.EngineOrchestrator``; there is no host
    GEMV in this backend."""
    name: str
    ncols: int
    nrows: int
    ggml_type: int
    data: np.ndarray

    def __post_init__(self):
        if self.ggml_type not in BLOCK:  # no kernel for it: the GEMV raises, not the constructor
            return
        qk, bs = BLOCK[self.ggml_type]
        if self.ncols % qk:
            raise CudaError(_lib.HC_ERR_INVALID, f"'{self.name}': ncols {self.ncols} is not a multiple of {qk}")
        need = self.nrows * (self.ncols // qk) * bs
        if self.data.nbytes < need:
            raise CudaError(_lib.HC_ERR_INVALID, f"'{self.name}': {self.data.nbytes} bytes, {need} needed")

    @classmethod
    def owned(cls, name: str, ncols: int, nrows: int, ggml_type: int, data) -> "QuantMatrix":
        return cls(name, ncols, nrows, ggml_type, np.array(_u8(data), copy=True))

    @classmethod
    def view(cls, name: str, ncols: int, nrows: int, ggml_type: int, data) -> "QuantMatrix":
        return cls(name, ncols, nrows, ggml_type, _u8(data))


def __getattr__(name):  # the orchestrator mirror moved to hayai_b200.orchestrator
    if name == "EngineOrchestrator":
        from .orchestrator import EngineOrchestrator

        return EngineOrchestrator
    raise AttributeError(name)
