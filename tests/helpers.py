"""Test helpers: seeded synthetic weights in every format, parity metrics."""
from __future__ import annotations

import numpy as np

import oracle

QK = {t: qk for t, (qk, _) in oracle.BLOCK.items()}
IQ_TYPES = [oracle.IQ2_XXS, oracle.IQ2_XS, oracle.IQ2_S, oracle.IQ3_XXS, oracle.IQ3_S]
# The other GGML block formats (raw GGUF rows, CUDA-core GEMV)
BLOCK_TYPES = [oracle.Q4_0, oracle.Q4_1, oracle.Q5_0, oracle.Q5_1, oracle.Q2_K, oracle.Q3_K, oracle.Q5_K,
               oracle.IQ4_NL, oracle.IQ4_XS]
# The plain element and 8-bit formats of gemv_row_bytes (compute.rs:877-907) beyond those above
ELEM_TYPES = [oracle.F16, oracle.BF16, oracle.Q8_1, oracle.Q8_K]
# typical |decoded value| / d for random codes: block scale factor x mean code or grid value
IQ_SCALE = {oracle.IQ2_XXS: 50.0, oracle.IQ2_XS: 50.0, oracle.IQ2_S: 50.0, oracle.IQ3_XXS: 120.0,
            oracle.IQ3_S: 130.0, oracle.Q4_0: 4.0, oracle.Q4_1: 4.0, oracle.Q5_0: 8.0, oracle.Q5_1: 8.0,
            oracle.Q2_K: 8.0, oracle.Q3_K: 32.0, oracle.Q5_K: 250.0, oracle.IQ4_NL: 60.0, oracle.IQ4_XS: 1000.0,
            oracle.Q8_1: 64.0}
# byte offsets of the f16 scale d inside a block
F16_AT = {oracle.Q4_K: (0, 2), oracle.Q6_K: (208,), oracle.Q8_0: (0,), oracle.IQ2_XXS: (0,), oracle.IQ2_XS: (0,),
          oracle.IQ2_S: (0,), oracle.IQ3_XXS: (0,), oracle.IQ3_S: (0,), oracle.Q4_0: (0,), oracle.Q4_1: (0,),
          oracle.Q5_0: (0,), oracle.Q5_1: (0,), oracle.Q2_K: (80,), oracle.Q3_K: (108,), oracle.Q5_K: (0,),
          oracle.IQ4_NL: (0,), oracle.IQ4_XS: (0,), oracle.Q8_1: (0,)}
# the f16 min / dmin: (byte offset, multiple of d) chosen to centre the decoded values near zero
MIN_AT = {oracle.Q4_1: (2, -7.5), oracle.Q5_1: (2, -15.5), oracle.Q2_K: (82, 1.5), oracle.Q5_K: (2, 15.5)}


def quantized(ggml_type: int, m: int, n: int, seed: int, std: float = 0.02) -> np.ndarray:
    """Seeded weights: N(0, std^2) quantized (Q4_K with the reference quantizer), or random
    valid blocks with their scales set for a realistic magnitude (~std) for the IQ formats and
    the other GGML block formats."""
    if ggml_type == oracle.F32:
        return oracle.normal(seed, m * n, 0.0, std).view(np.uint8).copy()
    if ggml_type == oracle.F16:
        return oracle.normal(seed, m * n, 0.0, std).astype(np.float16).view(np.uint8).copy()
    if ggml_type == oracle.BF16:  # the upper half of each f32 (truncation)
        return (oracle.normal(seed, m * n, 0.0, std).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).copy()
    if ggml_type == oracle.Q8_K:  # f32 d, random int8 codes and bsums
        nblk = m * n // 256
        b = oracle.random_bytes(seed, nblk * 292).reshape(nblk, 292)
        u = oracle.normal(seed ^ 0x5EED, nblk, 0.0, 1.0)
        d = (std / 64.0 * (0.5 + 0.5 * (1.0 + np.tanh(u)))).astype(np.float32)
        b[:, 0:4] = d.view(np.uint8).reshape(nblk, 4)
        return b.reshape(-1).copy()
    if ggml_type in (oracle.Q4_K, oracle.Q6_K, oracle.Q8_0):
        w = oracle.normal(seed, m * n, 0.0, std)
        return oracle.quantize(ggml_type, w)
    qk, bs = oracle.BLOCK[ggml_type]
    nblk = m * n // qk
    b = oracle.random_bytes(seed, nblk * bs).reshape(nblk, bs)
    u = oracle.normal(seed ^ 0x5EED, nblk, 0.0, 1.0)
    # d chosen so the decoded weights have a realistic magnitude (~std): a typical
    # |value| is about d * IQ_SCALE[type] for random codes
    d = (std / IQ_SCALE[ggml_type] * (0.5 + 0.5 * (1.0 + np.tanh(u)))).astype(np.float16)
    for off in F16_AT[ggml_type]:
        b[:, off:off + 2] = d.view(np.uint8).reshape(nblk, 2)
    if ggml_type in MIN_AT:
        off, ratio = MIN_AT[ggml_type]
        mn = (d.astype(np.float32) * np.float32(ratio)).astype(np.float16)
        b[:, off:off + 2] = mn.view(np.uint8).reshape(nblk, 2)
    return b.reshape(-1).copy()


def metrics(ref: np.ndarray, got: np.ndarray) -> tuple[float, float]:
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    err = got - ref
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    return rel, float(np.abs(err).max()) if err.size else 0.0


# The parity contract: rel-L2 <= 1e-4 and max-abs <= 1e-3 on FP32 outputs.
REL_L2 = 1e-4
MAX_ABS = 1e-3


def assert_parity(ref, got, rel_tol: float = REL_L2, abs_tol: float = MAX_ABS, what: str = "") -> None:
    rel, mx = metrics(ref, got)
    assert rel <= rel_tol and mx <= abs_tol, f"{what}: rel-L2 {rel:.3e} (tol {rel_tol}), max-abs {mx:.3e} (tol {abs_tol})"
