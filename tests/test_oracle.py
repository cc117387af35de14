"""CPU tests of the oracle against the reference's own known-answer tests and an
independent decoder.  These pin the oracle before it is trusted as the GPU checker.

Pins (reference file:line):
  * q4k.rs:283-350   empty_ok, block_roundtrip_finite, f16_roundtrip, q4k_quantize_roundtrip_error_small
  * matmul.rs:104-136 q4_matches_fp32_reference, q4_smollm_ffn_shape_smoke
  * main.rs:648-696  `hayai validate` (LUT-Q4 vs dense FP32 < 1e-4)
  * moe_infer.rs:1010-1120 routing KATs
  * gguf-py 0.19.0 (third-party GGUF decoder shipped in this image): dequantization of every
    format must agree bit-for-bit with the oracle's block decoders.
"""
import numpy as np
import pytest

import oracle
from tests.helpers import BLOCK_TYPES, ELEM_TYPES, IQ_TYPES, quantized

LUT = np.array([-0.5, -0.4, -0.3, -0.2, -0.1, 0.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0],
               dtype=np.float32)


# ----------------------------------------------------------------------------- q4k.rs tests
def test_q4k_empty_ok():
    assert oracle.dequant(oracle.Q4_K, np.zeros(0, np.uint8), 0).size == 0


def test_q4k_block_roundtrip_finite():
    block = np.zeros(144, np.uint8)
    block[0], block[1] = 0x00, 0x3C  # d = 1.0
    block[4:16] = 1
    block[16:144] = 0x11
    y = oracle.dequant(oracle.Q4_K, block, 256)
    assert np.all(np.isfinite(y))


@pytest.mark.parametrize("v", [0.0, 1.0, -1.0, 0.5, 123.45, 0.0001, -9876.5, 1.2345])
def test_f16_roundtrip(v):
    back = oracle.f16_to_f32(oracle.f32_to_f16(v))
    assert abs(v - back) < 0.01 * max(abs(v), 1e-3)


def test_f16_decoder_matches_ieee():
    for h in [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x7C00, 0xFC00, 0x3555, 0xC000]:
        ref = np.frombuffer(np.uint16(h).tobytes(), np.float16)[0].astype(np.float32)
        assert np.float32(oracle.f16_to_f32(h)).tobytes() == ref.tobytes()


def test_q4k_quantize_roundtrip_error_small():
    j = np.arange(256, dtype=np.float32)
    blocks = [(j - 128.0) * 0.01, (j % 17) * 0.5 - 4.0, np.sin(j) * 3.0, np.where(j % 2 == 0, 1.0, -1.0)]
    x = np.concatenate(blocks).astype(np.float32)
    back = oracle.dequant(oracle.Q4_K, oracle.quantize(oracle.Q4_K, x), x.size)
    range_rel = np.abs(x - back).max() / max(float(x.max()) - float(x.min()), 1e-6)
    assert range_rel < 0.2


def test_q4k_zero_padding_is_exact():
    # SmolLM's K=576 is stored zero-padded to 768: an all-zero sub-block quantizes to 0.
    x = oracle.normal(7, 1536 * 576, 0.0, 0.02).reshape(1536, 576)
    xp = np.zeros((1536, 768), np.float32)
    xp[:, :576] = x
    back = oracle.dequant(oracle.Q4_K, oracle.quantize(oracle.Q4_K, xp), xp.size).reshape(1536, 768)
    assert np.all(back[:, 576:] == 0.0)


# ----------------------------------------------------------------------------- matmul.rs / main.rs
def test_lut_matches_fp32_reference():
    m, n = 32, 64
    w = (np.arange(m * n // 2) % 256).astype(np.uint8)
    x = (np.arange(n, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    dense = np.empty((m, n), np.float32)
    dense[:, 0::2] = LUT[w.reshape(m, n // 2) & 15]
    dense[:, 1::2] = LUT[w.reshape(m, n // 2) >> 4]
    ref = oracle.fp32_matmul(m, n, dense, x)
    got = oracle.lut_matmul_q4(m, n, w, LUT, x)
    assert np.abs(ref - got).max() < 1e-4


def test_lut_smollm_shape_smoke():
    m, n = 96, 64
    out = oracle.lut_matmul_q4(m, n, np.full(m * n // 2, 0xAB, np.uint8), LUT, np.ones(n, np.float32))
    assert np.all(np.isfinite(out))


def test_cli_validate():
    m, n = 128, 256
    w = ((np.arange(m * n // 2) * 31) % 256).astype(np.uint8)
    x = (np.arange(n, dtype=np.float32) * np.float32(0.01) - np.float32(0.25)).astype(np.float32)
    dense = np.empty((m, n), np.float32)
    dense[:, 0::2] = LUT[w.reshape(m, n // 2) & 15]
    dense[:, 1::2] = LUT[w.reshape(m, n // 2) >> 4]
    assert np.abs(oracle.fp32_matmul(m, n, dense, x) - oracle.lut_matmul_q4(m, n, w, LUT, x)).max() < 1e-4


# ----------------------------------------------------------------------------- rms_norm
def test_rms_norm_matches_formula():
    x = oracle.normal(21, 1000)  # not a multiple of 8: exercises the scalar tail
    w = oracle.normal(22, 1000, 1.0, 0.1)
    ref = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-5) * w
    got = oracle.rms_norm(x, w, 1e-5)
    assert np.abs(got - ref).max() < 1e-5
    assert np.allclose(oracle.rms_norm(np.array([3, 4], np.float32), np.ones(2, np.float32), 0.0),
                       [3 / np.sqrt(12.5), 4 / np.sqrt(12.5)], rtol=1e-6)


# ----------------------------------------------------------------------------- moe_infer.rs tests
def test_top_k_picks_highest_scores():
    s = np.array([0.1, 0.9, 0.5, -0.2, 0.7], np.float32)
    assert list(oracle.route_experts(s, 2)[0]) == [1, 4]
    assert list(oracle.route_experts(s, 10)[0]) == [1, 4, 2, 0, 3]
    assert list(oracle.route_experts(s, 0)[0]) == [1]


def test_route_softmax_topk_uses_full_softmax():
    s = np.array([0.1, 0.9, 0.3, 0.7, 0.2], np.float32)
    top, w = oracle.route_experts(s, 2)
    assert list(top) == [1, 3]
    exps = np.exp(s - np.float32(0.9)).astype(np.float32)
    tot = exps.sum(dtype=np.float32)
    assert abs(w[0] - exps[1] / tot) < 1e-5 and abs(w[1] - exps[3] / tot) < 1e-5
    assert w.sum() < 1.0


def test_route_norm_topk_prob_renormalizes():
    _, w = oracle.route_experts(np.array([0.1, 0.9, 0.3, 0.7, 0.2], np.float32), 2, norm_topk_prob=True)
    assert abs(w.sum() - 1.0) < 1e-5


def test_route_correction_bias_selects_but_weights_raw_scores():
    s = np.array([1.0, 0.5, 0.0, -1.0], np.float32)
    top, w = oracle.route_experts(s, 1, bias=np.array([0.0, 10.0, 0.0, 0.0], np.float32))
    assert list(top) == [1]
    exps = np.exp(s)
    assert abs(w[0] - exps[1] / exps.sum()) < 1e-5


def test_route_grouped_selects_within_kept_groups():
    top, _ = oracle.route_experts(np.array([0.6, 0.5, 0.9, 0.1], np.float32), 1, n_group=2, topk_group=1, gating=1)
    assert list(top) == [0]


def test_route_sigmoid_and_scaling():
    top, w = oracle.route_experts(np.array([0.0, 1.0, -1.0], np.float32), 2, gating=1, routed_scaling_factor=2.0)
    assert list(top) == [1, 0]
    assert abs(w[0] - 2.0 * 0.7310586) < 1e-4 and abs(w[1] - 1.0) < 1e-4


def test_route_ties_keep_lower_expert_id():
    top, _ = oracle.route_experts(np.array([0.5, 0.7, 0.7, 0.1, 0.7], np.float32), 3)
    assert list(top) == [1, 2, 4]


# ----------------------------------------------------------------------------- independent decoder
@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, *IQ_TYPES, *BLOCK_TYPES])
def test_dequant_matches_gguf_py(t):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize

    qtype = gguf.GGMLQuantizationType(t)  # the GGML type ids are the same numbers
    qk, bs = oracle.BLOCK[t]
    m, n = 8, 1024
    w = quantized(t, m, n, seed=100 + t)
    ref = dequantize(w.reshape(-1, bs), qtype).reshape(-1).astype(np.float32)
    got = oracle.dequant(t, w, m * n)
    assert np.array_equal(ref, got)


@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, *IQ_TYPES, *BLOCK_TYPES, *ELEM_TYPES])
def test_gemv_matches_dequant_dot(t):
    m, n = 48, 1024
    w = quantized(t, m, n, seed=200 + t)
    x = oracle.normal(300 + t, n)
    dense = oracle.dequant(t, w, m * n).reshape(m, n).astype(np.float64)
    ref = dense @ x.astype(np.float64)
    got = oracle.gemv(t, m, n, w, x)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel < 1e-5


def test_gemv_thread_count_invariant():
    m, n = 64, 2048
    w = quantized(oracle.Q4_K, m, n, 11)
    x = oracle.normal(12, n)
    old = oracle.get_threads()
    oracle.set_threads(1)
    a = oracle.gemv(oracle.Q4_K, m, n, w, x)
    oracle.set_threads(max(old, 2))
    b = oracle.gemv(oracle.Q4_K, m, n, w, x)
    oracle.set_threads(old)
    assert np.array_equal(a, b)


def test_rng_is_seeded_and_normal():
    a = oracle.normal(5, 100000)
    assert np.array_equal(a, oracle.normal(5, 100000))
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1.0) < 0.02


def test_golden_vectors():
    """Committed golden vectors (tests/golden/make_golden.py) still reproduce."""
    import os

    path = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
    g = np.load(path)
    for key in [k for k in g.files if k.endswith("_w")]:
        name = key[:-2]
        t, m, n = (int(v) for v in g[name + "_meta"])
        got = oracle.gemv(t, m, n, g[name + "_w"], g[name + "_x"])
        assert np.array_equal(got, g[name + "_y"]), name


def test_golden_vectors_match_independent_decoder():
    import os

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    for key in [k for k in g.files if k.endswith("_y64")]:
        name = key[:-4]
        y, y64 = g[name + "_y"].astype(np.float64), g[key]
        assert np.linalg.norm(y - y64) / np.linalg.norm(y64) < 1e-5, name


def test_dequant_matches_gguf_py_on_arbitrary_blocks():
    """Any bytes are a valid block of these formats (scales and codes are bit fields): the
    oracle's decoders agree with gguf-py bit for bit on arbitrary blocks, not only on the seeded
    ones.  Blocks whose f16 scales are inf/NaN are skipped (both sides give non-finite values)."""
    gguf = pytest.importorskip("gguf")
    hyp = pytest.importorskip("hypothesis")
    from gguf.quants import dequantize
    from hypothesis import given, settings
    from hypothesis import strategies as st

    types = [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, *IQ_TYPES, *BLOCK_TYPES]

    @settings(max_examples=200, deadline=None)
    @given(t=st.sampled_from(types), data=st.data())
    def check(t, data):
        qk, bs = oracle.BLOCK[t]
        nblk = data.draw(st.integers(1, 4))
        raw = np.frombuffer(data.draw(st.binary(min_size=nblk * bs, max_size=nblk * bs)), np.uint8).copy()
        with np.errstate(all="ignore"):
            ref = dequantize(raw.reshape(-1, bs), gguf.GGMLQuantizationType(t)).reshape(-1).astype(np.float32)
        if not np.isfinite(ref).all():
            return
        got = oracle.dequant(t, raw, nblk * qk)
        assert np.array_equal(ref, got), t

    assert hyp is not None
    check()


def test_q8_1_and_q8_k_known_answers():
    # quant.rs:743-770 (q8_1_and_q8_k_gemv): d = 1, all codes 1, x = 1
    b = np.frombuffer(bytes([0x00, 0x3C, 0, 0]) + bytes([1] * 32), np.uint8)
    assert abs(oracle.gemv(oracle.Q8_1, 1, 32, b, np.ones(32, np.float32))[0] - 32.0) < 1e-3
    b = np.frombuffer(np.float32(1.0).tobytes() + bytes([1] * 256) + bytes(32), np.uint8)
    assert abs(oracle.gemv(oracle.Q8_K, 1, 256, b, np.ones(256, np.float32))[0] - 256.0) < 1e-3
    d = oracle.dequant(oracle.Q8_K, b, 256)
    assert d.size == 256 and abs(d[0] - 1.0) < 1e-6


@pytest.mark.parametrize("t", [oracle.F16, oracle.BF16])
def test_half_decoders_match_gguf_py(t):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize

    w = quantized(t, 8, 1024, seed=100 + t)
    raw = w.view(np.uint16).reshape(8, 1024) if t == oracle.F16 else w.reshape(8, 2048)  # gguf-py's own input forms
    ref = dequantize(raw, gguf.GGMLQuantizationType(t)).reshape(-1).astype(np.float32)
    assert np.array_equal(ref, oracle.dequant(t, w, 8 * 1024))


@pytest.mark.parametrize("t", [oracle.Q8_1, oracle.Q8_K])
def test_q8_1_q8_k_decoders_match_numpy(t):
    """gguf-py has no decoder for these two; numpy's own int8 and f16/f32 views are the check
    ({f16 d, f16 s, int8 qs[32]} and {f32 d, int8 qs[256], int16 bsums[16]})."""
    qk, bs = oracle.BLOCK[t]
    w = quantized(t, 4, 1024, seed=7 + t)
    blk = w.reshape(-1, bs)
    d = (blk[:, 0:2].copy().view(np.float16).astype(np.float32) if t == oracle.Q8_1
         else blk[:, 0:4].copy().view(np.float32))
    q = blk[:, 4:4 + qk].view(np.int8).astype(np.float32)
    assert np.array_equal((q * d).reshape(-1), oracle.dequant(t, w, 4 * 1024))
