"""GPU parity of the GEMV kernels against the oracle, through the C ABI.

Tolerance (the parity contract): rel-L2 <= 1e-4 and max-abs <= 1e-3 on FP32 outputs.
Fixtures include the reference's own OpenCL parity patterns
(crates/hayai-opencl/src/compute.rs:1034-1245, 1370-1496, 1648-1670).
"""
import numpy as np
import pytest
import torch

import hayai_b200 as hb
import oracle
from tests.helpers import BLOCK_TYPES, ELEM_TYPES, IQ_TYPES, MAX_ABS, REL_L2, assert_parity, quantized

pytestmark = pytest.mark.gpu

ALL = [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, oracle.F32, *IQ_TYPES, *BLOCK_TYPES]
LUT = np.array([-0.5, -0.4, -0.3, -0.2, -0.1, 0.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0], np.float32)


@pytest.mark.parametrize("t", ALL)
@pytest.mark.parametrize("m,n", [(32, 256), (100, 1024), (576, 1536), (1536, 768), (8, 4096)])
def test_gemv_seeded(engine, t, m, n):
    w = quantized(t, m, n, seed=1000 * t + m + n)
    x = oracle.normal(7 + m + n, n)
    ref = oracle.gemv(t, m, n, w, x)
    got = engine.ggml_gemv_dispatch(t, m, n, w, x)
    assert_parity(ref, got, what=f"{hb.TYPE_LABELS[t]} {m}x{n}")


def test_q8_0_k_not_multiple_of_128(engine):
    m, n = 64, 32 * 7  # 7 blocks: the GPU layout pads the last group of 4
    w = quantized(oracle.Q8_0, m, n, 5)
    x = oracle.normal(6, n)
    assert_parity(oracle.gemv(oracle.Q8_0, m, n, w, x), engine.ggml_gemv_q8_0(m, n, w, x))


def test_reference_q4_k_fixture(engine):
    m, n = 32, 256
    w = np.zeros((m, 144), np.uint8)
    for row in range(m):
        w[row, 0:2] = [0x00, 0x3C]
        w[row, 4:16] = 1
        w[row, 16:144] = (row + np.arange(16, 144)) % 256
    x = (np.arange(n, dtype=np.float32) * np.float32(0.005) - np.float32(0.2)).astype(np.float32)
    ref = oracle.gemv(oracle.Q4_K, m, n, w, x)
    assert np.abs(ref - engine.ggml_gemv_q4_k(m, n, w, x)).max() < 1e-3


def test_reference_q6_k_fixture(engine):
    m, n = 32, 256
    w = np.zeros((m, 210), np.uint8)
    for row in range(m):
        w[row, 0:128] = (row + np.arange(128)) % 256
        w[row, 128:192] = (row * 3 + np.arange(128, 192)) % 256
        w[row, 192:208] = 1
        w[row, 208:210] = [0x00, 0x3C]
    x = (np.arange(n, dtype=np.float32) * np.float32(0.005) - np.float32(0.2)).astype(np.float32)
    ref = oracle.gemv(oracle.Q6_K, m, n, w, x)
    assert np.abs(ref - engine.ggml_gemv_q6_k(m, n, w, x)).max() < 1e-3


def test_reference_q8_0_fixture(engine):
    m, n = 32, 256
    w = np.zeros((m, 8, 34), np.uint8)
    for row in range(m):
        for b in range(8):
            w[row, b, 0:2] = [0x66, 0x2E]
            w[row, b, 2:34] = (row + b + np.arange(32)) % 256
    x = (np.arange(n, dtype=np.float32) * np.float32(0.01) - np.float32(0.4)).astype(np.float32)
    ref = oracle.gemv(oracle.Q8_0, m, n, w, x)
    assert np.abs(ref - engine.ggml_gemv_q8_0(m, n, w, x)).max() < 1e-3


@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, *IQ_TYPES, *BLOCK_TYPES])
def test_reference_gemv_parity_pattern(engine, t):
    # gemv_parity (compute.rs:1370-1396): bytes (i*131+17)&0x1F, input i*0.003-0.2, m32 n256
    m, n = 32, 256
    nbytes = m * hb.row_bytes(t, n)
    w = ((np.arange(nbytes) * 131 + 17) & 0x1F).astype(np.uint8)
    x = (np.arange(n, dtype=np.float32) * np.float32(0.003) - np.float32(0.2)).astype(np.float32)
    ref = oracle.gemv(t, m, n, w, x)
    got = engine.ggml_gemv_dispatch(t, m, n, w, x)
    assert np.abs(ref - got).max() < 1e-3


def test_reference_batched_q4_k(engine):
    # compute.rs:1648-1670
    m, n, batch = 32, 256, 3
    w = ((np.arange(m * 144) * 131 + 17) & 0x1F).astype(np.uint8)
    inputs = (np.arange(batch * n, dtype=np.float32) * np.float32(0.003) - np.float32(0.2)).astype(np.float32)
    outputs = np.zeros(batch * m, np.float32)
    engine.ggml_gemv_batched_q4_k(m, n, w, inputs, outputs, batch)
    expected = np.concatenate([oracle.gemv(oracle.Q4_K, m, n, w, inputs[b * n:(b + 1) * n]) for b in range(batch)])
    assert np.abs(expected - outputs).max() < 1e-3


@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, oracle.IQ2_S, oracle.F32, oracle.Q5_0,
                               oracle.Q3_K, oracle.IQ4_XS])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8])
def test_batched_all_types(engine, t, batch):
    m, n = 80, 1024
    w = quantized(t, m, n, seed=31 + t)
    xs = oracle.normal(32 + batch, batch * n)
    rw = engine.upload(t, m, n, w)
    got = engine.ggml_gemv_batched(rw, xs, batch)
    ref = np.concatenate([oracle.gemv(t, m, n, w, xs[b * n:(b + 1) * n]) for b in range(batch)])
    assert_parity(ref, got, what=f"{hb.TYPE_LABELS[t]} batch {batch}")


@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0])
def test_dispatch_bound_dev_async_agree(engine, t):
    m, n = 256, 2048
    w = quantized(t, m, n, seed=77)
    x = oracle.normal(78, n)
    a = engine.ggml_gemv_dispatch(t, m, n, w, x)
    rw = engine.upload(t, m, n, w)
    b = engine.ggml_gemv_dispatch_bound(rw, x)
    c = engine.ggml_gemv_async(rw, x).wait()
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(m, device="cuda")
    engine.set_stream(torch.cuda.current_stream())
    engine.gemv_dev(rw, xd, yd)
    torch.cuda.synchronize()
    engine.set_stream(None)
    d = yd.cpu().numpy()
    assert np.array_equal(a, b) and np.array_equal(b, c) and np.array_equal(c, d)


def test_gemv_dev_residual(engine):
    m, n = 512, 1024
    w = quantized(oracle.Q4_K, m, n, 3)
    x = oracle.normal(4, n)
    r = oracle.normal(5, m)
    rw = engine.upload(oracle.Q4_K, m, n, w)
    xd, rd = torch.from_numpy(x).cuda(), torch.from_numpy(r).cuda()
    yd = torch.empty(m, device="cuda")
    engine.set_stream(torch.cuda.current_stream())
    engine.gemv_dev(rw, xd, yd, resid=rd)
    torch.cuda.synchronize()
    engine.set_stream(None)
    assert_parity(oracle.gemv(oracle.Q4_K, m, n, w, x) + r, yd.cpu().numpy())


def test_upload_from_device_matches_host_upload(engine):
    m, n = 128, 512
    w = quantized(oracle.Q6_K, m, n, 9)
    x = oracle.normal(10, n)
    a = engine.ggml_gemv_dispatch_bound(engine.upload(oracle.Q6_K, m, n, w), x)
    b = engine.ggml_gemv_dispatch_bound(engine.upload_from_device(oracle.Q6_K, m, n, torch.from_numpy(w).cuda()), x)
    assert np.array_equal(a, b)


def test_lut_reference_fixture(engine):
    # compute.rs:1034-1061
    m, n = 64, 128
    w = ((np.arange(m * n // 2) * 17) % 256).astype(np.uint8)
    x = (np.arange(n, dtype=np.float32) * np.float32(0.01) - np.float32(0.5)).astype(np.float32)
    assert np.abs(oracle.lut_matmul_q4(m, n, w, LUT, x) - engine.lut_matmul_q4(m, n, w, LUT, x)).max() < 1e-4


def test_lut_bench_and_validate_workloads(engine):
    m, n = 1536, 576  # `hayai bench` (main.rs:601-646): outputs ~317, where the oracle's own
    # sequential f32 sum drifts ~9e-4 from the exact 316.8, so the contract tolerance applies
    w = np.full(m * n // 2, 0xAB, np.uint8)
    x = np.ones(n, np.float32)
    got = engine.lut_matmul_q4(m, n, w, LUT, x)
    assert_parity(oracle.lut_matmul_q4(m, n, w, LUT, x), got, what="lut bench")
    assert np.abs(got - 316.8).max() < 1e-3
    m, n = 128, 256  # `hayai validate` (main.rs:648-696)
    w = ((np.arange(m * n // 2) * 31) % 256).astype(np.uint8)
    x = (np.arange(n, dtype=np.float32) * np.float32(0.01) - np.float32(0.25)).astype(np.float32)
    assert np.abs(oracle.lut_matmul_q4(m, n, w, LUT, x) - engine.lut_matmul_q4(m, n, w, LUT, x)).max() < 1e-4


def test_invalid_shapes_rejected(engine):
    with pytest.raises(hb.CudaError) as e:
        engine.ggml_gemv_dispatch(oracle.Q4_K, 4, 576, np.zeros(4 * 3 * 144, np.uint8), np.zeros(576, np.float32))
    assert e.value.code == 1
    with pytest.raises(hb.CudaError) as e:
        engine.ggml_gemv_dispatch(oracle.Q4_K, 4, 256, np.zeros(3 * 144, np.uint8), np.zeros(256, np.float32))
    assert "weight buffer" in str(e.value)
    with pytest.raises(hb.CudaError) as e:
        engine.ggml_gemv_dispatch(19, 4, 256, np.zeros(4 * 144, np.uint8), np.zeros(256, np.float32))  # IQ1_S
    assert e.value.code == 2


def test_activation_out_of_f16_range_is_reported(engine):
    m, n = 16, 256
    w = quantized(oracle.Q4_K, m, n, 1)
    x = np.zeros(n, np.float32)
    x[3] = 1e6
    with pytest.raises(hb.CudaError) as e:
        engine.ggml_gemv_q4_k(m, n, w, x)
    assert e.value.code == 4
    # the engine stays usable and the flag is cleared
    x[3] = 1.0
    assert_parity(oracle.gemv(oracle.Q4_K, m, n, w, x), engine.ggml_gemv_q4_k(m, n, w, x))


def test_zero_and_tiny_inputs(engine):
    m, n = 64, 512
    w = quantized(oracle.Q4_K, m, n, 2)
    assert np.all(engine.ggml_gemv_q4_k(m, n, w, np.zeros(n, np.float32)) == 0.0)
    x = oracle.normal(3, n) * np.float32(1e-6)
    assert_parity(oracle.gemv(oracle.Q4_K, m, n, w, x), engine.ggml_gemv_q4_k(m, n, w, x), abs_tol=MAX_ABS,
                  rel_tol=REL_L2)


def test_deterministic(engine):
    m, n = 4096, 4096
    w = quantized(oracle.Q4_K, m, n, 12)
    rw = engine.upload(oracle.Q4_K, m, n, w)
    x = oracle.normal(13, n)
    a = engine.ggml_gemv_dispatch_bound(rw, x)
    b = engine.ggml_gemv_dispatch_bound(rw, x)
    assert np.array_equal(a, b)


# ---------------------------------------------------------------- Q8_0 batches (9+) on tcgen05
@pytest.mark.parametrize("batch,m,n", [
    (9, 128, 1024),      # smallest Q8_0 tensor-core batch: rows padded to 16 in the MMA's N
    (13, 256, 2048),     # ragged batch
    (64, 512, 4096),     # config-3 batch, units split over several CTAs
    (100, 128, 14336),   # long K (Llama-3-8B down), N = 208 (one accumulator set)
    (128, 256, 1024),    # largest batch, N = 256
])
def test_q8_0_tensor_core_batches(engine, batch, m, n):
    t = oracle.Q8_0
    w = quantized(t, m, n, seed=71 + batch)
    xs = oracle.normal(72 + batch, batch * n)
    rw = engine.upload(t, m, n, w)
    got = engine.ggml_gemv_batched(rw, xs, batch)
    ref = np.concatenate([oracle.gemv(t, m, n, w, xs[b * n:(b + 1) * n]) for b in range(batch)])
    assert_parity(ref, got, what=f"q8_0 tensor-core batch {batch} {m}x{n}")
    again = engine.ggml_gemv_batched(rw, xs, batch)
    assert np.array_equal(got, again)


def test_q8_0_tensor_core_residual_dev(engine):
    import torch

    m, n, batch = 384, 1024, 24
    w = quantized(oracle.Q8_0, m, n, seed=91)
    xs = oracle.normal(92, batch * n).reshape(batch, n)
    rs = oracle.normal(93, batch * m).reshape(batch, m)
    rw = engine.upload(oracle.Q8_0, m, n, w)
    X, R = torch.from_numpy(xs).cuda(), torch.from_numpy(rs).cuda()
    Y = torch.empty(batch, m, device="cuda")
    engine.set_stream(torch.cuda.current_stream())
    try:
        engine.gemv_dev(rw, X, Y, resid=R, nvec=batch)
        torch.cuda.synchronize()
    finally:
        engine.set_stream(None)
    ref = np.stack([oracle.gemv(oracle.Q8_0, m, n, w, xs[b]) + rs[b] for b in range(batch)])
    assert_parity(ref, Y.cpu().numpy(), what="q8_0 tensor-core + residual")


# ---------------------------------------------------------------- Q4_K / Q6_K batches on tcgen05
@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K])
@pytest.mark.parametrize("batch,m,n", [
    (8, 128, 1024),      # smallest tensor-core batch
    (13, 256, 2048),     # ragged batch: rows padded to 16 in the MMA's N
    (16, 384, 8192),     # config-5 batch (70B d_model), several K splits
    (64, 128, 14336),    # Llama-3-8B down length, deep K split
    (33, 256, 4096),     # N = 80: one accumulator set pair beside the TMEM operand buffers
    (100, 128, 4096),    # N = 208: operands in shared memory (the TMEM form holds N <= 128)
])
def test_kquant_tensor_core_batches(engine, t, batch, m, n):
    w = quantized(t, m, n, seed=171 + batch)
    xs = oracle.normal(172 + batch, batch * n)
    rw = engine.upload(t, m, n, w)
    got = engine.ggml_gemv_batched(rw, xs, batch)
    ref = np.concatenate([oracle.gemv(t, m, n, w, xs[b * n:(b + 1) * n]) for b in range(batch)])
    assert_parity(ref, got, what=f"{hb.TYPE_LABELS[t]} tensor-core batch {batch} {m}x{n}")
    again = engine.ggml_gemv_batched(rw, xs, batch)
    assert np.array_equal(got, again)


@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K])
def test_kquant_tensor_core_reference_pattern(engine, t):
    """The byte pattern of gemv_parity (compute.rs:1370-1396) at a tensor-core shape (128 rows,
    batch 8).  Its Q6_K outputs reach |y| ~ 2300, where f32 summation order alone moves a
    result by more than 1e-3 (the sequential f32 oracle is 3e-4 from the exact f64 value), so
    besides rel-L2 <= 1e-4 against the oracle, each element is checked against the exact f64
    product: |y - exact| <= 1e-3 + 2^-18 * sum_k |w_k x_k| (a few dozen f32 roundings of the
    dot product's own scale)."""
    m, n, batch = 128, 256, 8
    w = ((np.arange(m * hb.row_bytes(t, n)) * 131 + 17) & 0x1F).astype(np.uint8)
    xs = (np.arange(batch * n, dtype=np.float32) * np.float32(0.003) - np.float32(0.2)).astype(np.float32)
    rw = engine.upload(t, m, n, w)
    got = engine.ggml_gemv_batched(rw, xs, batch)
    ref = np.concatenate([oracle.gemv(t, m, n, w, xs[b * n:(b + 1) * n]) for b in range(batch)])
    assert_parity(ref, got, abs_tol=np.inf, what=f"{hb.TYPE_LABELS[t]} pattern batch {batch}")
    W = oracle.dequant(t, w, m * n).reshape(m, n).astype(np.float64)
    X = xs.reshape(batch, n).astype(np.float64)
    exact = (X @ W.T).reshape(-1)
    scale = (np.abs(X) @ np.abs(W).T).reshape(-1)
    assert np.all(np.abs(got - exact) <= 1e-3 + scale * 2.0 ** -18)


def test_golden_fixtures_on_gpu(engine):
    """The committed golden vectors (tests/golden/make_golden.py): every format's CUDA GEMV
    against the oracle's pinned output and the gguf-py float64 product."""
    import os

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    names = sorted(k[:-2] for k in g.files if k.endswith("_w"))
    assert len(names) == 17
    for name in names:
        t, m, n = (int(v) for v in g[name + "_meta"])
        got = engine.ggml_gemv_dispatch(t, m, n, g[name + "_w"], g[name + "_x"])
        assert_parity(g[name + "_y"], got, what=f"golden {name}")
        assert_parity(g[name + "_y64"], got, what=f"golden {name} vs f64")


# ---------------------------------------------------------------- F16, BF16, Q8_1, Q8_K
def test_reference_f16_bf16_q8_1_q8_k_fixtures(engine):
    """compute.rs:1529-1641 (opencl_f32_f16_gemv_matches_cpu / opencl_bf16_q8_1_q8_k_match_cpu):
    the same byte patterns, inputs and tolerances, against the oracle."""
    m = 16
    # F16: raw masked bytes, input i * 0.01 - 0.3
    n = 64
    w = ((np.arange(m * n * 2) * 131 + 17) & 0x1F).astype(np.uint8)
    x = (np.arange(n, dtype=np.float32) * np.float32(0.01) - np.float32(0.3)).astype(np.float32)
    assert np.abs(oracle.gemv(oracle.F16, m, n, w, x) - engine.ggml_gemv_dispatch(oracle.F16, m, n, w, x)).max() < 1e-3
    inp = (np.arange(256, dtype=np.float32) * np.float32(0.01) - np.float32(0.7)).astype(np.float32)
    # BF16: ((i % 23) - 11) * 0.02 truncated to its upper 16 bits
    v = ((np.arange(m * n) % 23).astype(np.float32) - np.float32(11.0)) * np.float32(0.02)
    w = (v.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    got = engine.ggml_gemv_dispatch(oracle.BF16, m, n, w, inp[:n])
    assert np.abs(oracle.gemv(oracle.BF16, m, n, w, inp[:n]) - got).max() < 1e-2
    # Q8_1: d = f16 0.5, codes ((r + bi + j) % 11) - 5
    blocks = n // 32
    w = np.zeros((m, blocks, 36), np.uint8)
    w[:, :, 0:2] = np.frombuffer(np.uint16(0x3800).tobytes(), np.uint8)
    r, bi, j = np.meshgrid(np.arange(m), np.arange(blocks), np.arange(32), indexing="ij")
    w[:, :, 4:] = (((r + bi + j) % 11) - 5).astype(np.int8).view(np.uint8)
    w = w.reshape(-1)
    got = engine.ggml_gemv_dispatch(oracle.Q8_1, m, n, w, inp[:n])
    assert np.abs(oracle.gemv(oracle.Q8_1, m, n, w, inp[:n]) - got).max() < 1e-2
    # Q8_K: d = 0.013, codes ((r * 7 + j) % 13) - 6
    n = 256
    w = np.zeros((m, 292), np.uint8)
    w[:, 0:4] = np.frombuffer(np.float32(0.013).tobytes(), np.uint8)
    r, j = np.meshgrid(np.arange(m), np.arange(256), indexing="ij")
    w[:, 4:260] = (((r * 7 + j) % 13) - 6).astype(np.int8).view(np.uint8)
    w = w.reshape(-1)
    got = engine.ggml_gemv_dispatch(oracle.Q8_K, m, n, w, inp)
    assert np.abs(oracle.gemv(oracle.Q8_K, m, n, w, inp) - got).max() < 1e-2


@pytest.mark.parametrize("t", ELEM_TYPES)
@pytest.mark.parametrize("m,n", [(300, 4096), (37, 2816)])
def test_elem_types_match_oracle(engine, t, m, n):
    w = quantized(t, m, n, seed=40 + t)
    x = oracle.normal(41 + t, n)
    assert_parity(oracle.gemv(t, m, n, w, x), engine.ggml_gemv_dispatch(t, m, n, w, x), what=hb.TYPE_LABELS[t])


@pytest.mark.parametrize("t", [oracle.F16, oracle.BF16])
def test_half_rows_not_multiple_of_8(engine, t):
    # K % 8 != 0: rows are not 16-byte aligned, the kernel takes one element per lane
    m, n = 45, 1001
    w = quantized(t, m, n, seed=3)
    x = oracle.normal(4, n)
    assert_parity(oracle.gemv(t, m, n, w, x), engine.ggml_gemv_dispatch(t, m, n, w, x), what=hb.TYPE_LABELS[t])


@pytest.mark.parametrize("t", ELEM_TYPES)
def test_elem_types_batched(engine, t):
    m, n, batch = 64, 1024, 3
    w = quantized(t, m, n, seed=50 + t)
    xs = oracle.normal(51, batch * n)
    rw = engine.upload(t, m, n, w)
    got = engine.ggml_gemv_batched(rw, xs, batch)
    ref = np.concatenate([oracle.gemv(t, m, n, w, xs[b * n:(b + 1) * n]) for b in range(batch)])
    assert_parity(ref, got, what=f"{hb.TYPE_LABELS[t]} batch {batch}")
