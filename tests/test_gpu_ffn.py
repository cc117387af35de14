"""GPU parity of the SwiGLU FFN block and the layer stack against the oracle (C ABI).

Shapes follow BASELINE.json: SmolLM2-135M (Q4_K x3, K=576 zero-padded to 768),
Llama-3-8B (gate/up Q4_K, down Q6_K) and the Q8_0 variant.  Tolerance: rel-L2 <= 1e-4,
max-abs <= 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_parity, quantized

pytestmark = pytest.mark.gpu


def ffn_weights(tg, td, d_model, d_ff, seed, k_in=None):
    """gate/up d_ff x k_in (rows zero-padded from d_model), down d_model x d_ff."""
    k_in = k_in or d_model
    if tg == oracle.Q4_K and k_in != d_model:
        wg32 = np.zeros((d_ff, k_in), np.float32)
        wu32 = np.zeros((d_ff, k_in), np.float32)
        wg32[:, :d_model] = oracle.normal(seed, d_ff * d_model, 0, 0.02).reshape(d_ff, d_model)
        wu32[:, :d_model] = oracle.normal(seed + 1, d_ff * d_model, 0, 0.02).reshape(d_ff, d_model)
        wg, wu = oracle.quantize(tg, wg32), oracle.quantize(tg, wu32)
    else:
        wg, wu = quantized(tg, d_ff, k_in, seed), quantized(tg, d_ff, k_in, seed + 1)
    wd = quantized(td, d_model, d_ff, seed + 2)
    return wg, wu, wd


def run_ffn(engine, tg, td, d_model, d_ff, seed, nvec=1, k_in=None):
    k_in = k_in or d_model
    wg, wu, wd = ffn_weights(tg, td, d_model, d_ff, seed, k_in)
    x = np.zeros((nvec, k_in), np.float32)
    x[:, :d_model] = oracle.normal(seed + 3, nvec * d_model).reshape(nvec, d_model)
    G, U, D = engine.upload(tg, d_ff, k_in, wg), engine.upload(tg, d_ff, k_in, wu), engine.upload(td, d_model, d_ff, wd)
    got = engine.ffn_swiglu(G, U, D, x, nvec).reshape(nvec, d_model)
    ref = np.stack([oracle.ffn_swiglu(tg, wg, tg, wu, td, wd, k_in, d_ff, d_model, x[v]) for v in range(nvec)])
    return ref, got


def test_ffn_smollm_layer(engine):
    ref, got = run_ffn(engine, oracle.Q4_K, oracle.Q4_K, 576, 1536, 100, k_in=768)
    assert_parity(ref, got, what="smollm ffn")


def test_ffn_llama8b_layer(engine):
    ref, got = run_ffn(engine, oracle.Q4_K, oracle.Q6_K, 4096, 14336, 200)
    assert_parity(ref, got, what="llama-8b ffn")


@pytest.mark.parametrize("nvec", [1, 3, 8, 16, 40])
def test_ffn_q8_0(engine, nvec):
    ref, got = run_ffn(engine, oracle.Q8_0, oracle.Q8_0, 1024, 2816, 300, nvec=nvec)
    assert_parity(ref, got, what=f"q8_0 ffn nvec={nvec}")


def test_ffn_mixed_types_falls_back_to_unfused(engine):
    ref, got = run_ffn(engine, oracle.IQ3_S, oracle.Q4_K, 512, 1024, 400)
    assert_parity(ref, got, what="iq3_s/q4_k ffn")


EPS = 1e-5


def make_stack(engine, L, tg, td, d_model, d_ff, seed, k_in=None):
    k_in = k_in or d_model
    layers = [ffn_weights(tg, td, d_model, d_ff, seed + 10 * l, k_in) for l in range(L)]
    res = [(engine.upload(tg, d_ff, k_in, g), engine.upload(tg, d_ff, k_in, u),
            engine.upload(td, d_model, d_ff, d)) for g, u, d in layers]
    norms = [oracle.normal(seed + 10 * l + 7, d_model, 1.0, 0.1) for l in range(L)]
    return layers, res, norms


def oracle_stack(layers, norms, tg, td, d_model, d_ff, x, k_in=None):
    """x <- x + FFN(rms_norm(x)) per layer (stream_infer.rs:2166-2170, :3752-3864)."""
    k_in = k_in or d_model
    x = x.copy()
    for (g, u, d), nw in zip(layers, norms):
        xn = np.zeros(k_in, np.float32)
        xn[:d_model] = oracle.rms_norm(x[:d_model], nw, EPS)
        x[:d_model] = (x[:d_model] + oracle.ffn_swiglu(tg, g, tg, u, td, d, k_in, d_ff, d_model, xn)).astype(np.float32)
    return x


def split(res):
    return [r[0] for r in res], [r[1] for r in res], [r[2] for r in res]


def test_stack_parity(engine):
    L, dm, ff = 6, 1024, 2816
    layers, res, norms = make_stack(engine, L, oracle.Q4_K, oracle.Q6_K, dm, ff, 500)
    x = oracle.normal(501, dm)
    ref = oracle_stack(layers, norms, oracle.Q4_K, oracle.Q6_K, dm, ff, x)
    got = engine.ffn_stack(*split(res), x, norms=[torch.from_numpy(n).cuda() for n in norms], eps=EPS)
    assert_parity(ref, got, what="stack")


def test_bound_stack_matches_the_unbound_call(engine):
    """A stack bound once (BoundStack) gives the unbound call's bytes, call after call, into a
    caller's buffer or a new one, and checks its arguments."""
    L, dm, ff = 3, 1024, 2816
    layers, res, norms = make_stack(engine, L, oracle.Q4_K, oracle.Q6_K, dm, ff, 520)
    nd = [torch.from_numpy(n).cuda() for n in norms]
    x = oracle.normal(521, dm)
    want = engine.ffn_stack(*split(res), x, norms=nd, eps=EPS)
    bound = engine.bind_ffn_stack(*split(res), norms=nd, eps=EPS)
    out = np.empty(dm, np.float32)
    for _ in range(2):
        assert bound.run(x, out) is out
        assert np.array_equal(out, want)
    assert np.array_equal(bound.run(x), want)
    assert_parity(oracle_stack(layers, norms, oracle.Q4_K, oracle.Q6_K, dm, ff, x), out, what="bound stack")
    with pytest.raises(ValueError):
        bound.run(x, np.empty(dm - 1, np.float32))
    with pytest.raises(ValueError):
        engine.bind_ffn_stack(*split(res)[:2], split(res)[2][:1])


def test_stack_padded_k(engine):
    # SmolLM shape: K 576 zero-padded to 768 for Q4_K; norm and residual cover 576 entries
    L, dm, kin, ff = 3, 576, 768, 1536
    layers, res, norms = make_stack(engine, L, oracle.Q4_K, oracle.Q4_K, dm, ff, 550, k_in=kin)
    x = np.zeros(kin, np.float32)
    x[:dm] = oracle.normal(551, dm)
    ref = oracle_stack(layers, norms, oracle.Q4_K, oracle.Q4_K, dm, ff, x, k_in=kin)
    got = engine.ffn_stack(*split(res), x, norms=[torch.from_numpy(n).cuda() for n in norms], eps=EPS)
    assert np.all(got[dm:] == 0.0)
    assert_parity(ref, got, what="padded stack")


def test_stack_unfused_types(engine):
    L, dm, ff = 2, 512, 1024
    layers, res, norms = make_stack(engine, L, oracle.IQ3_S, oracle.Q8_0, dm, ff, 560)
    x = oracle.normal(561, dm)
    ref = oracle_stack(layers, norms, oracle.IQ3_S, oracle.Q8_0, dm, ff, x)
    got = engine.ffn_stack(*split(res), x, norms=[torch.from_numpy(n).cuda() for n in norms], eps=EPS)
    assert_parity(ref, got, what="unfused stack")


def test_stack_kernel_matches_per_layer_kernels(engine):
    L, dm, ff = 4, 4096, 14336
    layers, res, norms = make_stack(engine, L, oracle.Q4_K, oracle.Q6_K, dm, ff, 600)
    x = oracle.normal(601, dm)
    nd = [torch.from_numpy(n).cuda() for n in norms]
    xd = torch.from_numpy(x).cuda()
    engine.set_stream(torch.cuda.current_stream())
    try:
        engine.ffn_stack_dev(*split(res), xd, norms=nd, eps=EPS)
        torch.cuda.synchronize()
        y_graph = xd.cpu().numpy()
        xe = torch.from_numpy(x).cuda()
        h = torch.empty(ff, device="cuda")
        for (g, u, d), n in zip(res, nd):
            engine.ffn_gateup_dev(g, u, xe, h, norm=n, norm_len=dm, eps=EPS)
            ye = torch.empty_like(xe)
            engine.gemv_dev(d, h, ye, resid=xe)
            xe = ye
        torch.cuda.synchronize()
    finally:
        engine.set_stream(None)
    # the persistent stack kernel sums in a different (fixed) order than the per-layer kernels
    assert_parity(xe.cpu().numpy(), y_graph, what="stack kernel vs per-layer kernels")
    ref = oracle_stack(layers, norms, oracle.Q4_K, oracle.Q6_K, dm, ff, x)
    assert_parity(ref, y_graph, what="8b stack x4")
    # deterministic: the chunk order, not the CTA that ran a chunk, fixes every sum
    xd2 = torch.from_numpy(x).cuda()
    engine.set_stream(torch.cuda.current_stream())
    try:
        for _ in range(2):
            xd2.copy_(torch.from_numpy(x))
            engine.ffn_stack_dev(*split(res), xd2, norms=nd, eps=EPS)
            torch.cuda.synchronize()
            assert np.array_equal(y_graph, xd2.cpu().numpy())
    finally:
        engine.set_stream(None)


@pytest.mark.parametrize("tg,td,dm,ff", [
    (oracle.Q4_K, oracle.Q4_K, 1024, 5120),  # down needs 32-element sums of h; 2 chunks per down tile
    (oracle.Q6_K, oracle.Q6_K, 1024, 5120),
    (oracle.Q8_0, oracle.Q8_0, 1024, 2080),  # h table padded from 2080 to 17 x 128 elements
    (oracle.Q4_K, oracle.Q6_K, 2048, 8192),  # 2 chunks per down tile, 64 x 32 tiles
    # short d_ff (14 and 7 down blocks; 3584 is a 70B d_ff shard at 8 ranks): down K-parts of 4 blocks
    (oracle.Q4_K, oracle.Q6_K, 4096, 3584),
    (oracle.Q4_K, oracle.Q6_K, 4096, 1792),
])
def test_stack_kernel_formats(engine, tg, td, dm, ff):
    L = 3
    layers, res, norms = make_stack(engine, L, tg, td, dm, ff, 650)
    x = oracle.normal(651, dm)
    ref = oracle_stack(layers, norms, tg, td, dm, ff, x)
    nd = [torch.from_numpy(n).cuda() for n in norms]
    got = engine.ffn_stack(*split(res), x, norms=nd, eps=EPS)
    assert_parity(ref, got, what=f"stack kernel {tg}/{td} {dm}x{ff}")
    again = engine.ffn_stack(*split(res), x, norms=nd, eps=EPS)
    assert np.array_equal(got, again)


def test_stack_rejects_mismatched_layers(engine):
    import hayai_b200 as hb

    _, a, _ = make_stack(engine, 1, oracle.Q4_K, oracle.Q4_K, 512, 1024, 700)
    _, b, _ = make_stack(engine, 1, oracle.Q4_K, oracle.Q4_K, 768, 1024, 710)
    with pytest.raises(hb.CudaError):
        engine.ffn_stack([a[0][0], b[0][0]], [a[0][1], b[0][1]], [a[0][2], b[0][2]], np.zeros(512, np.float32))


@pytest.mark.parametrize("nvec", [8, 16, 64])
def test_stack_q8_0_tensor_core(engine, nvec):
    """Config-3 shape family: Q8_0 stack with RMSNorm at batch 8 (mma.sync GEMV), 16 and 64
    (tcgen05 path)."""
    L, dm, ff = 2, 1024, 2816
    layers, res, norms = make_stack(engine, L, oracle.Q8_0, oracle.Q8_0, dm, ff, 700)
    X = oracle.normal(701, nvec * dm).reshape(nvec, dm)
    nd = [torch.from_numpy(n).cuda() for n in norms]
    got = engine.ffn_stack(*split(res), X.reshape(-1), nvec=nvec, norms=nd, eps=EPS).reshape(nvec, dm)
    for b in range(0, nvec, max(1, nvec // 4)):
        ref = oracle_stack(layers, norms, oracle.Q8_0, oracle.Q8_0, dm, ff, X[b])
        assert_parity(ref, got[b], what=f"q8_0 stack batch {nvec} row {b}")


@pytest.mark.parametrize("nvec", [8, 16])
def test_stack_kquant_tensor_core(engine, nvec):
    """Config-5 batch shape family: Q4_K gate/up, Q6_K down with RMSNorm at batch 8 and 16
    (tcgen05 path)."""
    L, dm, ff = 2, 1024, 2816
    layers, res, norms = make_stack(engine, L, oracle.Q4_K, oracle.Q6_K, dm, ff, 720)
    X = oracle.normal(721, nvec * dm).reshape(nvec, dm)
    nd = [torch.from_numpy(n).cuda() for n in norms]
    got = engine.ffn_stack(*split(res), X.reshape(-1), nvec=nvec, norms=nd, eps=EPS).reshape(nvec, dm)
    for b in range(0, nvec, max(1, nvec // 4)):
        ref = oracle_stack(layers, norms, oracle.Q4_K, oracle.Q6_K, dm, ff, X[b])
        assert_parity(ref, got[b], what=f"q4_k/q6_k stack batch {nvec} row {b}")
