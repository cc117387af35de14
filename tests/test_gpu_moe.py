"""GPU parity of the MoE path (C ABI): router scores and top-k ids are bit-exact with the
oracle; routed expert FFN outputs meet rel-L2 <= 1e-4 / max-abs <= 1e-3."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_parity, quantized

pytestmark = pytest.mark.gpu


def on_stream(engine, fn):
    engine.set_stream(torch.cuda.current_stream())
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        engine.set_stream(None)


def test_router_scores_bit_exact(engine):
    E, D, T = 128, 2048, 16
    W = oracle.normal(1, E * D, 0, 0.02).reshape(E, D)
    X = oracle.normal(2, T * D).reshape(T, D)
    ref = np.stack([oracle.gemv(oracle.F32, E, D, W.view(np.uint8), X[t]) for t in range(T)])
    Wd, Xd = torch.from_numpy(W).cuda(), torch.from_numpy(X).cuda()
    S = torch.empty(T, E, device="cuda")
    on_stream(engine, lambda: engine.router_scores_dev(Wd, Xd, S, T))
    assert np.array_equal(ref, S.cpu().numpy())


@pytest.mark.parametrize("variant", ["plain", "ties", "bias", "norm_scale", "sigmoid", "grouped"])
def test_route_experts_bit_exact(engine, variant):
    T, E, k = 33, 128, 8
    S = oracle.normal(3, T * E).reshape(T, E)
    kw = {}
    if variant == "ties":
        S = np.round(S * 4) / 4  # many exact ties
    if variant == "bias":
        kw["bias"] = oracle.normal(4, E) * np.float32(0.5)
    if variant == "norm_scale":
        kw.update(norm_topk_prob=True, routed_scaling_factor=2.5)
    if variant == "sigmoid":
        kw.update(gating=1)
    if variant == "grouped":
        kw.update(n_group=8, topk_group=3, gating=1)
    S = S.astype(np.float32)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    Sd = torch.from_numpy(S).cuda()
    bias_d = torch.from_numpy(kw["bias"]).cuda() if "bias" in kw else None
    dkw = {kk: v for kk, v in kw.items() if kk != "bias"}
    on_stream(engine, lambda: engine.route_experts_dev(Sd, ids, wts, k, bias=bias_d, **dkw))
    gi, gw = ids.cpu().numpy(), wts.cpu().numpy()
    for t in range(T):
        ri, rw = oracle.route_experts(S[t], k, **kw)
        assert np.array_equal(ri, gi[t]), (t, ri, gi[t])
        assert np.abs(rw - gw[t]).max() <= 1e-6 * max(1.0, float(np.abs(rw).max())) * 4


@pytest.mark.parametrize("E,k,T,t,dm,ff", [
    (32, 4, 5, oracle.Q4_K, 2048, 768),
    (128, 8, 16, oracle.Q4_K, 2048, 768),   # Qwen3-30B-A3B shape
    (8, 4, 16, oracle.Q4_K, 2048, 768),     # ~8 pairs per expert: experts split over several segments
    (16, 2, 6, oracle.Q8_0, 1024, 512),
    (16, 2, 6, oracle.Q6_K, 1024, 512),
    (8, 2, 4, oracle.Q4_K, 4096, 512),      # gate/up K too long for one stage: per-pair kernel
])
def test_moe_ffn_parity(engine, E, k, T, t, dm, ff):
    wg = np.stack([quantized(t, ff, dm, 10 + 3 * e) for e in range(E)])
    wu = np.stack([quantized(t, ff, dm, 11 + 3 * e) for e in range(E)])
    wd = np.stack([quantized(t, dm, ff, 12 + 3 * e) for e in range(E)])
    R = oracle.normal(5, E * dm, 0, 0.02).reshape(E, dm)
    X = oracle.normal(6, T * dm).reshape(T, dm)
    ref_y, ref_ids, ref_w = oracle.moe_ffn(R, E, k, t, wg, t, wu, t, wd, dm, ff, X)
    G = [engine.upload(t, ff, dm, wg[e]) for e in range(E)]
    U = [engine.upload(t, ff, dm, wu[e]) for e in range(E)]
    Dn = [engine.upload(t, dm, ff, wd[e]) for e in range(E)]
    Rd, Xd = torch.from_numpy(R).cuda(), torch.from_numpy(X).cuda()
    Y = torch.empty(T, dm, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    on_stream(engine, lambda: engine.moe_ffn_dev(Rd, k, G, U, Dn, Xd, Y, ids, wts))
    assert np.array_equal(ref_ids, ids.cpu().numpy())
    assert_parity(ref_w, wts.cpu().numpy(), what="routing weights")
    assert_parity(ref_y, Y.cpu().numpy(), what=f"moe E={E} k={k} type={t}")


def test_moe_stack_parity(engine):
    """x <- x + MoE_l(x) over 3 layers through one graph launch; replays are deterministic."""
    E, k, T, dm, ff, L = 32, 4, 6, 2048, 768, 3
    t = oracle.Q4_K
    layers = []
    for l in range(L):
        wg = np.stack([quantized(t, ff, dm, 100 * l + 3 * e) for e in range(E)])
        wu = np.stack([quantized(t, ff, dm, 100 * l + 1 + 3 * e) for e in range(E)])
        wd = np.stack([quantized(t, dm, ff, 100 * l + 2 + 3 * e) for e in range(E)])
        R = oracle.normal(900 + l, E * dm, 0, 0.02).reshape(E, dm)
        layers.append((wg, wu, wd, R))
    X = oracle.normal(950, T * dm).reshape(T, dm)
    ref = X.copy()
    for wg, wu, wd, R in layers:
        y, _, _ = oracle.moe_ffn(R, E, k, t, wg, t, wu, t, wd, dm, ff, ref)
        ref = (ref + y).astype(np.float32)
    G = [[engine.upload(t, ff, dm, wg[e]) for e in range(E)] for wg, _, _, _ in layers]
    U = [[engine.upload(t, ff, dm, wu[e]) for e in range(E)] for _, wu, _, _ in layers]
    Dn = [[engine.upload(t, dm, ff, wd[e]) for e in range(E)] for _, _, wd, _ in layers]
    Rd = [torch.from_numpy(R).cuda() for _, _, _, R in layers]
    outs = []
    for _ in range(2):
        Xd = torch.from_numpy(X).cuda()
        on_stream(engine, lambda: engine.moe_stack_dev(Rd, k, G, U, Dn, Xd))
        outs.append(Xd.cpu().numpy())
    assert_parity(ref, outs[0], what="moe stack x3")
    assert np.array_equal(outs[0], outs[1])
