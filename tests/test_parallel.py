"""Tensor-parallel FFN stack (d_ff split) and expert-parallel MoE, one process per GPU.

CPU (gloo, world size 2): the d_ff sharding of gate/up rows and down columns reproduces the
unsharded FFN when the ranks' partial down outputs are added (oracle); the expert partition
with replicated routing and a top-k-ordered combine of the exchanged rows reproduces the
unpartitioned MoE (oracle); the IPC-handle exchange returns every rank's handle in rank
order.  GPU (2 devices, marked gpu): the persistent stack kernel with the in-kernel NVLink
exchange (batch 1), the per-layer kernels with the all-reduce kernel (batch > 1), and the
expert-parallel MoE with its fused exchange match the oracle and leave identical results on
both ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from hayai_b200 import tp as tpmod
from tests.helpers import assert_parity, quantized

EPS = 1e-5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, backend="gloo"):
    import datetime

    import torch.distributed as dist

    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


@pytest.mark.parametrize("t,m,n", [(oracle.Q4_K, 64, 1024), (oracle.Q6_K, 32, 2048), (oracle.Q8_0, 48, 256)])
@pytest.mark.parametrize("world", [2, 4])
def test_shards_cover_the_matrix(t, m, n, world):
    w = quantized(t, m, n, 11)
    rows = [tpmod.shard_rows(w, t, m, n, r, world)[0] for r in range(world)]
    assert np.array_equal(np.concatenate(rows), w)
    qk, bs = oracle.BLOCK[t]
    cols = [tpmod.shard_cols(w, t, m, n, r, world)[0].reshape(m, -1) for r in range(world)]
    assert np.array_equal(np.concatenate(cols, axis=1).reshape(-1), w)
    x = oracle.normal(12, n)
    # a column shard is an exact GEMV over its slice of x
    lo, hi = tpmod.shard_range(n, 1, world, qk)
    y1 = oracle.gemv(t, m, hi - lo, cols[1].reshape(-1), x[lo:hi])
    assert np.all(np.isfinite(y1))


def test_shard_rejects_partial_blocks():
    with pytest.raises(ValueError):
        tpmod.shard_range(14336, 0, 3, 256)


def _cpu_rank(rank, world, port, case):
    dist = _init(rank, world, port)
    try:
        tg, td, dm, ff = case
        wg, wu, wd = quantized(tg, ff, dm, 31), quantized(tg, ff, dm, 32), quantized(td, dm, ff, 33)
        x = oracle.normal(34, dm)
        g, _ = tpmod.shard_rows(wg, tg, ff, dm, rank, world)
        u, ffl = tpmod.shard_rows(wu, tg, ff, dm, rank, world)
        d, _ = tpmod.shard_cols(wd, td, dm, ff, rank, world)
        h = oracle.swiglu(oracle.gemv(tg, ffl, dm, g, x), oracle.gemv(tg, ffl, dm, u, x))
        part = oracle.gemv(td, dm, ffl, d, h)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        got = tpmod.tp_partial_sum(parts)
        ref = oracle.ffn_swiglu(tg, wg, tg, wu, td, wd, dm, ff, dm, x)
        assert_parity(ref, got, what=f"tp{world} oracle rank {rank}")
        handles = tpmod.gather_handles(bytes([rank]) * 64)
        assert handles == [bytes([r]) * 64 for r in range(world)]
    finally:
        dist.destroy_process_group()


def _cpu_rank_batch(rank, world, port, nvec):
    """The batched exchange's semantics: every row's partial down outputs, summed over the ranks
    in rank order and added to the replicated residual, reproduce the unsharded stack layer."""
    dist = _init(rank, world, port)
    try:
        tg, td, dm, ff = oracle.Q4_K, oracle.Q6_K, 512, 2048
        wg, wu, wd = quantized(tg, ff, dm, 41), quantized(tg, ff, dm, 42), quantized(td, dm, ff, 43)
        nw = oracle.normal(44, dm, 1.0, 0.1)
        X = oracle.normal(45, nvec * dm).reshape(nvec, dm)
        g, ffl = tpmod.shard_rows(wg, tg, ff, dm, rank, world)
        u, _ = tpmod.shard_rows(wu, tg, ff, dm, rank, world)
        d, _ = tpmod.shard_cols(wd, td, dm, ff, rank, world)
        parts = []
        for v in range(nvec):
            xn = oracle.rms_norm(X[v], nw, EPS)
            h = oracle.swiglu(oracle.gemv(tg, ffl, dm, g, xn), oracle.gemv(tg, ffl, dm, u, xn))
            parts.append(oracle.gemv(td, dm, ffl, d, h))
        gathered = [None] * world
        dist.all_gather_object(gathered, np.stack(parts))
        got = (X + tpmod.tp_partial_sum(gathered)).astype(np.float32)
        for v in range(nvec):
            ref = _oracle_stack([(wg, wu, wd)], [nw], tg, td, dm, ff, X[v])
            assert_parity(ref, got[v], what=f"tp{world} batch row {v} rank {rank}")
    finally:
        dist.destroy_process_group()


def test_tp_batched_exchange_two_ranks_gloo():
    port = _free_port()
    mp.spawn(_cpu_rank_batch, args=(2, port, 3), nprocs=2, join=True)


def test_tp_sharding_two_ranks_gloo():
    port = _free_port()
    mp.spawn(_cpu_rank, args=(2, port, (oracle.Q4_K, oracle.Q6_K, 512, 2048)), nprocs=2, join=True)


# ---------------------------------------------------------------- GPU (2 devices)
def _oracle_stack(layers, norms, tg, td, dm, ff, x):
    x = x.copy()
    for (g, u, d), nw in zip(layers, norms):
        xn = oracle.rms_norm(x, nw, EPS)
        x = (x + oracle.ffn_swiglu(tg, g, tg, u, td, d, dm, ff, dm, xn)).astype(np.float32)
    return x


def _gpu_rank(rank, world, port, case, result_path):
    import hayai_b200 as hb

    torch.cuda.set_device(rank)
    dist = _init(rank, world, port)
    eng = hb.CudaEngine(rank)
    peers = None
    try:
        tg, td, dm, ff, L, nvec = case
        layers = [(quantized(tg, ff, dm, 40 + 3 * l), quantized(tg, ff, dm, 41 + 3 * l),
                   quantized(td, dm, ff, 42 + 3 * l)) for l in range(L)]
        norms = [oracle.normal(70 + l, dm, 1.0, 0.1) for l in range(L)]
        X = oracle.normal(80, nvec * dm).reshape(nvec, dm)
        G, U, D = [], [], []
        for g, u, d in layers:
            gs, ffl = tpmod.shard_rows(g, tg, ff, dm, rank, world)
            us, _ = tpmod.shard_rows(u, tg, ff, dm, rank, world)
            ds, _ = tpmod.shard_cols(d, td, dm, ff, rank, world)
            G.append(eng.upload(tg, ffl, dm, gs))
            U.append(eng.upload(tg, ffl, dm, us))
            D.append(eng.upload(td, dm, ffl, ds))
        nd = [torch.from_numpy(n).cuda(rank) for n in norms]
        peers = tpmod.PeerGroup(eng)
        got = eng.ffn_stack_tp(G, U, D, X.reshape(-1), nvec, norms=nd, eps=EPS).reshape(nvec, dm)
        # the cross-GPU counters and device epochs carry over, also across the batch-1 and
        # batched exchanges, which use separate counters and buffers
        one = eng.ffn_stack_tp(G, U, D, X[0], norms=nd, eps=EPS) if nvec > 1 else None
        again = eng.ffn_stack_tp(G, U, D, X.reshape(-1), nvec, norms=nd, eps=EPS).reshape(nvec, dm)
        outs = [None] * world
        dist.all_gather_object(outs, (got, again, one))
        if rank == 0:
            for r, (a, b, o) in enumerate(outs):
                for v in range(nvec):
                    ref = _oracle_stack(layers, norms, tg, td, dm, ff, X[v])
                    assert_parity(ref, a[v], what=f"tp{world} stack rank {r} row {v}")
                    if v == 0 and o is not None:
                        assert_parity(ref, o, what=f"tp{world} batch-1 stack between batched calls, rank {r}")
                assert np.array_equal(a, outs[0][0]), "ranks disagree"
                assert np.array_equal(a, b), "second call differs"
            with open(result_path, "w") as f:
                f.write("ok")
    finally:
        if peers is not None:
            peers.close()
        eng.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("case", [
    (oracle.Q4_K, oracle.Q6_K, 1024, 4096, 3, 1),   # one down chunk per tile and rank
    (oracle.Q4_K, oracle.Q6_K, 1024, 16384, 2, 1),  # two down chunks per tile and rank
    (oracle.Q4_K, oracle.Q6_K, 1024, 4096, 3, 16),  # batch 16: per-layer kernels + all-reduce kernel
    (oracle.Q8_0, oracle.Q8_0, 1024, 4096, 2, 12),  # batch 12 on the tcgen05 GEMM
    (oracle.Q4_K, oracle.Q6_K, 1024, 4096, 2, 3),   # ragged batch
])
def test_tp_stack_two_gpus(tmp_path, case):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    res = tmp_path / "ok"
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_gpu_rank, args=(2, port, case, str(res)), nprocs=2, join=True)
    assert res.read_text() == "ok"


# ---------------------------------------------------------------- expert parallelism
def _moe_case(E, T, dm, ff, seed=90):
    t = oracle.Q4_K
    wg = np.stack([quantized(t, ff, dm, seed + 3 * e) for e in range(E)])
    wu = np.stack([quantized(t, ff, dm, seed + 1 + 3 * e) for e in range(E)])
    wd = np.stack([quantized(t, dm, ff, seed + 2 + 3 * e) for e in range(E)])
    R = oracle.normal(seed + 500, E * dm, 0, 0.02).reshape(E, dm)
    X = oracle.normal(seed + 501, T * dm).reshape(T, dm)
    return wg, wu, wd, R, X


def _cpu_ep_rank(rank, world, port, E, k, T, dm, ff):
    dist = _init(rank, world, port)
    try:
        t = oracle.Q4_K
        wg, wu, wd, R, X = _moe_case(E, T, dm, ff)
        lo, hi = tpmod.expert_range(E, rank, world)
        rows = {}
        for tok in range(T):
            scores = oracle.gemv(oracle.F32, E, dm, R.view(np.uint8), X[tok])
            ids, _ = oracle.route_experts(scores, k)
            for i, e in enumerate(ids):
                if lo <= e < hi:  # this rank's expert: the row it stores into every region
                    rows[(tok, i)] = oracle.ffn_swiglu(t, wg[e], t, wu[e], t, wd[e], dm, ff, dm, X[tok])
        parts = [None] * world
        dist.all_gather_object(parts, rows)
        allrows = {}
        for p in parts:
            assert not set(p) & set(allrows), "a pair computed by two ranks"
            allrows.update(p)
        assert len(allrows) == T * k
        ref_y, ref_ids, ref_w = oracle.moe_ffn(R, E, k, t, wg, t, wu, t, wd, dm, ff, X)
        y = np.zeros((T, dm), np.float32)
        for tok in range(T):
            acc = np.zeros(dm, np.float32)
            for i in range(k):  # top-k order, as the combine kernel
                acc = (acc + (ref_w[tok, i] * allrows[(tok, i)]).astype(np.float32)).astype(np.float32)
            y[tok] = acc
        assert_parity(ref_y, y, what=f"ep{world} oracle rank {rank}")
    finally:
        dist.destroy_process_group()


def test_ep_partition_two_ranks_gloo():
    port = _free_port()
    mp.spawn(_cpu_ep_rank, args=(2, port, 16, 4, 6, 512, 256), nprocs=2, join=True)


def _gpu_ep_rank(rank, world, port, case, result_path):
    import hayai_b200 as hb

    torch.cuda.set_device(rank)
    dist = _init(rank, world, port)
    eng = hb.CudaEngine(rank)
    peers = None
    try:
        E, k, T, dm, ff = case
        t = oracle.Q4_K
        wg, wu, wd, R, X = _moe_case(E, T, dm, ff)
        lo, hi = tpmod.expert_range(E, rank, world)
        G = [eng.upload(t, ff, dm, wg[e]) for e in range(lo, hi)]
        U = [eng.upload(t, ff, dm, wu[e]) for e in range(lo, hi)]
        Dn = [eng.upload(t, dm, ff, wd[e]) for e in range(lo, hi)]
        Rd, Xd = torch.from_numpy(R).cuda(rank), torch.from_numpy(X).cuda(rank)
        peers = tpmod.PeerGroup(eng)
        stream = torch.cuda.current_stream(rank)
        eng.set_stream(stream)
        outs = []
        for _ in range(3):  # the exchange buffers alternate; the counters carry over
            Y = torch.empty(T, dm, device=f"cuda:{rank}")
            ids = torch.empty(T, k, dtype=torch.int32, device=f"cuda:{rank}")
            eng.moe_ffn_ep_dev(Rd, k, G, U, Dn, lo, Xd, Y, ids)
            torch.cuda.synchronize(rank)
            eng.sync()
            outs.append((Y.cpu().numpy(), ids.cpu().numpy()))
        eng.set_stream(None)
        # the stack entry point (one graph launch per call; the epochs live on the device)
        Xs = Xd.clone()
        eng.set_stream(stream)
        for _ in range(2):
            Xs.copy_(Xd)
            eng.moe_stack_dev([Rd, Rd], k, [G, G], [U, U], [Dn, Dn], Xs, expert_lo=lo, ep=True)
            torch.cuda.synchronize(rank)
            eng.sync()
        eng.set_stream(None)
        outs.append((Xs.cpu().numpy(), None))
        gathered = [None] * world
        dist.all_gather_object(gathered, outs)
        if rank == 0:
            ref_y, ref_ids, _ = oracle.moe_ffn(R, E, k, t, wg, t, wu, t, wd, dm, ff, X)
            x1 = (X + ref_y).astype(np.float32)
            y1, _, _ = oracle.moe_ffn(R, E, k, t, wg, t, wu, t, wd, dm, ff, x1)
            ref_stack = (x1 + y1).astype(np.float32)
            for r, runs in enumerate(gathered):
                for y, ids in runs[:-1]:
                    assert np.array_equal(ids, ref_ids), f"rank {r} routing"
                    assert_parity(ref_y, y, what=f"ep{world} moe rank {r}")
                    assert np.array_equal(y, gathered[0][0][0]), "ranks or calls disagree"
                assert_parity(ref_stack, runs[-1][0], what=f"ep{world} moe stack x2 rank {r}")
                assert np.array_equal(runs[-1][0], gathered[0][-1][0]), "ranks disagree on the stack"
            with open(result_path, "w") as f:
                f.write("ok")
    finally:
        if peers is not None:
            peers.close()
        eng.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_moe_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    res = tmp_path / "ok"
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_gpu_ep_rank, args=(2, port, (16, 4, 8, 2048, 768), str(res)), nprocs=2, join=True)
    assert res.read_text() == "ok"


# ---------------------------------------------------------------- failure detection
@pytest.mark.gpu
def test_exchange_wait_expires_and_engine_recovers(engine):
    """A rank whose peers never signal: the exchange's wait is bounded (about a second), the
    call reports HC_ERR_TIMEOUT, and the engine keeps working.  A one-rank group whose device
    epoch is moved ahead of its counter stands in for a peer that never arrives (a counter
    that nothing will raise); no GPU fault is involved."""
    import time

    from cuda.bindings import runtime as rt

    import hayai_b200 as hb
    from hayai_b200 import _lib

    tg, td, dm, ff, nvec = oracle.Q4_K, oracle.Q6_K, 1024, 2048, 16
    g, u, d = quantized(tg, ff, dm, 301), quantized(tg, ff, dm, 302), quantized(td, dm, ff, 303)
    nw = oracle.normal(304, dm, 1.0, 0.1)
    G, U, D = [engine.upload(tg, ff, dm, g)], [engine.upload(tg, ff, dm, u)], [engine.upload(td, dm, ff, d)]
    N = [torch.from_numpy(nw).cuda()]
    X = oracle.normal(305, nvec * dm).reshape(nvec, dm)
    engine.peer_connect([engine.peer_open(0, 1)])
    try:
        got = engine.ffn_stack_tp(G, U, D, X.reshape(-1), nvec, norms=N, eps=EPS).reshape(nvec, dm)
        for v in (0, nvec - 1):
            assert_parity(_oracle_stack([(g, u, d)], [nw], tg, td, dm, ff, X[v]), got[v], what=f"one-rank tp row {v}")
        region, _ = engine.peer_region()
        epoch = np.zeros(1, np.uint32)
        kind = rt.cudaMemcpyKind
        assert rt.cudaMemcpy(epoch.ctypes.data, region + 512, 4, kind.cudaMemcpyDeviceToHost)[0] == \
            rt.cudaError_t.cudaSuccess
        assert epoch[0] == 1  # one exchange so far
        epoch[0] += 5  # the next exchange now waits for signals that never come
        assert rt.cudaMemcpy(region + 512, epoch.ctypes.data, 4, kind.cudaMemcpyHostToDevice)[0] == \
            rt.cudaError_t.cudaSuccess
        t0 = time.time()
        with pytest.raises(hb.CudaError) as e:
            engine.ffn_stack_tp(G, U, D, X.reshape(-1), nvec, norms=N, eps=EPS)
        assert e.value.code == _lib.HC_ERR_TIMEOUT
        assert time.time() - t0 < 30
    finally:
        engine.peer_close()
    # the context is intact: the same weights still give the oracle's answer
    x = X[0].copy()
    assert_parity(oracle.gemv(tg, ff, dm, g, x), engine.ggml_gemv_dispatch_bound(G[0], x), what="after timeout")


@pytest.mark.gpu
def test_ep_rows_beyond_their_exchange_area_are_rejected(engine):
    """The expert-parallel MoE exchanges its routed rows through a fixed area of the peer
    region; the batched tensor-parallel exchange owns the bytes after it.  A call whose rows
    would not fit (2 x tokens x top-k x d_model x 4 B above the area) is rejected before any
    launch, and the same one-rank group still runs a call that fits, matching the oracle."""
    import hayai_b200 as hb
    from hayai_b200 import _lib

    t, E, k, dm, ff = oracle.Q4_K, 4, 4, 2048, 256
    g = [quantized(t, ff, dm, 400 + e) for e in range(E)]
    u = [quantized(t, ff, dm, 410 + e) for e in range(E)]
    d = [quantized(t, dm, ff, 420 + e) for e in range(E)]
    G = [engine.upload(t, ff, dm, w) for w in g]
    U = [engine.upload(t, ff, dm, w) for w in u]
    D = [engine.upload(t, dm, ff, w) for w in d]
    r = oracle.normal(430, E * dm, 0.0, 0.02).reshape(E, dm)
    R = torch.from_numpy(r).cuda()
    engine.peer_connect([engine.peer_open(0, 1)])
    try:
        T = 400  # 1600 routed rows: 2 x 1600 x 2048 x 4 B = 26.2 MB, above the 24 MiB area
        X = torch.zeros(T, dm, device="cuda")
        Y = torch.zeros(T, dm, device="cuda")
        with pytest.raises(hb.CudaError) as e:
            engine.moe_ffn_ep_dev(R, k, G, U, D, 0, X, Y)
        assert e.value.code == _lib.HC_ERR_INVALID
        assert "EP area" in str(e.value)
        T = 8
        xh = oracle.normal(431, T * dm).reshape(T, dm)
        X = torch.from_numpy(xh).cuda()
        Y = torch.zeros(T, dm, device="cuda")
        ids = torch.zeros(T, k, dtype=torch.int32, device="cuda")
        engine.moe_ffn_ep_dev(R, k, G, U, D, 0, X, Y, ids)
        torch.cuda.synchronize()
        want, want_ids, _ = oracle.moe_ffn(r, E, k, t, np.stack(g), t, np.stack(u), t, np.stack(d), dm, ff, xh)
        assert np.array_equal(ids.cpu().numpy(), want_ids)
        assert_parity(want, Y.cpu().numpy(), what="one-rank EP after the rejection")
    finally:
        engine.peer_close()
        for w in G + U + D:
            w.free()
