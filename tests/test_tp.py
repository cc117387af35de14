"""Tensor-parallel FFN stack (d_ff split, one process per GPU).

CPU (gloo, world size 2): the d_ff sharding of gate/up rows and down columns reproduces the
unsharded FFN when the ranks' partial down outputs are added (oracle), and the IPC-handle
exchange returns every rank's handle in rank order.  GPU (2 devices, marked gpu): the
persistent stack kernel with the in-kernel NVLink exchange matches the unsharded oracle and
leaves x identical on both ranks.
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
        tg, td, dm, ff, L = case
        layers = [(quantized(tg, ff, dm, 40 + 3 * l), quantized(tg, ff, dm, 41 + 3 * l),
                   quantized(td, dm, ff, 42 + 3 * l)) for l in range(L)]
        norms = [oracle.normal(70 + l, dm, 1.0, 0.1) for l in range(L)]
        x = oracle.normal(80, dm)
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
        got = eng.ffn_stack_tp(G, U, D, x, norms=nd, eps=EPS)
        again = eng.ffn_stack_tp(G, U, D, x, norms=nd, eps=EPS)  # the cross-GPU counters carry over
        outs = [None] * world
        dist.all_gather_object(outs, (got, again))
        if rank == 0:
            ref = _oracle_stack(layers, norms, tg, td, dm, ff, x)
            for r, (a, b) in enumerate(outs):
                assert_parity(ref, a, what=f"tp{world} stack rank {r}")
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
    (oracle.Q4_K, oracle.Q6_K, 1024, 4096, 3),   # one down chunk per tile and rank
    (oracle.Q4_K, oracle.Q6_K, 1024, 16384, 2),  # two down chunks per tile and rank
])
def test_tp_stack_two_gpus(tmp_path, case):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    res = tmp_path / "ok"
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_gpu_rank, args=(2, port, case, str(res)), nprocs=2, join=True)
    assert res.read_text() == "ok"
