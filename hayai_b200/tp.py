"""Tensor and expert parallelism over the GPUs of one box (one process per GPU).

Sharding (the d_ff split of the Llama-3-70B configuration): rank p of P holds gate/up rows
[p*F/P, (p+1)*F/P) and the same range of down columns, cut at whole quantization blocks, so
h never leaves its GPU.  The down projection then yields a partial sum on every rank; the
persistent stack kernel pushes each layer's partials into every rank's exchange region over
NVLink and adds them in rank order (hc_ffn_stack_tp_dev, batch 1; at batch > 1 one all-reduce
kernel after each layer's down GEMV does the same), so the replicated residual stream stays
identical on all ranks.  Expert parallelism (the MoE layer) gives rank p the experts
``expert_range(E, p, P)``; the router and top-k run replicated, each rank computes the pairs
routed to its experts and stores their rows into every rank's region, and every rank
combines them in top-k order (hc_moe_ffn_ep_dev).  ``PeerGroup`` sets up the exchange regions over a
torch.distributed process group (gloo or nccl), which only carries the IPC handles.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np

from .engine import BLOCK


def shard_range(total: int, rank: int, world: int, align: int) -> tuple[int, int]:
    """[lo, hi) of rank's equal share of `total`, in whole units of `align`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if total % (align * world):
        raise ValueError(f"{total} does not split into {world} shards of whole {align}-element blocks")
    step = total // world
    return rank * step, (rank + 1) * step


def shard_rows(raw: np.ndarray, ggml_type: int, m: int, n: int, rank: int, world: int) -> tuple[np.ndarray, int]:
    """Rows [lo, hi) of an m x n packed matrix (row shard of gate/up): (bytes, rows)."""
    qk, bs = BLOCK[ggml_type]
    rb = n // qk * bs
    lo, hi = shard_range(m, rank, world, 1)
    raw = np.frombuffer(memoryview(raw), dtype=np.uint8)
    return np.ascontiguousarray(raw[lo * rb:hi * rb]), hi - lo


def shard_cols(raw: np.ndarray, ggml_type: int, m: int, n: int, rank: int, world: int) -> tuple[np.ndarray, int]:
    """Columns [lo, hi) of an m x n packed matrix, whole blocks (column shard of down): (bytes, cols)."""
    qk, bs = BLOCK[ggml_type]
    lo, hi = shard_range(n, rank, world, qk)
    nb = n // qk
    blocks = np.frombuffer(memoryview(raw), dtype=np.uint8).reshape(m, nb, bs)
    return np.ascontiguousarray(blocks[:, lo // qk:hi // qk, :]).reshape(-1), hi - lo


def expert_range(n_expert: int, rank: int, world: int) -> tuple[int, int]:
    """Experts [lo, hi) held by rank under expert parallelism (n_expert / world each)."""
    return shard_range(n_expert, rank, world, 1)


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's IPC handle, in rank order, over a torch.distributed group."""
    import torch.distributed as dist

    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return [bytes(h) for h in out]


class PeerGroup:
    """The exchange regions of one process group: open, gather handles, connect, barrier."""

    def __init__(self, engine, group=None, nbytes: int = 64 << 20):
        import torch.distributed as dist

        self.engine = engine
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        handle = engine.peer_open(self.rank, self.world, nbytes)
        engine.peer_connect(gather_handles(handle, group))
        dist.barrier(group)  # every region mapped and zeroed before the first parallel call

    def close(self) -> None:
        import torch.distributed as dist

        dist.barrier(self.group)  # no rank still stores into another's region
        self.engine.peer_close()


def tp_partial_sum(partials: Sequence[np.ndarray]) -> np.ndarray:
    """The ranks' partial down outputs added in rank order (the kernel's order)."""
    acc = np.zeros_like(np.asarray(partials[0], np.float32))
    for p in partials:
        acc = (acc + np.asarray(p, np.float32)).astype(np.float32)
    return acc
