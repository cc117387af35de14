#!/usr/bin/env python
"""Benchmark of the quantized-FFN hot path (BASELINE.json metric: FFN GEMV achieved HBM GB/s
and FFN tokens/s).

Default workload: Llama-3-8B-shaped FFN stack, 32 layers resident
in HBM, gate/up Q4_K, down Q6_K, batch-1 decode, x <- x + FFN_l(rms_norm(x)).  One step = one
token through all 32 layers: at batch 1 the whole stack is ONE persistent kernel launch
(ffn_stack.cu), otherwise the per-layer kernels as one CUDA graph (two GEMV launches per layer,
six on the tcgen05 batch path).  Weights are seeded N(0, 0.02^2)
quantized on the device with the reference's Q4_K quantizer (and this project's Q6_K
quantizer); activations N(0, 1).  --layers N shrinks the stack (a small case for profilers).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

Multi-GPU (torchrun, one rank per GPU): configs 1-3 do not shard, so every rank runs an
independent replica ("weak" scaling, no collective on the data path); value = all ranks'
bytes / max-over-ranks time.  --tp (llama70b) and --ep (qwen3moe) shard the model instead.

Other workloads: --config smollm | llama8b-q8 | llama70b | qwen3moe | lut-q4 | gemv-<format>.

--impl reference times the reference's CPU implementation of the path (the C restatement
in oracle/, the Rust reference cannot be built here) on this host's cores, on a bounded
sample of the same workload (one layer per step), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FFN GEMV achieved HBM GB/s (fraction of 8 TB/s) and FFN tokens/sec at 1/2/4/8 B200"

# ---------------------------------------------------------------- workloads
Q4_K, Q6_K, Q8_0 = 12, 14, 8
BLK = {Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34)}


def mat_bytes(t, m, n):
    qk, bs = BLK[t]
    return m * n // qk * bs


CONFIGS = {
    # name: (layers, d_model, k_in, d_ff, gate/up type, down type, description)
    "llama8b": dict(layers=32, d_model=4096, k_in=4096, d_ff=14336, tg=Q4_K, td=Q6_K,
                    workload="Llama-3-8B FFN stack x32, gate/up Q4_K, down Q6_K, batch-1 decode"),
    "smollm": dict(layers=256, d_model=576, k_in=768, d_ff=1536, tg=Q4_K, td=Q4_K,
                   workload="SmolLM2-135M FFN layer (Q4_K x3, K 576 zero-padded to 768), 256 distinct "
                            "resident copies streamed as a stack (HBM figure; one copy fits in L2)"),
    "llama8b-q8": dict(layers=8, d_model=4096, k_in=4096, d_ff=14336, tg=Q8_0, td=Q8_0,
                       workload="Llama-3-8B FFN shape, Q8_0 x3, stack of 8 distinct layers"),
    "llama70b": dict(layers=80, d_model=8192, k_in=8192, d_ff=28672, tg=Q4_K, td=Q6_K,
                     workload="Llama-3-70B FFN stack x80, gate/up Q4_K, down Q6_K, batch-1 decode"),
    # MoE: experts' gate/up d_ff x d_model and down d_model x d_ff
    "qwen3moe": dict(layers=48, d_model=2048, k_in=2048, d_ff=768, tg=Q4_K, td=Q4_K, n_expert=128, top_k=8,
                     tokens=16, workload="Qwen3-30B-A3B MoE FFN x48, 128 experts top-8, Q4_K experts, F32 router, "
                                         "16 tokens, x <- x + MoE_l(x)"),
}


# Single-GEMV workloads, one per GGML format: the Llama-3-8B gate shape (14336 x 4096), batch 1,
# enough distinct resident copies to exceed L2.  (type id, elements, bytes per block)
GEMV_FORMATS = {"q4_0": (2, 32, 18), "q4_1": (3, 32, 20), "q5_0": (6, 32, 22), "q5_1": (7, 32, 24),
                "q8_0": (8, 32, 34), "q2_k": (10, 256, 84), "q3_k": (11, 256, 110), "q4_k": (12, 256, 144),
                "q5_k": (13, 256, 176), "q6_k": (14, 256, 210), "iq2_xxs": (16, 256, 66), "iq2_xs": (17, 256, 74),
                "iq3_xxs": (18, 256, 98), "iq4_nl": (20, 32, 18), "iq3_s": (21, 256, 110), "iq2_s": (22, 256, 82),
                "iq4_xs": (23, 256, 136)}
for _name, (_t, _qk, _bs) in GEMV_FORMATS.items():
    BLK.setdefault(_t, (_qk, _bs))
    CONFIGS["gemv-" + _name] = dict(gemv=True, t=_t, m=14336, k=4096,
                                    workload=f"single {_name} GEMV, Llama-3-8B gate shape 14336 x 4096, batch 1")
# The toy LUT-Q4 matmul of the reference's `hayai bench` (crates/hayai-cli/src/main.rs:601-646):
# SmolLM-135M FFN shape 1536 x 576, weights 0xAB, x = 1, a fixed 16-entry LUT.
CONFIGS["lut-q4"] = dict(lut=True, m=1536, n=576,
                         workload="toy LUT-Q4 matmul of `hayai bench`: 1536 x 576, weights 0xAB, x = 1")
LUT16 = [-0.5, -0.4, -0.3, -0.2, -0.1, 0.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0]
# f16 scale offsets and typical |value| / d of random codes (random valid blocks for the formats
# without a quantizer here), and (offset, multiple of d) of a min field that centres the values
_RAND_D_AT = {2: (0,), 3: (0,), 6: (0,), 7: (0,), 10: (80,), 11: (108,), 13: (0,), 16: (0,), 17: (0,), 18: (0,),
              20: (0,), 21: (0,), 22: (0,), 23: (0,)}
_RAND_SCALE = {2: 4.0, 3: 4.0, 6: 8.0, 7: 8.0, 10: 8.0, 11: 32.0, 13: 250.0, 16: 50.0, 17: 50.0, 18: 120.0, 20: 60.0,
               21: 130.0, 22: 50.0, 23: 1000.0}
_RAND_MIN_AT = {3: (2, -7.5), 7: (2, -15.5), 10: (82, 1.5), 13: (2, 15.5)}


def random_blocks(t, m, n, seed, std=0.02):
    """Random valid blocks of format t with the scales set for |w| ~ std (host numpy)."""
    import numpy as np

    qk, bs = BLK[t]
    nblk = m * n // qk
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(nblk, bs), dtype=np.uint8)
    d = (std / _RAND_SCALE[t] * rng.uniform(0.5, 1.5, nblk)).astype(np.float16)
    for off in _RAND_D_AT[t]:
        b[:, off:off + 2] = d.view(np.uint8).reshape(nblk, 2)
    if t in _RAND_MIN_AT:
        off, ratio = _RAND_MIN_AT[t]
        b[:, off:off + 2] = (d.astype(np.float32) * np.float32(ratio)).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    return b.reshape(-1)


def expert_bytes(c):
    return 2 * mat_bytes(c["tg"], c["d_ff"], c["d_model"]) + mat_bytes(c["td"], c["d_model"], c["d_ff"])


def router_bytes(c):
    return c["n_expert"] * c["d_model"] * 4


def layer_bytes(c):
    return 2 * mat_bytes(c["tg"], c["d_ff"], c["k_in"]) + mat_bytes(c["td"], c["d_model"], c["d_ff"])


# ---------------------------------------------------------------- clocks sampler
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [v.strip() for v in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax.append(float(p[2]))
            except ValueError:
                continue
            for name, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- helpers
def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic(kernel_key: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel_key)
    except (OSError, ValueError):
        return None


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------- CPU baseline (oracle port)
EPS = 1e-5


def oracle_layer(c, g, u, d, nw, x):
    """One FFN sublayer on the CPU path: FFN(rms_norm(x)) (stream_infer.rs:2166-2170, :3752-3864)."""
    import numpy as np

    import oracle

    dm = c["d_model"]
    xn = np.zeros(c["k_in"], np.float32)
    xn[:dm] = oracle.rms_norm(x[:dm], nw, EPS)
    return oracle.ffn_swiglu(c["tg"], g, c["tg"], u, c["td"], d, c["k_in"], c["d_ff"], dm, xn)


def host_layer(c, seed):
    """Seeded layer generated on the host with the oracle (zero-padded K where needed)."""
    import numpy as np

    import oracle

    dm, kin, ff = c["d_model"], c["k_in"], c["d_ff"]

    def gu(s):
        w = np.zeros((ff, kin), np.float32)
        w[:, :dm] = oracle.normal(s, ff * dm, 0.0, 0.02).reshape(ff, dm)
        return oracle.quantize(c["tg"], w)

    d = oracle.quantize(c["td"], oracle.normal(seed + 2, dm * ff, 0.0, 0.02))
    return gu(seed), gu(seed + 1), d, oracle.normal(seed + 3, dm, 1.0, 0.1)


def cpu_baseline(c, layers_raw, x0, seconds: float):
    """Time the oracle's FFN on all host cores over the sampled layers, for ~`seconds`."""
    import numpy as np

    import oracle

    cores = oracle.get_threads()
    x = x0.copy()
    lb = layer_bytes(c)
    done = 0
    t0 = time.perf_counter()
    while True:
        x[:c["d_model"]] += oracle_layer(c, *layers_raw[done % len(layers_raw)], x)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds and done >= 2:
            break
    gbs = lb * done / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "tokens_per_s": round(done / c["layers"] / el, 4),
            "sample": f"{done} FFN layers ({len(layers_raw)} distinct, {lb / 1e6:.1f} MB each) on the C "
                      f"restatement of the reference CPU path, {el:.1f} s, {cores} OpenMP threads"}, np.isfinite(x).all()


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    world, rank, local = dist_setup(args)
    if rank != 0:
        return 0
    import numpy as np

    import oracle
    from hayai_b200 import _build

    _build.build_oracle()
    c = dict(CONFIGS[args.config])
    if "n_expert" in c:
        return run_reference_moe(args, c, world)
    if c.get("gemv") or c.get("lut"):
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm is timed on the FFN configs; "
                          "the GEMV and LUT configs carry the oracle's CPU baseline in their own line"}))
        return 0
    if args.layers:
        c["layers"] = args.layers
    cores = oracle.get_threads()
    # a few distinct layers of the same shapes, generated on the host with the oracle
    S = 3
    layers = [host_layer(c, 1000 + 4 * l) for l in range(S)]
    x = np.zeros(c["k_in"], np.float32)
    x[:c["d_model"]] = oracle.normal(7, c["d_model"])
    lb = layer_bytes(c)

    def step(i):
        x[:c["d_model"]] = x0[:c["d_model"]] + oracle_layer(c, *layers[i % S], x)

    x0 = x.copy()
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    el = time.perf_counter() - t0
    gbs = lb * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": c_dtype(c),
        "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) activations)",
        "config": {"workload": c["workload"] + f"; reference arm step = 1 FFN layer ({lb / 1e6:.1f} MB)",
                   "batch": 1, "layers": c["layers"], "parallelism": "replicas"},
        "tokens_per_s": round(args.steps / c["layers"] / el, 4),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"1 FFN layer per step, {S} distinct layers rotated, {cores} OpenMP threads; "
                                   "C restatement of the reference Rust CPU path (no Rust toolchain here)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_moe(args, c, world):
    """The reference's CPU MoE path (router, top-k, per-pair expert FFN, combine: the C
    restatement in oracle/) on one MoE layer per step, rank 0 only."""
    import numpy as np

    import oracle

    E, k, T, dm, ff = c["n_expert"], c["top_k"], c["tokens"], c["d_model"], c["d_ff"]
    t = c["tg"]
    cores = oracle.get_threads()
    wg = np.stack([oracle.quantize(t, oracle.normal(5000 + 3 * e, ff * dm, 0.0, 0.02)) for e in range(E)])
    wu = np.stack([oracle.quantize(t, oracle.normal(5001 + 3 * e, ff * dm, 0.0, 0.02)) for e in range(E)])
    wd = np.stack([oracle.quantize(t, oracle.normal(5002 + 3 * e, dm * ff, 0.0, 0.02)) for e in range(E)])
    R = oracle.normal(4999, E * dm, 0.0, 0.02).reshape(E, dm)
    x0 = oracle.normal(7, T * dm).reshape(T, dm)
    x = x0.copy()
    nbytes = []

    def step():
        nonlocal x
        y, ids, _ = oracle.moe_ffn(R, E, k, t, wg, t, wu, t, wd, dm, ff, x)
        nbytes.append(router_bytes(c) + len(np.unique(ids)) * expert_bytes(c))
        x = (x + y).astype(np.float32)

    for _ in range(args.warmup):
        step()
    nbytes.clear()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = sum(nbytes) / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": c_dtype(c),
        "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) activations)",
        "config": {"workload": c["workload"] + "; reference arm step = 1 MoE layer", "batch": T,
                   "layers": c["layers"], "parallelism": "replicas"},
        "tokens_per_s": round(args.steps * T / c["layers"] / el, 4),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"1 MoE layer ({E} experts, top-{k}, {T} tokens) per step, {cores} OpenMP "
                                   "threads; algorithmic bytes = router + distinct experts selected; C restatement "
                                   "of the reference Rust CPU path"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_moe(args):
    """Config 4: the MoE FFN stack, 16 tokens per step through 48 MoE layers
    (x <- x + MoE_l(x)); with --ep the experts are split over the ranks (expert parallelism,
    in-kernel exchange of the routed outputs), otherwise every rank is a replica."""
    import numpy as np
    import torch

    world, rank, local = dist_setup(args)
    result = None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import hayai_b200 as hb
    import oracle
    from hayai_b200.tp import PeerGroup, expert_range

    c = dict(CONFIGS[args.config])
    if args.layers:
        c["layers"] = args.layers
    L, E, k, T, dm, ff, tq = c["layers"], c["n_expert"], c["top_k"], c["tokens"], c["d_model"], c["d_ff"], c["tg"]
    ep = args.ep and world > 1
    lo, hi = expert_range(E, rank, world) if ep else (0, E)
    eng = hb.CudaEngine(local)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    eng.set_stream(stream)

    scratch = torch.empty(ff * dm, dtype=torch.float32, device=dev)

    def synth(t, m, n, seed):
        qk, bs = BLK[t]
        src = scratch[:m * n]
        eng.synth_normal_dev(seed, src, 0.0, 0.02)
        q = torch.empty(m * n // qk * bs, dtype=torch.uint8, device=dev)
        eng.quantize_dev(t, src, q)
        return eng.upload_from_device(t, m, n, q)

    # expert weights seeded by (layer, expert, role): identical wherever an expert lives
    R, G, U, D = [], [], [], []
    for l in range(L):
        r = torch.empty(E, dm, dtype=torch.float32, device=dev)
        eng.synth_normal_dev(9_000_011 * (l + 1), r, 0.0, 0.02)
        R.append(r)
        G.append([synth(tq, ff, dm, 3 * (l * E + e) + 1) for e in range(lo, hi)])
        U.append([synth(tq, ff, dm, 3 * (l * E + e) + 2) for e in range(lo, hi)])
        D.append([synth(c["td"], dm, ff, 3 * (l * E + e) + 3) for e in range(lo, hi)])
    del scratch
    x0 = torch.empty(T, dm, dtype=torch.float32, device=dev)
    eng.synth_normal_dev(7, x0, 0.0, 1.0)
    x = x0.clone()
    y = torch.empty_like(x)
    ids = [torch.empty(T, k, dtype=torch.int32, device=dev) for _ in range(L)]
    peers = PeerGroup(eng) if ep else None
    torch.cuda.synchronize(dev)

    def layers(xx):  # all layers: one graph launch (hc_moe_stack_dev / _ep_dev)
        eng.moe_stack_dev(R, k, G, U, D, xx, expert_lo=lo, ep=ep)

    def step():
        x.copy_(x0)
        layers(x)

    # the routing of every layer (untimed, per-layer calls): algorithmic bytes of a step =
    # every layer's router + the distinct experts its 16 tokens selected (the same every step)
    xr = x0.clone()
    y0 = None
    for l in range(L):
        if ep:
            eng.moe_ffn_ep_dev(R[l], k, G[l], U[l], D[l], lo, xr, y, ids[l])
        else:
            eng.moe_ffn_dev(R[l], k, G[l], U[l], D[l], xr, y, ids[l])
        if l == 0:
            y0 = y.clone()
        xr.add_(y)
    barrier(world)  # expert parallelism: the ranks' combine kernels wait for each other (bounded)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    eng.sync()
    assert torch.allclose(x, xr, rtol=1e-4, atol=1e-3), "graph stack and per-layer calls disagree"
    parity = None
    if rank == 0 and not args.no_parity:
        # layer 0 of the timed model (every expert, wherever it lives: the seeds are per expert)
        # against the C oracle: router + top-k + expert FFNs + combine on the same bytes
        def synth_bytes(t, m, n, seed):
            qk, bs = BLK[t]
            src = torch.empty(m * n, dtype=torch.float32, device=dev)
            eng.synth_normal_dev(seed, src, 0.0, 0.02)
            q = torch.empty(m * n // qk * bs, dtype=torch.uint8, device=dev)
            eng.quantize_dev(t, src, q)
            return q.cpu().numpy()
        wg = np.stack([synth_bytes(tq, ff, dm, 3 * e + 1) for e in range(E)])
        wu = np.stack([synth_bytes(tq, ff, dm, 3 * e + 2) for e in range(E)])
        wd = np.stack([synth_bytes(c["td"], dm, ff, 3 * e + 3) for e in range(E)])
        t0 = time.perf_counter()
        y_ref, ids_ref, _ = oracle.moe_ffn(R[0].cpu().numpy(), E, k, tq, wg, tq, wu, c["td"], wd, dm, ff,
                                          x0.cpu().numpy())
        got = y0.cpu().numpy().astype(np.float64)
        err = got - y_ref.astype(np.float64)
        rel = float(np.linalg.norm(err) / max(np.linalg.norm(y_ref), 1e-30))
        mx = float(np.abs(err).max())
        same_ids = bool(np.array_equal(ids[0].cpu().numpy(), ids_ref))
        parity = {"rel_l2": rel, "max_abs": mx, "ids_bit_exact": same_ids, "layers": 1, "tokens": T,
                  "pass": rel <= 1e-4 and mx <= 1e-3 and same_ids, "tolerance": {"rel_l2": 1e-4, "max_abs": 1e-3},
                  "vs": "oracle/ moe_ffn (C restatement of the reference CPU path) on layer 0's bytes, all experts",
                  "oracle_s": round(time.perf_counter() - t0, 2)}
        del wg, wu, wd
    distinct = [len(np.unique(i.cpu().numpy())) for i in ids]
    step_bytes = L * router_bytes(c) + sum(distinct) * expert_bytes(c)
    barrier(world)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    t_local = ev0.elapsed_time(ev1) / 1e3
    eng.sync()
    t = max_over_ranks(t_local, world, dev)
    barrier(world)
    jobs = 1 if ep else world
    value = jobs * args.steps * step_bytes / t / 1e9

    # roofline: the stack graph (per layer: router, top-k, grouping, two expert-grouped TMA
    # GEMVs, combine) timed alone on its stream, against this rank's algorithmic bytes
    peak, peak_kind = measured_peak()
    reps = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(reps):
        layers(xr)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    k_time = e0.elapsed_time(e1) / 1e3 / reps
    local_experts = [len([e for e in np.unique(i.cpu().numpy()) if lo <= e < hi]) for i in ids]
    k_bytes = L * router_bytes(c) + sum(local_experts) * expert_bytes(c)
    achieved = k_bytes / k_time / 1e9
    roofline = {"bound": "hbm", "kernel": f"MoE stack graph, {L} layers x (router_staged_kernel + "
                "route_group_kernel + moe_tma_kernel<FmtQ4K,true> + moe_tma_kernel<FmtQ4K,false> + "
                + ("ep_signal_kernel + moe_combine_wait_kernel), the expert shard with the in-kernel exchange"
                   if ep else "moe_combine_kernel)"),
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy burst)" if peak_kind == "measured"
                else "fallback 6.65 TB/s", "traffic": committed_traffic(f"moe_{args.config}"),
                "algorithmic_bytes_per_launch": round(k_bytes), "avg_launch_us": round(k_time * 1e6, 2)}

    # e2e: pinned host tokens in, the stack through the device API, the result out, every step
    n_e2e = min(args.steps, 50)
    x_in = x0.cpu().pin_memory()
    x_out = torch.empty_like(x_in).pin_memory()
    barrier(world)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(n_e2e):
        x.copy_(x_in, non_blocking=True)
        layers(x)
        x_out.copy_(x, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    assert torch.isfinite(x_out).all()
    e2e = {"value": round(jobs * n_e2e * step_bytes / t_e2e / 1e9, 2), "unit": "GB/s",
           "tokens_per_s": round(jobs * n_e2e * T / t_e2e, 2), "steps": n_e2e,
           "h2d_bytes_per_step": T * dm * 4, "d2h_bytes_per_step": T * dm * 4,
           "api": "hc_moe_ffn_ep_dev" if ep else "hc_moe_ffn_dev"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "strong" if ep else "weak", "vs_baseline": None, "dtype": c_dtype(c),
            "data": "synthetic (seeded N(0,0.02^2) weights quantized on device, N(0,1) activations)",
            "config": {"workload": c["workload"], "batch": T, "layers": L, "d_model": dm, "d_ff": ff,
                       "n_expert": E, "top_k": k, "distinct_experts_per_layer": round(sum(distinct) / L, 2),
                       "bytes_per_step": step_bytes,
                       "parallelism": f"ep{world} (in-kernel NVLink exchange)" if ep else
                       f"replicas x{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (weights per step %.2f GB > 126 MB)" % (step_bytes / 1e9)},
            "tokens_per_s": round(jobs * args.steps * T / t, 2),
            "frac_of_8tbs": round(value / world / 8000.0, 4),
            "roofline": roofline, "e2e": e2e, "clocks": clocks,
            "gpu_launches": args.steps * L * (7 if ep else 6),  # per rank: router, top-k, grouping, 2 GEMVs, combine (+EP signal)
        }
        if parity is not None:
            line["parity"] = parity
        result = line
    if peers is not None:
        peers.close()
    for group in G + U + D:
        for w in group:
            w.free()
    eng.close()
    return result


def c_dtype(c):
    return {Q4_K: "q4_k/f32", Q6_K: "q6_k/f32", Q8_0: "q8_0/f32"}[c["tg"]] + (
        "+" + {Q4_K: "q4_k", Q6_K: "q6_k", Q8_0: "q8_0"}[c["td"]] if c["td"] != c["tg"] else "")


# ---------------------------------------------------------------- our arm
def run_ours(args):
    import numpy as np
    import torch

    world, rank, local = dist_setup(args)
    result = None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import hayai_b200 as hb

    c = dict(CONFIGS[args.config])
    if args.layers:
        c["layers"] = args.layers
    L, dm, kin, ff, tg, td = c["layers"], c["d_model"], c["k_in"], c["d_ff"], c["tg"], c["td"]
    B = args.batch
    # tensor parallelism: every rank holds a d_ff shard of every layer (gate/up rows, down
    # columns); the down partials are exchanged inside the stack kernel at batch 1, by one
    # all-reduce kernel per layer at batch > 1 (or by NCCL with --tp-impl nccl, the
    # library-collective baseline)
    tp = args.tp and world > 1
    if tp and kin != dm:
        raise SystemExit("--tp runs the stack of an unpadded model")
    ffl = ff // world if tp else ff  # this rank's d_ff
    # the persistent stack kernel serves batch 1 when the FFN input width is d_model (or d_model
    # zero-padded to whole super-blocks)
    padded_ok = kin == dm or (c["tg"] != Q8_0 and kin == -(-dm // 256) * 256)
    uses_stack = B == 1 and padded_ok and (tp or os.environ.get("HAYAI_STACK_KERNEL", "1") != "0")
    if tp and args.tp_impl == "nccl":
        uses_stack = False

    def tensor_core(t, m, k):  # 8..128 rows run on tcgen05: prep + GEMM + slot-sum launches
        if os.environ.get("HAYAI_TC_GEMM", "1") == "0" or not 8 <= B <= 128 or m % 128:
            return False
        return (t == Q8_0 and B >= 9 and k % 128 == 0) or (t in (Q4_K, Q6_K) and k % 256 == 0)

    tc_gu, tc_dn = tensor_core(tg, ffl, kin), tensor_core(td, dm, ffl)
    launches_per_layer = (3 if tc_gu else 1) + (3 if tc_dn else 1) + (1 if tp and args.tp_impl == "ours" else 0)
    eng = hb.CudaEngine(local)
    stream = torch.cuda.Stream(dev)  # one stream for torch's copies, our kernels and the CUDA events
    torch.cuda.set_stream(stream)
    eng.set_stream(stream)

    # ---- resident weights, generated and quantized on the device
    scratch = torch.empty(max(ffl * kin, dm * ffl), dtype=torch.float32, device=dev)
    want_cpu = (rank == 0 and world == 1 and not args.no_cpu_baseline)
    # parity: the whole timed stack when its weights fit the host comfortably (the 8B stack:
    # 3.7 GB), else its first two layers run alone through the same entry point.  Rank 0 keeps
    # the layers' bytes for the CPU oracle; under tensor parallelism it regenerates the other
    # ranks' shards instead (same seeds, same device quantizer: the same bytes).
    parity_on = not args.no_parity and not (tp and args.tp_impl == "nccl")
    whole = L * layer_bytes(c) <= 6e9
    Lp = L if whole else min(L, 2)
    S_cpu = Lp if (parity_on and rank == 0 and not tp) else (3 if want_cpu else 0)
    G, U, D, raw = [], [], [], []
    seed0 = 1_000_003 * (rank + 1)

    padded = torch.zeros(ffl, kin, dtype=torch.float32, device=dev) if kin != dm else None

    def synth(t, m, n, seed, keep, n_real=None):
        """Seeded N(0, 0.02^2) m x n_real weights, zero-padded to n columns, quantized on device."""
        qk, bs = BLK[t]
        n_real = n_real or n
        src = scratch[:m * n_real]
        eng.synth_normal_dev(seed, src, 0.0, 0.02)
        if n_real != n:  # zero-padded K (SmolLM 576 -> 768): pad sub-blocks quantize to exact zeros
            padded[:, :n_real] = src.view(m, n_real)
            src = padded.view(-1)
        q = torch.empty(m * n // qk * bs, dtype=torch.uint8, device=dev)
        eng.quantize_dev(t, src, q)
        rw = eng.upload_from_device(t, m, n, q)
        host = q.cpu().numpy() if keep else None
        del q
        return rw, host

    NW = []  # per-layer RMSNorm weights (ffn_norm), N(1, 0.1^2)
    for l in range(L):
        keep = l < S_cpu
        g, gh = synth(tg, ffl, kin, seed0 + 4 * l, keep, dm)
        u, uh = synth(tg, ffl, kin, seed0 + 4 * l + 1, keep, dm)
        d, dh = synth(td, dm, ffl, seed0 + 4 * l + 2, keep)
        nw = torch.empty(dm, dtype=torch.float32, device=dev)
        # the norm weights and x are replicated: the same seed on every rank under TP
        eng.synth_normal_dev((1_000_003 if tp else seed0) + 4 * l + 3, nw, 1.0, 0.1)
        G.append(g)
        U.append(u)
        D.append(d)
        NW.append(nw)
        if keep:
            raw.append((gh, uh, dh, nw.cpu().numpy()))
    del scratch, padded
    x0 = torch.zeros(B, kin, dtype=torch.float32, device=dev)
    xs = torch.empty(B * dm, dtype=torch.float32, device=dev)
    eng.synth_normal_dev(7 + (0 if tp else rank), xs, 0.0, 1.0)
    x0[:, :dm] = xs.view(B, dm)
    x = x0.clone()
    torch.cuda.synchronize(dev)
    peers = None
    if tp:
        from hayai_b200.tp import PeerGroup

        peers = PeerGroup(eng)

    def run_stack(xx):
        if tp:
            eng.ffn_stack_tp_dev(G, U, D, xx, B, norms=NW, eps=EPS)
        else:
            eng.ffn_stack_dev(G, U, D, xx, B, norms=NW, eps=EPS)

    if tp and args.tp_impl == "nccl":
        import torch.distributed as dist

        h_ws = torch.empty(B, ffl, dtype=torch.float32, device=dev)
        y_ws = torch.empty(B, dm, dtype=torch.float32, device=dev)

        def run_stack(xx):  # noqa: F811 -- per-layer kernels + one NCCL all-reduce per layer
            for l in range(L):
                eng.ffn_gateup_dev(G[l], U[l], xx, h_ws, B, norm=NW[l], norm_len=dm, eps=EPS)
                eng.gemv_dev(D[l], h_ws, y_ws, nvec=B)
                dist.all_reduce(y_ws)
                xx.view(-1).add_(y_ws.view(-1))

    def step():
        x.copy_(x0)
        run_stack(x)

    barrier(world)  # under tensor parallelism the ranks' kernels wait for each other (bounded)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    parity = None
    if parity_on:
        # Every layer is run alone through the same entry point on the GPU's own x_l, and the
        # oracle takes the same x_l: the tolerance is stated per FFN call.  Then row 0 of x_Lp (the
        # timed step's output when the whole stack is checked) against the oracle chained from
        # x_0.  Over the depth the two f32 paths' summation orders drift apart (about 2e-5
        # relative per layer, the size of the oracle's own distance from exact arithmetic), so
        # the chained figure is held to the relative bound.
        def run_sub(xx, lo, hi):
            if tp:
                eng.ffn_stack_tp_dev(G[lo:hi], U[lo:hi], D[lo:hi], xx, B, norms=NW[lo:hi], eps=EPS)
            else:
                eng.ffn_stack_dev(G[lo:hi], U[lo:hi], D[lo:hi], xx, B, norms=NW[lo:hi], eps=EPS)

        def regen(t, m, n, seed):
            qk, bs = BLK[t]
            src = torch.empty(m * n, dtype=torch.float32, device=dev)
            eng.synth_normal_dev(seed, src, 0.0, 0.02)
            q = torch.empty(m * n // qk * bs, dtype=torch.uint8, device=dev)
            eng.quantize_dev(t, src, q)
            return q.cpu().numpy()

        def full_layer(l):  # rank 0: the whole layer's bytes
            if not tp:
                return raw[l]
            gs, us, ds = [], [], []
            for q in range(world):
                s0 = 1_000_003 * (q + 1) + 4 * l
                gs.append(regen(tg, ffl, kin, s0))
                us.append(regen(tg, ffl, kin, s0 + 1))
                ds.append(regen(td, dm, ffl, s0 + 2).reshape(dm, -1))  # column shards of each row
            return (np.concatenate(gs), np.concatenate(us), np.hstack(ds).reshape(-1), NW[l].cpu().numpy())

        xin = x0.clone()
        xr = x0[0].cpu().numpy().copy()
        worst_rel = worst_abs = 0.0
        t_or = 0.0
        for l in range(Lp):
            xl = xin[0].cpu().numpy().copy()
            # the ranks' kernels wait (bounded, ~1 s) for each other inside the exchange: start
            # them together, not while rank 0 is still busy with the oracle of the last layer
            barrier(world)
            run_sub(xin, l, l + 1)
            if rank == 0:
                w = full_layer(l)
                t0 = time.perf_counter()
                yl = xl.copy()
                yl[:dm] += oracle_layer(c, *w, xl)
                xr[:dm] += oracle_layer(c, *w, xr)
                t_or += time.perf_counter() - t0
                el = xin[0, :dm].cpu().numpy().astype(np.float64) - yl[:dm].astype(np.float64)
                worst_rel = max(worst_rel, float(np.linalg.norm(el) / max(np.linalg.norm(yl[:dm]), 1e-30)))
                worst_abs = max(worst_abs, float(np.abs(el).max()))
        torch.cuda.synchronize(dev)
        if rank == 0:
            got = (x if whole else xin)[0, :dm].cpu().numpy().astype(np.float64)
            ref = xr[:dm].astype(np.float64)
            err = got - ref
            rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
            mx = float(np.abs(err).max())
            per_ok = worst_rel <= 1e-4 and worst_abs <= 1e-3
            parity = {"rel_l2": rel, "max_abs": mx, "layers": Lp, "of_layers": L, "row": 0,
                      "checked": "the timed stack's output" if whole else f"the first {Lp} layers run alone",
                      "per_layer": {"worst_rel_l2": worst_rel, "worst_max_abs": worst_abs, "pass": per_ok},
                      "pass": per_ok and rel <= 1e-4,
                      "tolerance": {"rel_l2": 1e-4, "max_abs": 1e-3,
                                    "applies_to": "each FFN call (every layer); rel_l2 also over the chain"},
                      "vs": "oracle/ (C restatement of the reference CPU path, f32) on the same weight bytes"
                            + (f", every rank's shards joined ({world} ranks)" if tp else ""),
                      "oracle_s": round(t_or, 2)}
    barrier(world)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    t_local = ev0.elapsed_time(ev1) / 1e3
    eng.sync()  # surfaces any device-side error flag
    t = max_over_ranks(t_local, world, dev)
    barrier(world)
    tok_bytes = L * layer_bytes(c)  # the whole model's weights per token (all shards under TP)
    jobs = 1 if tp else world       # TP: one token stream over all ranks; else independent replicas
    value = jobs * args.steps * tok_bytes / t / 1e9
    tokens_per_s = jobs * args.steps * B / t

    # ---- roofline of the dominant kernel, timed with CUDA events on the stream it runs on.
    # Batch 1 with uniform layers runs the whole stack as one persistent kernel per step
    # (ffn_stack.cu); otherwise the fused gate/up GEMV is the largest kernel of a layer.
    peak, peak_kind = measured_peak()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    names = {Q4_K: "FmtQ4K", Q6_K: "FmtQ6K", Q8_0: "FmtQ80"}
    if uses_stack:
        reps = max(3, min(args.steps, 20))
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(reps):
            run_stack(x)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        k_time = e0.elapsed_time(e1) / 1e3 / reps
        k_bytes = tok_bytes // world if tp else tok_bytes  # this GPU's shard under TP
        flow = not tp and td == Q6_K and os.environ.get("HAYAI_FLOW_KERNEL", "1") != "0" and kin == dm
        kname = f"{'ffn_flow_kernel' if flow else 'ffn_stack_kernel'}<{names[tg]},{names[td]}> (all {L} layers, " + \
            "one launch" + (f", d_ff shard 1/{world} + in-kernel exchange)" if tp else ")")
        kkey = f"stack_{args.config}_L{L}" + (f"_tp{world}" if tp else "")
    else:
        h = torch.empty(B, ffl, dtype=torch.float32, device=dev)
        reps = 3 * L if L >= 8 else 96
        for i in range(L):
            eng.ffn_gateup_dev(G[i % L], U[i % L], x0, h, B, norm=NW[i % L], norm_len=dm, eps=EPS)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for i in range(reps):
            eng.ffn_gateup_dev(G[i % L], U[i % L], x0, h, B, norm=NW[i % L], norm_len=dm, eps=EPS)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        k_time = e0.elapsed_time(e1) / 1e3 / reps
        k_bytes = 2 * mat_bytes(tg, ffl, kin)
        kname = ("tc_prep_kernel (RMSNorm, f16 hi/lo) + tc_gemm_kernel (tcgen05, gate and up) + "
                 "tc_finish_kernel (split sums, SiLU*up)" if tc_gu else
                 f"gemv_tma_kernel<{names[tg]},{min(B, 4)},true> (fused gate/up + SiLU*up)")
        kkey = f"gateup_{args.config}_b{B}"
    achieved = k_bytes / k_time / 1e9
    roofline = {"bound": "hbm", "kernel": kname,
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy burst)" if peak_kind == "measured"
                else "fallback 6.65 TB/s",
                "traffic": committed_traffic(kkey), "algorithmic_bytes_per_launch": k_bytes,
                "avg_launch_us": round(k_time * 1e6, 2)}

    # ---- e2e through the host C-ABI call: pinned host x in, result out, every step
    n_e2e = min(args.steps, 200)
    x_in = torch.empty(B * kin, dtype=torch.float32).pin_memory()
    x_in.copy_(x0.view(-1).cpu())
    x_out = torch.empty_like(x_in).pin_memory()
    xi, xo = x_in.numpy(), x_out.numpy()

    # the stack bound once (weights and norms marshalled at binding), then one call per step
    bound = None if (tp and args.tp_impl != "ours") else eng.bind_ffn_stack(G, U, D, norms=NW, eps=EPS, tp=tp)

    def host_call():
        if bound is None:  # NCCL baseline: the same per-layer loop on a device copy of the host vector
            xd = torch.from_numpy(xi).to(dev, non_blocking=True)
            run_stack(xd)
            return xd.cpu().numpy()
        return bound.run(xi, xo, B)

    for _ in range(3):
        host_call()
    barrier(world)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(n_e2e):
        r = host_call()
        if r is not xo:
            xo[:] = r
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    e2e = {"value": round(jobs * n_e2e * tok_bytes / t_e2e / 1e9, 2), "unit": "GB/s",
           "tokens_per_s": round(jobs * n_e2e * B / t_e2e, 2), "steps": n_e2e,
           "h2d_bytes_per_step": B * kin * 4, "d2h_bytes_per_step": B * kin * 4,
           "api": ("CudaEngine.bind_ffn_stack(..., tp=True).run -> hc_ffn_stack_tp" if tp and args.tp_impl == "ours" else
                   "per-layer kernels + torch.distributed all_reduce" if tp else
                   "CudaEngine.bind_ffn_stack(...).run -> hc_ffn_stack") + " (host buffers)"}
    assert np.isfinite(xo).all()

    # ---- the per-layer path beside the persistent kernel (rank 0, unsharded, unpadded): the
    # same layers as per-layer kernels replayed from one captured CUDA graph (the path batches
    # take), and launched eagerly one call at a time
    per_layer = None
    if rank == 0 and not tp and kin == dm and not args.no_per_layer:
        os.environ["HAYAI_STACK_KERNEL"] = "0"
        try:
            eng2 = hb.CudaEngine(local)
        finally:
            os.environ.pop("HAYAI_STACK_KERNEL", None)
        eng2.set_stream(stream)
        reps = max(3, min(args.steps, 20))
        xg = x0.clone()

        def graph_step():
            xg.copy_(x0)
            eng2.ffn_stack_dev(G, U, D, xg, B, norms=NW, eps=EPS)

        hh = torch.empty(B, ffl, dtype=torch.float32, device=dev)
        xa, xb = x0.clone(), torch.empty_like(x0)

        def eager_step():
            cur, nxt = xa, xb
            cur.copy_(x0)
            for l in range(L):
                eng2.ffn_gateup_dev(G[l], U[l], cur, hh, B, norm=NW[l], norm_len=dm, eps=EPS)
                eng2.gemv_dev(D[l], hh, nxt, resid=cur, nvec=B)
                cur, nxt = nxt, cur

        timings = {}
        for name, fn in (("graph", graph_step), ("eager", eager_step)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize(dev)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            timings[name] = e0.elapsed_time(e1) / reps
        eng2.sync()
        per_layer = {"graph_ms_per_step": round(timings["graph"], 4), "eager_ms_per_step": round(timings["eager"], 4),
                     "persistent_ms_per_step": round(t / args.steps * 1e3, 4),
                     "graph_GBps": round(tok_bytes / (timings["graph"] / 1e3) / 1e9, 1),
                     "eager_GBps": round(tok_bytes / (timings["eager"] / 1e3) / 1e9, 1),
                     "kernels_per_layer": launches_per_layer,
                     "note": "same weights and parity contract; graph = the per-layer kernels captured once and "
                             "replayed (hc_ffn_stack_dev with the stack kernel off), eager = one C-ABI call per "
                             "GEMV; both include a copy of x_0 per step"}
        del eng2

    cpu = None
    if want_cpu:
        x_np = x0[0].cpu().numpy()
        cpu, ok = cpu_baseline(c, raw[:3], x_np, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": c_dtype(c),
            "data": "synthetic (seeded N(0,0.02^2) weights quantized on device, N(0,1) activations)",
            "config": {"workload": c["workload"].replace("batch-1 decode", f"batch {B}") if B > 1 else c["workload"],
                       "batch": B, "layers": L, "d_model": dm, "d_ff": ff,
                       "kernel_path": "persistent stack kernel" if uses_stack else
                       "per-layer kernels" + (" (tcgen05 GEMM)" if tc_gu or tc_dn else ""),
                       "bytes_per_token": tok_bytes,
                       "parallelism": (f"tp{world} ({'in-kernel NVLink exchange' if args.tp_impl == 'ours' else 'NCCL all_reduce'})"
                                       if tp else f"replicas x{world}" if world > 1 else "single"),
                       "l2": "inputs larger than L2 (weights per step %.2f GB > 126 MB)" % (tok_bytes / 1e9)},
            "tokens_per_s": round(tokens_per_s, 2),
            "frac_of_8tbs": round(value / world / 8000.0, 4),  # per GPU
            "roofline": roofline, "e2e": e2e, "clocks": clocks,
            "gpu_launches": args.steps * (1 if uses_stack else launches_per_layer * L),  # per rank
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if parity is not None:
            line["parity"] = parity
        if per_layer is not None:
            line["per_layer_path"] = per_layer
        result = line
    if peers is not None:
        peers.close()
    for w in G + U + D:
        w.free()
    eng.close()
    return result


def run_gemv(args):
    """One GEMV of the config's format per step (batch 1), rotating over resident copies."""
    import numpy as np
    import torch

    import hayai_b200 as hb

    c = CONFIGS[args.config]
    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    t, M, K = c["t"], c["m"], c["k"]
    mbytes = mat_bytes(t, M, K)
    copies = max(2, -(-400_000_000 // mbytes))  # > L2 between reuses of one copy
    eng = hb.CudaEngine(local)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    eng.set_stream(stream)
    W, raw = [], None
    for i in range(copies):
        if t in (Q4_K, Q6_K, Q8_0):
            src = torch.empty(M * K, dtype=torch.float32, device=dev)
            eng.synth_normal_dev(1000 + i, src, 0.0, 0.02)
            q = torch.empty(mbytes, dtype=torch.uint8, device=dev)
            eng.quantize_dev(t, src, q)
            W.append(eng.upload_from_device(t, M, K, q))
            if i == 0:
                raw = q.cpu().numpy()
            del src, q
        else:
            hb_bytes = random_blocks(t, M, K, 1000 + i)
            W.append(eng.upload(t, M, K, hb_bytes))
            if i == 0:
                raw = hb_bytes
    x = torch.randn(K, device=dev)
    y = torch.empty(M, device=dev)
    torch.cuda.synchronize(dev)
    for i in range(max(args.warmup, 3)):
        eng.gemv_dev(W[i % copies], x, y)
    torch.cuda.synchronize(dev)
    barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        eng.gemv_dev(W[i % copies], x, y)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    eng.sync()
    t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    value = world * args.steps * mbytes / t_dev / 1e9
    peak, peak_kind = measured_peak()
    # e2e: host x in, host y out through the reference-facing call, every step
    xh = x.cpu().numpy()
    n_e2e = min(args.steps, 100)
    for i in range(3):
        eng.ggml_gemv_dispatch_bound(W[i % copies], xh)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    e0.record(stream)
    for i in range(n_e2e):
        yh = eng.ggml_gemv_dispatch_bound(W[i % copies], xh)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    assert np.isfinite(yh).all()
    parity = None
    if rank == 0 and not args.no_parity:
        # the first 2048 rows of the timed matrix (copy 0) against the C oracle on the same bytes
        import oracle

        prow = min(M, 2048)
        eng.gemv_dev(W[0], x, y)
        got = y[:prow].double().cpu().numpy()
        ref = np.asarray(oracle.gemv(t, prow, K, raw[:prow * mbytes // M], xh.astype(np.float32)), np.float64)
        rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
        mx = float(np.abs(got - ref).max())
        parity = {"rel_l2": rel, "max_abs": mx, "rows": prow, "of_rows": M, "pass": rel <= 1e-4 and mx <= 1e-3}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        rows = 2048
        xr = xh.astype(np.float32)
        done, t0 = 0, time.perf_counter()
        while True:
            oracle.gemv(t, rows, K, raw[:rows * mbytes // M], xr)
            done += 1
            el = time.perf_counter() - t0
            if el >= min(args.cpu_seconds, 10.0) and done >= 2:
                break
        cpu = {"value": round(done * rows * mbytes / M / el / 1e9, 3), "unit": "GB/s", "cores": oracle.get_threads(),
               "kind": "port", "sample": f"{done} GEMVs of the first {rows} rows on the C restatement, {el:.1f} s"}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(t_dev / args.steps * 1e3, 5), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": args.config[len("gemv-"):] + "/f32",
                "data": "synthetic (random valid blocks, or seeded N(0,0.02^2) weights quantized on device)",
                "config": {"workload": c["workload"], "m": M, "k": K, "copies": copies,
                           "l2": f"inputs larger than L2 ({copies} copies of {mbytes / 1e6:.1f} MB rotated)"},
                "roofline": {"bound": "hbm", "kernel": "GEMV (one launch)", "achieved": round(value / world, 1),
                             "peak": peak, "unit": "GB/s", "frac": round(value / world / peak, 4),
                             "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy burst)",
                             "traffic": None, "algorithmic_bytes_per_launch": mbytes,
                             "avg_launch_us": round(t_dev / args.steps * 1e6, 2)},
                "e2e": {"value": round(world * n_e2e * mbytes / t_e2e / 1e9, 2), "unit": "GB/s", "steps": n_e2e,
                        "h2d_bytes_per_step": K * 4, "d2h_bytes_per_step": M * 4,
                        "api": "ggml_gemv_dispatch_bound (host buffers)"},
                "clocks": clocks, "gpu_launches": args.steps}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if parity is not None:
            line["parity"] = parity
        print(json.dumps(line))
    for w in W:
        w.free()
    eng.close()
    return 0


def run_lut(args):
    """The `hayai bench` LUT-Q4 matmul.  value: device-timed, rotating copies past L2 (the HBM
    figure); e2e: the reference's own bench loop, one host-buffer call per step on the same
    442 KB of weights (cache-resident, as in the reference), also reported as GFLOP/s."""
    import numpy as np
    import torch

    import hayai_b200 as hb

    c = CONFIGS[args.config]
    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    M, N = c["m"], c["n"]
    wbytes = M * N // 2
    copies = -(-400_000_000 // wbytes)
    eng = hb.CudaEngine(local)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    eng.set_stream(stream)
    W = torch.full((copies, wbytes), 0xAB, dtype=torch.uint8, device=dev)
    lut = torch.tensor(LUT16, dtype=torch.float32, device=dev)
    x = torch.ones(N, dtype=torch.float32, device=dev)
    y = torch.empty(M, dtype=torch.float32, device=dev)
    for i in range(max(args.warmup, 3)):
        eng.lut_matmul_q4_dev(M, N, W[i % copies], lut, x, y)
    torch.cuda.synchronize(dev)
    # a launch from Python takes longer than the kernel: the device figure replays the
    # launches from a CUDA graph (per_graph launches over rotating copies)
    per_graph = min(args.steps, 100)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(per_graph):
            eng.lut_matmul_q4_dev(M, N, W[i % copies], lut, x, y)
    reps = max(1, args.steps // per_graph)
    graph.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    eng.sync()
    launches = reps * per_graph
    t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    value = world * launches * wbytes / t_dev / 1e9
    wh = np.full(wbytes, 0xAB, np.uint8)
    lh, xh = np.asarray(LUT16, np.float32), np.ones(N, np.float32)
    for _ in range(5):
        yh = eng.lut_matmul_q4(M, N, wh, lh, xh)
    n_e2e = 500
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(n_e2e):
        yh = eng.lut_matmul_q4(M, N, wh, lh, xh)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    assert np.isfinite(yh).all()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        done, t0 = 0, time.perf_counter()
        while True:
            oracle.lut_matmul_q4(M, N, wh, lh, xh)
            done += 1
            el = time.perf_counter() - t0
            if el >= min(args.cpu_seconds, 5.0) and done >= 2:
                break
        cpu = {"value": round(done * wbytes / el / 1e9, 3), "unit": "GB/s", "cores": oracle.get_threads(),
               "kind": "port", "gflops": round(done * 2 * M * N / el / 1e9, 3),
               "sample": f"{done} calls of the C restatement of cpu_lut_matmul_q4, {el:.1f} s"}
    peak, peak_kind = measured_peak()
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": launches,
                "warmup": args.warmup, "ms_per_step": round(t_dev / launches * 1e3, 5), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "lut-q4/f32",
                "data": "synthetic (the reference bench's constant weights, LUT and input)",
                "config": {"workload": c["workload"], "m": M, "n": N, "copies": copies,
                           "l2": f"inputs larger than L2 ({copies} copies of {wbytes / 1e3:.0f} KB rotated)"},
                "roofline": {"bound": "hbm", "kernel": "lut_q4_kernel (one launch)", "achieved": round(value / world, 1),
                             "peak": peak, "unit": "GB/s", "frac": round(value / world / peak, 4),
                             "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy burst)",
                             "traffic": None, "algorithmic_bytes_per_launch": wbytes,
                             "avg_launch_us": round(t_dev / launches * 1e6, 2), "gflops": round(
                                 world * launches * 2 * M * N / t_dev / 1e9, 2)},
                "e2e": {"value": round(world * n_e2e * wbytes / t_e2e / 1e9, 2), "unit": "GB/s", "steps": n_e2e,
                        "gflops": round(world * n_e2e * 2 * M * N / t_e2e / 1e9, 2),
                        "h2d_bytes_per_step": wbytes + 16 * 4 + N * 4, "d2h_bytes_per_step": M * 4,
                        "api": "hc_lut_matmul_q4 (host buffers, as the reference bench calls execute_lut_matmul)"},
                "clocks": clocks, "gpu_launches": launches, "timing": "CUDA graph replay of the launches"}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line))
    del graph, W
    eng.close()
    return 0


def nvlink_bytes_per_layer(name, a, world):
    """Bytes one rank stores into its peers' exchange regions per layer (the in-kernel exchange),
    0 with one GPU."""
    if world == 1:
        return 0
    c = CONFIGS[a.config]
    if name.startswith("tp"):
        if a.batch == 1:  # every down chunk's 16 partial sums go to every rank (16-block chunks)
            nbk = c["d_ff"] // world // 256
            return (world - 1) * c["d_model"] * (-(-nbk // 16)) * 4
        return (world - 1) * a.batch * c["d_model"] * 4  # the all-reduce kernel's slices
    # EP: each routed row computed here goes to every other rank (T k / P rows on average)
    return round((world - 1) * c["tokens"] * c["top_k"] / world * c["d_model"] * 4)


def run_sharded(args):
    """The two configs that shard (BASELINE configs[4] and [3]) at this run's GPU count: the
    Llama-3-70B FFN stack tensor-parallel over the ranks at batch 1 and 16, and the Qwen3-30B-A3B
    MoE stack expert-parallel.  With one GPU they run unsharded (the start of each curve).
    Returns {name: summary} on rank 0."""
    world, rank, local = dist_setup(args)
    peak, _ = measured_peak()
    out = {}
    base = dict(vars(args))
    for name, kw in (("tp_llama70b_b1", dict(config="llama70b", tp=True, ep=False, batch=1, steps=20)),
                     ("tp_llama70b_b16", dict(config="llama70b", tp=True, ep=False, batch=16, steps=6)),
                     ("ep_qwen3moe", dict(config="qwen3moe", tp=False, ep=True, batch=1, steps=20))):
        a = argparse.Namespace(**{**base, **kw, "warmup": 3, "layers": 0, "no_cpu_baseline": True,
                                  "no_parity": False, "no_per_layer": True, "tp_impl": "ours"})
        try:
            line = (run_moe if "n_expert" in CONFIGS[a.config] else run_ours)(a)
        except Exception as exc:  # the headline line is still printed; the failure is reported
            if rank == 0:
                out[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            print(f"sharded {name} failed on rank {rank}: {exc}", file=sys.stderr)
            break  # a failed collective may leave the ranks out of step: no further sharded runs
        barrier(world)
        if rank == 0 and line:
            out[name] = {"value": line["value"], "unit": "GB/s", "ms_per_step": line["ms_per_step"],
                         "tokens_per_s": line["tokens_per_s"],
                         "per_gpu_hbm_frac": round(line["value"] / world / peak, 4),
                         "workload": line["config"]["workload"], "batch": line["config"]["batch"],
                         "parallelism": line["config"]["parallelism"], "scaling": line["scaling"],
                         "nvlink_bytes_per_layer_per_gpu": nvlink_bytes_per_layer(name, a, world),
                         "kernel_path": line["config"].get("kernel_path"), "roofline": line["roofline"],
                         "e2e": line["e2e"]}
            if "parity" in line:
                out[name]["parity"] = line["parity"]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="llama8b")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="override the config's layer count (small profiling case)")
    ap.add_argument("--tp", action="store_true", help="tensor-parallel d_ff split over the ranks (any --batch)")
    ap.add_argument("--tp-impl", choices=["ours", "nccl"], default="ours",
                    help="exchange of the down partials: in-kernel NVLink stores, or NCCL all_reduce per layer")
    ap.add_argument("--ep", action="store_true", help="expert-parallel MoE over the ranks (qwen3moe)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed stack's output")
    ap.add_argument("--no-per-layer", action="store_true",
                    help="skip the per-layer path timing (CUDA graph replay and eager launches)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sharded configs (70B tensor-parallel, Qwen3 expert-parallel) the default "
                         "llama8b run also measures at the same GPU count")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    world, rank, local = dist_setup(args)
    import torch

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        c = CONFIGS[args.config]
        if c.get("gemv"):
            return run_gemv(args)
        if c.get("lut"):
            return run_lut(args)
        line = run_moe(args) if "n_expert" in c else run_ours(args)
        if (args.config == "llama8b" and not args.tp and args.batch == 1 and not args.layers
                and not args.no_sharded):
            # the headline line also carries the sharded configs at the same GPU count
            barrier(world)
            sharded = run_sharded(args)
            if rank == 0:
                line["sharded"] = sharded
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
