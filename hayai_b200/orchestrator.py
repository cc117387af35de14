"""Mirror of hayai-core's op dispatch for the CUDA backend: per-op bindings, the planner's
placement and the orchestrator's GEMV entry points, over the native library.

Reference: ``EngineOrchestrator`` (crates/hayai-core/src/orchestrator.rs:55-480), the
per-op hardware bindings ``OpBinding`` / ``op_binding`` (crates/hayai-core/src/exec_plan.rs:
16-216), and the planner's ``ComputeTarget`` placement (crates/hayai-core/src/planner.rs:19-30).

What this backend changes, on purpose:

* Every op that computes runs on a GPU of the pool.  The reference keeps the ops its static
  table binds to the CPU (router, attention projections, norms) on the host even when a GPU
  pool exists; here they run on the GPU too -- the backend has no CPU path, and the MoE
  router's scores are bit-exact on the GPU (one sequential f32 chain per (token, expert)).
* There is no CPU fallback anywhere: a quant type without a CUDA kernel, a planner placement
  on the CPU and an empty device pool are errors (the reference's own rule for a GPU host,
  orchestrator.rs:403-409), never a silent host computation.
* ``execute_op_bound`` / ``submit_op_bound`` run from the matrix's resident HBM copy, which
  plays the role of the reference's per-layer device mirror (``StreamingScratch``): weights
  are uploaded once per device and reused by every later op on that matrix.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Mapping, Sequence

import numpy as np

from .engine import TYPE_LABELS, CudaEngine, CudaError, PendingGemv, QuantMatrix, ResidentWeights, _lib


class LayerOpKind(enum.Enum):
    """Op roles of a layer (exec_plan.rs:16-130)."""
    TokenEmbed = enum.auto()
    TokenEmbedNorm = enum.auto()
    PositionEmbed = enum.auto()
    OutputNorm = enum.auto()
    OutputProj = enum.auto()
    AttnNorm = enum.auto()
    AttnQ = enum.auto()
    AttnK = enum.auto()
    AttnV = enum.auto()
    AttnO = enum.auto()
    AttnGate = enum.auto()
    MlaQa = enum.auto()
    MlaQaNorm = enum.auto()
    MlaQb = enum.auto()
    MlaKvA = enum.auto()
    MlaKvANorm = enum.auto()
    MlaKb = enum.auto()
    MlaVb = enum.auto()
    MlaKvB = enum.auto()
    EncOutputNorm = enum.auto()
    DecOutputNorm = enum.auto()
    CrossAttnQ = enum.auto()
    CrossAttnK = enum.auto()
    CrossAttnV = enum.auto()
    CrossAttnO = enum.auto()
    CrossAttnNorm = enum.auto()
    RelPosBias = enum.auto()
    AttnQkv = enum.auto()
    AttnQNorm = enum.auto()
    AttnKNorm = enum.auto()
    PostAttnNorm = enum.auto()
    FfnNorm = enum.auto()
    FfnGate = enum.auto()
    FfnUp = enum.auto()
    FfnDown = enum.auto()
    FfnGateUp = enum.auto()
    FfnDagAdjacency = enum.auto()
    FfnDagWeights = enum.auto()
    PostFfnNorm = enum.auto()
    LayerOutputScale = enum.auto()
    Router = enum.auto()
    RouterBias = enum.auto()
    RouterScale = enum.auto()
    ExpertScale = enum.auto()
    ExpertGate = enum.auto()
    ExpertUp = enum.auto()
    ExpertDown = enum.auto()
    ExpertGateUp = enum.auto()
    SharedExpert = enum.auto()
    DeltaNet = enum.auto()
    Mamba = enum.auto()
    NextN = enum.auto()
    PleEmbed = enum.auto()
    PleModelProj = enum.auto()
    PleProjNorm = enum.auto()
    PleGate = enum.auto()
    PleProj = enum.auto()
    PlePostNorm = enum.auto()
    Recurrence = enum.auto()
    Conv = enum.auto()
    Aux = enum.auto()


class OpDevice(enum.Enum):
    """Hardware class an op is bound to (exec_plan.rs:131-140)."""
    Cpu = "CPU"
    GpuAsync = "GPU-async"
    HostRowRead = "HOST-row"
    Discard = "discard"


class OpKernel(enum.Enum):
    Gemv = enum.auto()
    GemvAsync = enum.auto()
    RmsNorm = enum.auto()
    Row = enum.auto()
    Nothing = enum.auto()  # the reference's OpKernel::None


@dataclass(frozen=True)
class OpBinding:
    device: OpDevice
    kernel: OpKernel


CPU_GEMV = OpBinding(OpDevice.Cpu, OpKernel.Gemv)
CPU_NORM = OpBinding(OpDevice.Cpu, OpKernel.RmsNorm)
GPU_ASYNC = OpBinding(OpDevice.GpuAsync, OpKernel.GemvAsync)
HOST_ROW = OpBinding(OpDevice.HostRowRead, OpKernel.Row)
DISCARD = OpBinding(OpDevice.Discard, OpKernel.Nothing)

_K = LayerOpKind
# The static binding table (exec_plan.rs:192-216): data, kept identical to the reference's.
_BINDINGS = {}
for _k in (_K.TokenEmbed, _K.PleEmbed, _K.PositionEmbed):
    _BINDINGS[_k] = HOST_ROW
for _k in (_K.OutputNorm, _K.AttnNorm, _K.AttnQNorm, _K.AttnKNorm, _K.PostAttnNorm, _K.FfnNorm, _K.PostFfnNorm,
           _K.PleProjNorm, _K.PlePostNorm, _K.TokenEmbedNorm, _K.MlaQaNorm, _K.MlaKvANorm):
    _BINDINGS[_k] = CPU_NORM
for _k in (_K.AttnQ, _K.AttnK, _K.AttnV, _K.AttnO, _K.AttnGate, _K.AttnQkv, _K.PleGate, _K.PleProj, _K.Router,
           _K.DeltaNet, _K.Mamba, _K.NextN, _K.Recurrence, _K.Conv, _K.MlaQa, _K.MlaQb, _K.MlaKvA, _K.MlaKb,
           _K.MlaVb, _K.MlaKvB, _K.CrossAttnQ, _K.CrossAttnK, _K.CrossAttnV, _K.CrossAttnO):
    _BINDINGS[_k] = CPU_GEMV
for _k in (_K.FfnGate, _K.FfnUp, _K.FfnDown, _K.FfnGateUp, _K.ExpertGate, _K.ExpertUp, _K.ExpertDown,
           _K.ExpertGateUp, _K.SharedExpert, _K.OutputProj, _K.PleModelProj, _K.FfnDagAdjacency,
           _K.FfnDagWeights):
    _BINDINGS[_k] = GPU_ASYNC
for _k in (_K.LayerOutputScale, _K.Aux, _K.RouterBias, _K.RouterScale, _K.ExpertScale, _K.EncOutputNorm,
           _K.DecOutputNorm, _K.CrossAttnNorm, _K.RelPosBias):
    _BINDINGS[_k] = DISCARD
assert len(_BINDINGS) == len(LayerOpKind)


def op_binding(kind: LayerOpKind) -> OpBinding:
    """Hardware binding per op (exec_plan.rs:192-216)."""
    return _BINDINGS[kind]


@dataclass(frozen=True)
class ComputeTarget:
    """The planner's placement of an op (planner.rs:19-30): ``device`` None = the CPU."""
    device: int | None = None

    @staticmethod
    def cpu() -> "ComputeTarget":
        return ComputeTarget(None)

    @staticmethod
    def dev(i: int) -> "ComputeTarget":
        return ComputeTarget(int(i))

    def __str__(self) -> str:
        return "CPU" if self.device is None else f"dev{self.device}"


class OpPending:
    """Handle of an op submitted with ``submit_op_bound`` (orchestrator.rs:36-53): in flight on
    a device (``wait()`` joins it and returns the output) or already done inline (``wait()``
    returns None and the caller's output buffer holds the result)."""

    def __init__(self, pending: PendingGemv | None):
        self._pending = pending

    @property
    def done(self) -> bool:
        return self._pending is None

    def wait(self) -> np.ndarray | None:
        if self._pending is None:
            return None
        p, self._pending = self._pending, None
        return p.wait()


# ggml types with a CUDA GEMV in this backend (the match of orchestrator.rs:72-98 for this arm)
_CUDA_GEMV_TYPES = frozenset(TYPE_LABELS)


def gemv_kernel(ggml_type: int) -> str | None:
    """Label of the CUDA GEMV for a quant type, None when the backend has none
    (orchestrator.rs:72-98; the None case is a hard error on a GPU host)."""
    return TYPE_LABELS[ggml_type] if ggml_type in _CUDA_GEMV_TYPES else None


def _missing(ggml_type: int) -> CudaError:
    return CudaError(_lib.HC_ERR_UNSUPPORTED,
                     f"CUDA GEMV missing for ggml type {ggml_type} -- GPU present, CPU fallback disabled")


class EngineOrchestrator:
    """GPU-only dispatch of the FFN-path GEMVs over a pool of CUDA engines (one per device).

    Matrices are uploaded once per device on first use and stay resident; ``close()``
    releases them with the engines.  Like the reference's, an orchestrator is used by one
    thread at a time (callers serialise it, orchestrator.rs:65-68)."""

    def __init__(self, devices: Sequence[int] = (0,)):
        if not devices:
            raise CudaError(_lib.HC_ERR_INVALID, "empty device pool: this backend has no CPU path")
        self.pool = [CudaEngine(d) for d in devices]
        self._placement: dict[LayerOpKind, ComputeTarget] = {}
        # (id(matrix), pool index) -> (matrix, resident copy); holding the matrix keeps its id unique
        self._resident_cache: dict[tuple[int, int], tuple[QuantMatrix, ResidentWeights]] = {}
        self.gemv_calls = [0] * len(self.pool)

    # ---------------------------------------------------------------- pool and placement
    @property
    def engine(self) -> CudaEngine:
        """The primary (first) device of the pool."""
        return self.pool[0]

    def for_role(self, role: int) -> CudaEngine:
        """Device for an FFN role (gate 0, up 1, down 2): round-robin over the pool."""
        return self.pool[role % len(self.pool)]

    def set_placement(self, placement: Mapping[LayerOpKind, ComputeTarget]) -> None:
        """Install the planner's cost-driven placement (orchestrator.rs:177-180)."""
        self._placement = dict(placement)

    def placed_target(self, kind: LayerOpKind) -> ComputeTarget | None:
        return self._placement.get(kind)

    def using_gpu(self) -> bool:
        return True

    def ffn_device_name(self) -> str:
        return f"cuda:{self.pool[0].device}"

    def format_compute_plan(self) -> str:
        """Role -> device assignment and per-device GEMV counts (orchestrator.rs:444-470)."""
        lines = ["Compute plan (FFN roles):"]
        for role, name in enumerate(("gate", "up", "down")):
            lines.append(f"  {name:<5} -> cuda:{self.for_role(role).device}")
        for i, e in enumerate(self.pool):
            lines.append(f"  cuda:{e.device}: {self.gemv_calls[i]} FFN GEMVs")
        return "\n".join(lines) + "\n"

    # ---------------------------------------------------------------- residency
    def resident(self, matrix: QuantMatrix, idx: int = 0) -> ResidentWeights:
        """The matrix's HBM copy on pool device ``idx`` (uploaded on first use)."""
        key = (id(matrix), idx)
        hit = self._resident_cache.get(key)
        if hit is None or hit[0] is not matrix:
            if gemv_kernel(matrix.ggml_type) is None:
                raise _missing(matrix.ggml_type)
            rw = self.pool[idx].upload(matrix.ggml_type, matrix.nrows, matrix.ncols, matrix.data)
            self._resident_cache[key] = (matrix, rw)
            return rw
        return hit[1]

    def evict(self, matrix: QuantMatrix) -> None:
        """Free every resident copy of a matrix."""
        for key in [k for k in self._resident_cache if k[0] == id(matrix)]:
            self._resident_cache.pop(key)[1].free()

    def close(self) -> None:
        for _, rw in self._resident_cache.values():
            rw.free()
        self._resident_cache.clear()
        for e in self.pool:
            e.close()
        self.pool = []

    # ---------------------------------------------------------------- GEMVs
    def _gpu_gemv(self, idx: int, matrix: QuantMatrix, input, output=None) -> np.ndarray:
        if not 0 <= idx < len(self.pool):
            raise CudaError(_lib.HC_ERR_INVALID, f"placed device {idx} not in pool")
        rw = self.resident(matrix, idx)
        self.gemv_calls[idx] += 1
        return self.pool[idx].ggml_gemv_dispatch_bound(rw, input, output)

    def execute_quant_gemv(self, matrix: QuantMatrix, input, output=None) -> np.ndarray:
        """orchestrator.rs:222-234: the FFN / weight GEMV on the primary device."""
        return self._gpu_gemv(0, matrix, input, output)

    def execute_quant_gemv_batched(self, matrix: QuantMatrix, inputs, batch: int, outputs=None) -> np.ndarray:
        """orchestrator.rs:240-269: ``batch`` vectors through one pass over the weights (every
        type here, not only Q4_K; 8+ rows of the K-quants and Q8_0 use the tcgen05 tensor cores)."""
        rw = self.resident(matrix, 0)
        self.gemv_calls[0] += 1
        return self.engine.ggml_gemv_batched(rw, inputs, batch, outputs)

    def execute_lut_matmul(self, m, n, weights_q4, lut, input, output=None) -> np.ndarray:
        """orchestrator.rs:198-218 (on the GPU only: the reference's CPU retry is not mirrored)."""
        return self.engine.lut_matmul_q4(m, n, weights_q4, lut, input, output)

    def _target(self, op: LayerOpKind) -> int:
        placed = self._placement.get(op)
        if placed is None:
            return 0
        if placed.device is None:
            raise CudaError(_lib.HC_ERR_UNSUPPORTED,
                            f"{op.name} placed on the CPU: this backend has no CPU path")
        if not 0 <= placed.device < len(self.pool):
            raise CudaError(_lib.HC_ERR_INVALID, f"placed device {placed.device} not in pool")
        return placed.device

    def execute_op(self, op: LayerOpKind, binding: OpBinding, matrix: QuantMatrix, input, output=None):
        """orchestrator.rs:276-306: a GEMV honouring the planner's placement, else the op's
        binding.  Discard ops are no-ops (``output`` untouched, returned as given); every other
        binding computes on the GPU (see the module note on CPU-bound ops)."""
        if op in self._placement:
            return self._gpu_gemv(self._target(op), matrix, input, output)
        if binding.device is OpDevice.Discard:
            return output
        return self._gpu_gemv(0, matrix, input, output)

    def execute_op_bound(self, op: LayerOpKind, binding: OpBinding, matrix: QuantMatrix, input, output=None,
                         layer: int = 0, tensor_off: int = 0):
        """orchestrator.rs:308-342: like ``execute_op``, from the resident copy of the matrix on
        the placed device (the resident upload is this backend's device mirror; ``layer`` and
        ``tensor_off`` locate a tensor inside the reference's streaming scratch and have no
        role here)."""
        return self.execute_op(op, binding, matrix, input, output)

    def submit_op_bound(self, op: LayerOpKind, binding: OpBinding, matrix: QuantMatrix, input, output=None,
                        layer: int = 0, tensor_off: int = 0) -> OpPending:
        """orchestrator.rs:344-374: non-blocking for a computing op: the GEMV is enqueued on its
        device and the returned handle joins it.  Discard ops return a done handle."""
        if op not in self._placement and binding.device is OpDevice.Discard:
            return OpPending(None)
        idx = self._target(op)
        rw = self.resident(matrix, idx)
        self.gemv_calls[idx] += 1
        return OpPending(self.pool[idx].ggml_gemv_async(rw, input))

    def begin_gemv_on(self, role: int, matrix: QuantMatrix, input) -> PendingGemv:
        """orchestrator.rs:424-440 / begin_gemv_engine (:479-517): an async GEMV on the role's
        device."""
        idx = role % len(self.pool)
        rw = self.resident(matrix, idx)
        self.gemv_calls[idx] += 1
        return self.pool[idx].ggml_gemv_async(rw, input)


__all__ = ["LayerOpKind", "OpDevice", "OpKernel", "OpBinding", "op_binding", "ComputeTarget", "OpPending",
           "EngineOrchestrator", "gemv_kernel", "CPU_GEMV", "CPU_NORM", "GPU_ASYNC", "HOST_ROW", "DISCARD"]
