"""The host mirror of hayai-core's dispatch: ``QuantMatrix`` (crates/hayai-model/src/quant.rs:
31-117), the per-op bindings (crates/hayai-core/src/exec_plan.rs:131-216) and
``EngineOrchestrator`` (crates/hayai-core/src/orchestrator.rs:72-98, 198-422, 479-517).

CPU: the binding table, the type -> kernel map, QuantMatrix construction and validation.
GPU: every orchestrator entry point against the oracle, resident uploads reused, the
binding and placement rules of this backend (computing ops run on the GPU, Discard ops are
no-ops, a CPU placement or a type without a kernel is an error, never a host fallback), and
the analogue of the reference's own ``execute_op_honors_binding`` test."""
import numpy as np
import pytest

import oracle
from hayai_b200 import _lib
from hayai_b200.engine import CudaError, QuantMatrix
from hayai_b200.orchestrator import (CPU_GEMV, CPU_NORM, DISCARD, GPU_ASYNC, HOST_ROW, ComputeTarget,
                                     EngineOrchestrator, LayerOpKind, OpDevice, gemv_kernel, op_binding)
from tests.helpers import assert_parity, quantized

K = LayerOpKind


# ---------------------------------------------------------------- CPU
def test_binding_table_matches_reference_classes():
    # exec_plan.rs:192-216, one representative per class plus the FFN-path ops
    assert op_binding(K.TokenEmbed) == HOST_ROW
    assert op_binding(K.FfnNorm) == CPU_NORM
    assert op_binding(K.Router) == CPU_GEMV
    assert op_binding(K.AttnQ) == CPU_GEMV
    for k in (K.FfnGate, K.FfnUp, K.FfnDown, K.FfnGateUp, K.ExpertGate, K.ExpertUp, K.ExpertDown,
              K.SharedExpert, K.OutputProj):
        assert op_binding(k) == GPU_ASYNC, k
    for k in (K.LayerOutputScale, K.RouterBias, K.RouterScale, K.ExpertScale, K.Aux):
        assert op_binding(k) == DISCARD, k
    assert {op_binding(k).device for k in LayerOpKind} == set(OpDevice)
    assert str(ComputeTarget.cpu()) == "CPU" and str(ComputeTarget.dev(3)) == "dev3"


def test_kernel_map_covers_supported_types_only():
    for t, label in ((oracle.Q4_K, "q4_k"), (oracle.Q6_K, "q6_k"), (oracle.Q8_0, "q8_0"),
                     (oracle.IQ2_XXS, "iq2_xxs"), (oracle.IQ3_S, "iq3_s"), (oracle.F32, "f32")):
        assert gemv_kernel(t) == label
    for t in (19, 29, 34, 35):  # IQ1_S, IQ1_M, TQ1_0, TQ2_0: no GEMV anywhere
        assert gemv_kernel(t) is None


def test_quant_matrix_owned_view_and_validation():
    raw = quantized(oracle.Q4_K, 4, 256, 3)
    own = QuantMatrix.owned("w", 256, 4, oracle.Q4_K, raw)
    view = QuantMatrix.view("w", 256, 4, oracle.Q4_K, raw)
    assert not np.shares_memory(own.data, raw)
    assert np.shares_memory(view.data, raw)  # quant.rs:97-117: a view borrows the caller's bytes
    with pytest.raises(CudaError):
        QuantMatrix.view("w", 255, 4, oracle.Q4_K, raw)  # ncols not a multiple of the block
    with pytest.raises(CudaError):
        QuantMatrix.view("w", 256, 5, oracle.Q4_K, raw)  # too few bytes
    QuantMatrix.view("iq1", 256, 1, 19, np.zeros(50, np.uint8))  # no kernel: the GEMV fails, not this


# ---------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def orch():
    o = EngineOrchestrator((0,))
    yield o
    o.close()


def _mat(t, m, n, seed):
    raw = quantized(t, m, n, seed)
    return QuantMatrix.owned(f"m{seed}", n, m, t, raw), raw


@pytest.mark.gpu
@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0, oracle.IQ2_XXS, oracle.Q5_0])
def test_execute_quant_gemv_matches_oracle_and_uploads_once(orch, t):
    m, n = 384, 1024
    qm, raw = _mat(t, m, n, 50 + t)
    x = oracle.normal(60 + t, n)
    want = oracle.gemv(t, m, n, raw, x)
    before = len(orch._resident_cache)
    assert_parity(want, orch.execute_quant_gemv(qm, x), what="first call")
    assert_parity(want, orch.execute_quant_gemv(qm, x), what="second call")
    assert len(orch._resident_cache) == before + 1  # one resident copy, reused
    xs = oracle.normal(70 + t, 3 * n)
    got = orch.execute_quant_gemv_batched(qm, xs, 3).reshape(3, m)
    for b in range(3):
        assert_parity(oracle.gemv(t, m, n, raw, xs[b * n:(b + 1) * n]), got[b], what=f"batched row {b}")
    orch.evict(qm)
    assert len(orch._resident_cache) == before


@pytest.mark.gpu
def test_execute_op_honours_bindings_like_the_reference(orch):
    # the reference's execute_op_honors_binding (orchestrator.rs:548-612): a 4 x 6 F32 matrix
    w = np.array([0.5, -1.0, 0.25, 2.0, 1.0, 0.0, -0.5, 1.5, 2.0, -2.0, 0.75, -1.25, 0.1, 0.2,
                  0.3, 0.4, 1.0, 1.0, 1.0, 1.0, -1.0, -1.0, -1.0, -1.0], np.float32)
    qm = QuantMatrix.owned("w.weight", 4, 6, oracle.F32, w.view(np.uint8))
    x = np.array([i * 0.5 - 0.25 for i in range(4)], np.float32)
    want = w.reshape(6, 4).astype(np.float64) @ x.astype(np.float64)
    # GPU-bound FFN op
    np.testing.assert_allclose(orch.execute_op(K.FfnGate, op_binding(K.FfnGate), qm, x), want, atol=1e-5)
    # CPU-bound in the reference (router): computed on the GPU here, same result
    np.testing.assert_allclose(orch.execute_op(K.Router, op_binding(K.Router), qm, x), want, atol=1e-5)
    # Discard: a no-op, the output is untouched
    out = np.full(6, 9.9, np.float32)
    orch.execute_op(K.LayerOutputScale, op_binding(K.LayerOutputScale), qm, x, out)
    assert np.all(out == np.float32(9.9))
    # the bound variant runs from the resident copy
    np.testing.assert_allclose(orch.execute_op_bound(K.FfnDown, op_binding(K.FfnDown), qm, x, layer=3), want,
                               atol=1e-5)
    orch.evict(qm)


@pytest.mark.gpu
def test_placement_and_async_submission(orch):
    t, m, n = oracle.Q4_K, 256, 512
    qm, raw = _mat(t, m, n, 81)
    x = oracle.normal(82, n)
    want = oracle.gemv(t, m, n, raw, x)
    try:
        p = orch.submit_op_bound(K.ExpertUp, op_binding(K.ExpertUp), qm, x)
        assert not p.done
        assert_parity(want, p.wait(), what="submit_op_bound")
        assert p.wait() is None and p.done
        assert orch.submit_op_bound(K.Aux, op_binding(K.Aux), qm, x).wait() is None  # Discard: done inline
        pend = orch.begin_gemv_on(2, qm, x)  # the down role's device
        assert_parity(want, pend.wait(), what="begin_gemv_on")
        # the planner's placement wins over the static class, on any device of the pool...
        orch.set_placement({K.Router: ComputeTarget.dev(0)})
        assert orch.placed_target(K.Router) == ComputeTarget.dev(0)
        assert_parity(want, orch.execute_op(K.Router, DISCARD, qm, x), what="placed on dev0")
        # ...but a placement on the CPU or outside the pool is an error, never a host GEMV
        orch.set_placement({K.FfnDown: ComputeTarget.cpu(), K.FfnUp: ComputeTarget.dev(7)})
        with pytest.raises(CudaError) as e:
            orch.execute_op(K.FfnDown, GPU_ASYNC, qm, x)
        assert e.value.code == _lib.HC_ERR_UNSUPPORTED
        with pytest.raises(CudaError) as e:
            orch.submit_op_bound(K.FfnUp, GPU_ASYNC, qm, x)
        assert "not in pool" in str(e.value)
    finally:
        orch.set_placement({})
        orch.evict(qm)
    assert "gate  -> cuda:0" in orch.format_compute_plan()


@pytest.mark.gpu
def test_type_without_kernel_is_a_hard_error(orch):
    qm = QuantMatrix.view("blk.0.ffn_gate.weight", 256, 2, 19, np.zeros(100, np.uint8))  # IQ1_S
    with pytest.raises(CudaError) as e:
        orch.execute_quant_gemv(qm, np.zeros(256, np.float32))
    assert e.value.code == _lib.HC_ERR_UNSUPPORTED
    assert "CPU fallback disabled" in str(e.value)
