"""GPU tests of hc_gemv_dev_noalloc, the GEMV entry point that allocates nothing.

Callers whose device memory belongs to their own pool allocator, or whose decode loop cannot
absorb a cudaMalloc, use this entry point instead of hc_gemv_dev: its stream-K scratch is a
static array inside the library.  These tests call both entry points through the C ABI on
the same resident weights and inputs and require bit-identical results (the same kernel with
the same split runs behind both) and parity with the CPU oracle, twice in a row (the second
call runs on the scratch the first one left behind).

The file name sorts last so that a run stopping at the first failure has run every other
test before this one; the tests pass alone in a fresh process and after the others.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from hayai_b200 import _lib
from hayai_b200._lib import lib
from tests.helpers import assert_parity, quantized

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _call(name, engine, w, x, y, resid, nvec):
    f = getattr(lib(), name)
    ldr = resid.shape[-1] if resid is not None else 0
    return f(engine.handle, w.handle, _p(x), x.shape[-1], _p(y), y.shape[-1], _p(resid), ldr, nvec)


@pytest.mark.parametrize("t,m,n,nvec,with_resid", [
    (oracle.Q4_K, 4096, 4096, 1, False),    # tiles split over ~10 warps
    (oracle.Q6_K, 1024, 14336, 1, False),   # FFN-down shape: long rows
    (oracle.Q8_0, 2048, 4096, 3, True),     # several vectors + residual
    (oracle.Q4_K, 14336, 4096, 2, True),    # Llama-3-8B gate/up shape
    # 9 vectors: three launches of the kernel (4 + 4 + 1 vectors); 1000 rows (not a multiple
    # of 128) keep hc_gemv_dev off the tcgen05 batch path, so both calls run the same kernel
    (oracle.Q6_K, 1000, 2048, 9, True),
])
def test_noalloc_matches_gemv_dev_and_oracle_twice(engine, t, m, n, nvec, with_resid):
    raw = quantized(t, m, n, seed=101 + t)
    w = engine.upload(t, m, n, raw)
    xh = oracle.normal(7 + t, nvec * n).reshape(nvec, n)
    rh = oracle.normal(9 + t, nvec * m).reshape(nvec, m) if with_resid else None
    want = np.stack([oracle.gemv(t, m, n, raw, xh[v]) for v in range(nvec)])
    if rh is not None:
        want = want + rh
    x = torch.from_numpy(xh).cuda()
    resid = torch.from_numpy(rh).cuda() if rh is not None else None
    stream = torch.cuda.current_stream()
    engine.set_stream(stream)
    try:
        ref = torch.full((nvec, m), float("nan"), device="cuda")
        assert _call("hc_gemv_dev", engine, w, x, ref, resid, nvec) == _lib.HC_OK, lib().hc_last_error()
        torch.cuda.synchronize()
        assert_parity(want, ref.cpu().numpy(), what="hc_gemv_dev vs oracle")
        for call in range(2):
            y = torch.full((nvec, m), float("nan"), device="cuda")
            rc = _call("hc_gemv_dev_noalloc", engine, w, x, y, resid, nvec)
            assert rc == _lib.HC_OK, lib().hc_last_error()
            torch.cuda.synchronize()
            # the same kernel with the same split as hc_gemv_dev: bit-identical results
            assert torch.equal(ref, y), f"call {call + 1}: differs from hc_gemv_dev"
            assert_parity(want, y.cpu().numpy(), what=f"call {call + 1} vs oracle")
        engine.sync()  # device error flag clear
    finally:
        engine.set_stream(None)
        w.free()


def test_noalloc_rejects_oversized_and_unsupported(engine):
    # 16385 row tiles: one more than the static counters hold; rejected before any launch
    m, n = 16385 * 16, 32
    big = engine.upload(oracle.Q8_0, m, n, torch.zeros(m * 34, dtype=torch.uint8).numpy())
    x = torch.zeros(1, n, device="cuda")
    y = torch.zeros(1, m, device="cuda")
    try:
        rc = _call("hc_gemv_dev_noalloc", engine, big, x, y, None, 1)
        assert rc == _lib.HC_ERR_INVALID
        assert b"static scratch" in lib().hc_last_error()
    finally:
        big.free()

    # formats without a stream-K kernel are refused, not silently routed elsewhere
    f32 = engine.upload(oracle.F32, 16, 32, torch.zeros(16 * 32, dtype=torch.float32).numpy())
    try:
        rc = _call("hc_gemv_dev_noalloc", engine, f32, x, torch.zeros(1, 16, device="cuda"), None, 1)
        assert rc == _lib.HC_ERR_UNSUPPORTED
    finally:
        f32.free()

    # the engine still works after the rejections
    w = engine.synth_weights(oracle.Q6_K, 256, 512, seed=5)
    xs = torch.randn(1, 512, generator=torch.Generator().manual_seed(1)).cuda()
    ref = torch.empty(1, 256, device="cuda")
    got = torch.empty(1, 256, device="cuda")
    engine.set_stream(torch.cuda.current_stream())
    try:
        assert _call("hc_gemv_dev", engine, w, xs, ref, None, 1) == _lib.HC_OK
        assert _call("hc_gemv_dev_noalloc", engine, w, xs, got, None, 1) == _lib.HC_OK, lib().hc_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ref, got), "after the rejections: differs from hc_gemv_dev"
    finally:
        engine.set_stream(None)
        w.free()
