// noalloc.cu -- hc_gemv_dev_noalloc: the stream-K tensor-core GEMV with its scratch memory
// taken from a fixed array compiled into this library instead of the engine's workspace.
//
// Who needs it.  hc_gemv_dev grows its stream-K workspace (partial sums of tiles split
// between warps, plus one arrival counter per 16-row tile) with cudaMalloc the first time a
// shape needs more than it holds.  Some callers cannot allow that: a host application whose
// device memory is entirely owned by its own pool allocator (a library cudaMalloc there can
// fail or fragment the pool), and latency-bound decode loops in which a cudaMalloc/cudaFree,
// which can synchronise the device, would stall the token.  This entry point performs no
// allocation of any kind.  The engine and the weight handles it is given are created
// beforehand, at set-up, as for every other entry point.
//
// The scratch is g_gemv_scratch below: kScratchWsFloats partial-sum floats followed by
// kScratchCounters tile counters (4 MiB + 64 KiB, held by every GPU that loads the library
// until the process exits).  Matrices whose split needs more are rejected with
// HC_ERR_INVALID before anything is enqueued.  Every call on a device shares the one array
// and leaves its contents behind, so calls whose kernels overlap on the GPU (two streams,
// two engines on one device) race on it: serialise them.
#include "engine.h"
#include "gemv_launch.h"
#include "gemv_mma.cuh"
#include "hayai_cuda.h"

namespace hc {

constexpr size_t kScratchWsFloats = size_t(1) << 20;  // 4 MiB of partial sums
constexpr size_t kScratchCounters = 16384;            // one counter per 16-row tile: M <= 262144

// One array: the partial sums, then the tile counters (stored as int).
static __device__ __align__(256) float g_gemv_scratch[kScratchWsFloats + kScratchCounters];

// Device address of the scratch array on `dev`, which must be the current device.  Host code
// only sees a host-side stand-in under the name g_gemv_scratch; the address a kernel may use
// comes from cudaGetSymbolAddress.  It is looked up on every call (a lookup allocates
// nothing): a cached address would go stale if the device's context were reset and the module
// loaded again.  The first lookup on a device loads this library's device code there.
static int scratch_address(int dev, float** out) {
    int cur = -1;
    cudaError_t ce = cudaGetDevice(&cur);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "cudaGetDevice");
    if (cur != dev) return hc_set_error(HC_ERR_INVALID, "device %d is not current (%d is)", dev, cur);
    void* p = nullptr;
    ce = cudaGetSymbolAddress(&p, g_gemv_scratch);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "cudaGetSymbolAddress(static GEMV scratch)");
    *out = static_cast<float*>(p);
    return HC_OK;
}

}  // namespace hc

using namespace hc;

extern "C" int hc_gemv_dev_noalloc(hc_engine* e, const hc_weights* w, const float* x, size_t ldx, float* y,
                                   size_t ldy, const float* resid, size_t ldr, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!w || !x || !y) return hc_set_error(HC_ERR_INVALID, "null argument");
    if (w->device != e->device)
        return hc_set_error(HC_ERR_INVALID, "weights live on device %d, engine on %d", w->device, e->device);
    if (!gemv_mma_supported(w->type))
        return hc_set_error(HC_ERR_UNSUPPORTED,
                            "hc_gemv_dev_noalloc covers Q4_K, Q6_K and Q8_0 (got %s); the other formats need no "
                            "scratch and run through hc_gemv_dev",
                            hc_type_label(w->type));
    if (ldx < w->n || ldy < w->m || (resid && ldr < w->m))
        return hc_set_error(HC_ERR_INVALID, "leading dimension smaller than the row length");
    if (((uintptr_t)x & 15) || (ldx & 3))
        return hc_set_error(HC_ERR_INVALID, "x must be 16-byte aligned with ldx a multiple of 4");
    size_t ws_floats = 0, counters = 0;
    gemv_sk_workspace(w->type, (int)w->m, (int)w->n, false, e->num_sms, &ws_floats, &counters);
    if (ws_floats > kScratchWsFloats || counters > kScratchCounters)
        return hc_set_error(HC_ERR_INVALID,
                            "%zu x %zu %s matrix needs %zu scratch floats and %zu tile counters; the static scratch "
                            "holds %zu and %zu",
                            w->m, w->n, hc_type_label(w->type), ws_floats, counters, kScratchWsFloats,
                            kScratchCounters);
    if (nvec == 0) return HC_OK;
    float* scratch = nullptr;
    rc = scratch_address(e->device, &scratch);
    if (rc) return rc;
    int* cnt = reinterpret_cast<int*>(scratch + kScratchWsFloats);
    // the counters must start at zero; a kernel re-arms the ones it used, but clear them
    // anyway so a call never depends on how the previous one ended
    cudaError_t ce = cudaMemsetAsync(cnt, 0, counters * sizeof(int), e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "clearing the static scratch counters");
    GemvArgs a{};
    a.w = (const uint8_t*)w->dev;
    a.row_stride = (long long)w->stride;
    a.M = (int)w->m;
    a.K = (int)w->n;
    a.x = x;
    a.ldx = (int)ldx;
    a.y = y;
    a.ldy = (int)ldy;
    a.resid = resid;
    a.ldr = (int)ldr;
    a.w2 = nullptr;
    a.err = e->d_err;
    a.sk_ws = scratch;
    a.sk_cnt = cnt;
    ce = launch_gemv_mma(w->type, a, (int)nvec, false, e->num_sms, e->smem_optin, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "gemv launch (static scratch)");
    return HC_OK;
}
