// gemv_tma.cu -- dense Q4_K / Q6_K / Q8_0 GEMV and fused SwiGLU gate/up: one warp-specialised
// TMA pipeline (gemv_tma.cuh) per launch.
//
// Reference semantics: gemv_q4_k (crates/hayai-model/src/q4k.rs:206-256), gemv_q6_k
// (crates/hayai-model/src/q6k.rs:59-90), gemv_q8_0 (crates/hayai-model/src/quant.rs:598-615)
// and the host SwiGLU combine (crates/hayai-core/src/stream_infer.rs:3836-3840).  Summation
// order differs from the reference's sequential sums (tensor-core tiles, then a fixed-order
// reduction over warps and CTAs); results agree within the f32 parity tolerance and are
// deterministic.
#include "gemv_launch.h"
#include "gemv_tma.cuh"
#include "gemv_iq.cuh"

namespace hc {

// Shared memory: [2 x kMaxStages mbarriers, 128 B][table][zero block][Sx][tile slots][IQ LUT][ring]
struct TmaSmem {
    int table, zero, sx, red, lut, ring;  // byte offsets
};

static_assert(2 * kMaxStages * 8 <= 128, "the ring's mbarriers fit the 128-byte head of shared memory");

template <class F>
__host__ __device__ inline TmaSmem tma_smem_layout(int K, int nv, int stages, bool fused) {
    const GemvSmem g = gemv_smem_layout<F>(K, nv, false);
    TmaSmem s;
    s.table = 128;
    s.zero = s.table + g.table_bytes;
    s.sx = s.zero + g.zero_bytes;
    s.red = s.sx + g.sx_bytes;
    s.lut = (s.red + (stages + 2) * tile_slot_bytes(nv) + 15) & ~15;
    s.ring = (s.lut + iq_lut_bytes(F::kType) + 127) & ~127;
    return s;
}

template <class F, int NV, bool FUSED>
__global__ void __launch_bounds__(kTThreads, 1) gemv_tma_kernel(GemvArgs a, int nvec) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_tcnt[kMaxTileSlots];  // arrivals per tile slot
    __shared__ float s_red[32];
    const int S = a.stages;
    const TmaSmem L = tma_smem_layout<F>(a.K, NV, S, FUSED);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring r;
    r.full0 = smem_addr(smem);
    r.empty0 = r.full0 + 8 * kMaxStages;
    r.base = smem + L.ring;
    r.base_s = smem_addr(r.base);
    r.S = S;
    r.slot_bytes = tma_stage_bytes<F>(FUSED);
    r.slot = r.round = 0;
    const GemvPhase p = make_phase<F>(a.w, a.w2, a.row_stride, a.M, a.K);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(r.full0 + 8 * s, 1);
            mbar_init(r.empty0 + 8 * s, kCW);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < kMaxTileSlots) s_tcnt[threadIdx.x] = 0;
    __syncthreads();

    if (warp == kCW) {  // producer
        const bool ok = produce_phase<F, FUSED>(r, p, lane);
        drain_ring(r, r.round * S + r.slot);
        if (!ok && lane == 0 && a.err) atomicOr(a.err, 2);
        return;
    }

    uint2* xt = reinterpret_cast<uint2*>(smem + L.table);
    uint2* zero = reinterpret_cast<uint2*>(smem + L.zero);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    float* red = reinterpret_cast<float*>(smem + L.red);
    for (int i = threadIdx.x; i < table_entries_per_block<F>(NV); i += kCW * 32) zero[i] = make_uint2(0u, 0u);
    if constexpr (is_iq_type(F::kType)) iq_fill_lut<F::kType>(smem + L.lut, threadIdx.x, kCW * 32);
    const NormArgs nrm{a.norm_w, a.norm_len, a.norm_eps};
    build_prologue<F, NV>(xt, sx, a.x, a.ldx, a.K, nvec, nrm, s_red, a.err, kCW * 32, kBarPro);
    named_bar_sync(kBarPro, kCW * 32);
    LaneCtx<NV> ctx = make_ctx<F, NV>(xt, zero, sx, a.K, lane);
    ctx.lut = smem + L.lut;
    const TileOut o{a.y, a.ldy, a.resid, a.ldr, nvec, a.sk_ws, a.sk_cnt, a.sk_slots};
    int tslot = 0;
    bool aborted = false;
    consume_phase<F, NV, FUSED>(r, p, ctx, o, red, s_tcnt, tslot, aborted, a.err);
}

// ------------------------------------------------------------------ host launch
template <class F>
static int tma_stages(int K, int nv, bool fused, int smem_limit) {
    const int fixed = tma_smem_layout<F>(K, nv, 0, fused).ring + 512;  // + static shared
    int s = (smem_limit - fixed) / (tma_stage_bytes<F>(fused) + tile_slot_bytes(nv));
    return s > kMaxStages ? kMaxStages : s;
}

static int tma_grid(int M, int nbk, int num_sms) {
    const long long T = (long long)((M + 15) / 16) * nbk;
    return (int)(T < num_sms ? (T < 1 ? 1 : T) : num_sms);
}

// Most CTAs any tile is split over (the stream-K slots a tile needs).
static int tma_slots(int M, int nbk, int grid) {
    const int T = ((M + 15) / 16) * nbk;
    int best = 1;
    for (int tile = 0; tile * nbk < T; ++tile) {
        const int c = cta_owner(tile * nbk + nbk - 1, grid, T) - cta_owner(tile * nbk, grid, T) + 1;
        best = c > best ? c : best;
    }
    return best;
}

template <class F, int NV, bool FUSED>
static cudaError_t tma_launch_one(GemvArgs a, int nvec, int num_sms, int smem_limit, cudaStream_t stream) {
    const int S = tma_stages<F>(a.K, NV, FUSED, smem_limit);
    if (S < 2) return cudaErrorInvalidConfiguration;
    a.stages = S;
    const int smem = tma_smem_layout<F>(a.K, NV, S, FUSED).ring + S * tma_stage_bytes<F>(FUSED);
    auto kern = gemv_tma_kernel<F, NV, FUSED>;
    static int configured_smem[64];  // per template instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && configured_smem[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured_smem[dev] = smem;
    }
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    kern<<<tma_grid(a.M, nbk, num_sms), kTThreads, smem, stream>>>(a, nvec);
    return cudaGetLastError();
}

template <class F>
static int tma_max_nv(int K, bool fused, int smem_limit) {
    for (int nv = 4; nv >= 1; nv >>= 1)
        if (tma_stages<F>(K, nv, fused, smem_limit) >= 2) return nv;
    return 0;
}

template <class F>
static cudaError_t tma_launch_fmt(GemvArgs a, int nvec, bool fused, int num_sms, int smem_limit,
                                  cudaStream_t stream) {
    const int cap = tma_max_nv<F>(a.K, fused, smem_limit);
    if (cap == 0) return cudaErrorInvalidConfiguration;
    for (int v0 = 0; v0 < nvec;) {
        const int left = nvec - v0;
        int nv = left >= 4 && cap >= 4 ? 4 : (left >= 2 && cap >= 2 ? 2 : 1);
        if (left == 3 && cap >= 4) nv = 4;
        const int cnt = left < nv ? left : nv;
        GemvArgs b = a;
        b.x = a.x + (size_t)v0 * a.ldx;
        b.y = a.y + (size_t)v0 * a.ldy;
        b.resid = a.resid ? a.resid + (size_t)v0 * a.ldr : nullptr;
        cudaError_t e;
        if (nv == 4)
            e = fused ? tma_launch_one<F, 4, true>(b, cnt, num_sms, smem_limit, stream)
                      : tma_launch_one<F, 4, false>(b, cnt, num_sms, smem_limit, stream);
        else if (nv == 2)
            e = fused ? tma_launch_one<F, 2, true>(b, cnt, num_sms, smem_limit, stream)
                      : tma_launch_one<F, 2, false>(b, cnt, num_sms, smem_limit, stream);
        else
            e = fused ? tma_launch_one<F, 1, true>(b, cnt, num_sms, smem_limit, stream)
                      : tma_launch_one<F, 1, false>(b, cnt, num_sms, smem_limit, stream);
        if (e != cudaSuccess) return e;
        v0 += cnt;
    }
    return cudaSuccess;
}

// Workspace the stream-K split needs for an M x K launch of `type`: partial-sum floats and
// per-tile counters (which must be zero before the first launch; kernels leave them zero).
void gemv_sk_workspace(int type, int M, int K, bool fused, int num_sms, size_t* ws_floats, size_t* counters) {
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nbk = (K + be - 1) / be;
    const int slots = tma_slots(M, nbk, tma_grid(M, nbk, num_sms));
    *ws_floats = (size_t)((M + 15) / 16) * slots * (fused ? 2 : 1) * 4 * 16;
    *counters = (size_t)((M + 15) / 16);
}

int gemv_sk_slots(int type, int M, int K, int num_sms) {
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nbk = (K + be - 1) / be;
    return tma_slots(M, nbk, tma_grid(M, nbk, num_sms));
}

cudaError_t launch_gemv_mma(int type, const GemvArgs& a0, int nvec, bool fused, int num_sms, int smem_limit,
                            cudaStream_t stream) {
    GemvArgs a = a0;
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nbk = (a.K + be - 1) / be;
    a.sk_slots = tma_slots(a.M, nbk, tma_grid(a.M, nbk, num_sms));
    switch (type) {
        case T_Q4_K: return tma_launch_fmt<FmtQ4K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q6_K: return tma_launch_fmt<FmtQ6K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q8_0: return tma_launch_fmt<FmtQ80>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_IQ2_XXS: return tma_launch_fmt<FmtIQ<T_IQ2_XXS>>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_IQ2_XS: return tma_launch_fmt<FmtIQ<T_IQ2_XS>>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_IQ2_S: return tma_launch_fmt<FmtIQ<T_IQ2_S>>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_IQ3_XXS: return tma_launch_fmt<FmtIQ<T_IQ3_XXS>>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_IQ3_S: return tma_launch_fmt<FmtIQ<T_IQ3_S>>(a, nvec, fused, num_sms, smem_limit, stream);
        default: return cudaErrorInvalidValue;
    }
}

bool gemv_mma_supported(int type) {
    return type == T_Q4_K || type == T_Q6_K || type == T_Q8_0 || is_iq_type(type);
}

}  // namespace hc
