// gemv_mma.cu -- Q4_K / Q6_K / Q8_0 GEMV and fused SwiGLU gate/up on mma.m16n8k16.
//
// Reference semantics: gemv_q4_k (crates/hayai-model/src/q4k.rs:206-256), gemv_q6_k
// (crates/hayai-model/src/q6k.rs:59-90), gemv_q8_0 (crates/hayai-model/src/quant.rs:598-615)
// and the host SwiGLU combine (crates/hayai-core/src/stream_infer.rs:3836-3840).
// Summation order differs from the reference's sequential sums (tensor-core tiles +
// tree reduction); results agree within the f32 tolerance of the parity contract.
#include "gemv_mma.cuh"
#include "gemv_launch.h"
#include "gemv_mma_impl.cuh"

namespace hc {

// ------------------------------------------------------------------ kernel
template <class F, int NV, bool FUSED>
__global__ void __launch_bounds__(256) gemv_mma_kernel(GemvArgs a, int nvec) {
    extern __shared__ __align__(16) uint8_t smem[];
    const GemvSmem L = gemv_smem_layout<F>(a.K, NV, FUSED);
    uint2* xt = reinterpret_cast<uint2*>(smem);
    float* sx = reinterpret_cast<float*>(smem + L.table_bytes);
    uint2* lut = reinterpret_cast<uint2*>(smem + L.table_bytes + L.sx_bytes);
    float* red = reinterpret_cast<float*>(smem + L.table_bytes + L.sx_bytes + L.lut_bytes);

    __shared__ float s_red[32];
    const NormArgs nrm{a.norm_w, a.norm_len, a.norm_eps};
    build_prologue<F, NV>(xt, sx, a.x, a.ldx, a.K, nvec, nrm, s_red, a.err);
    if constexpr (F::kType == T_Q4_K) build_q4k_lut(lut);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int WK = a.wk, groups = 8 / WK, grp = warp / WK, wk = warp % WK;
    const int nb = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    const int nbw = (nb + WK - 1) / WK;
    const int kb0 = min(nb, wk * nbw), kb1 = min(nb, kb0 + nbw);
    const int ntiles = (a.M + 15) / 16;
    constexpr int kMats = FUSED ? 2 : 1;
    LaneCtx<NV> ctx;
    ctx.xt = xt + g * 4 + t;
    ctx.sx = sx;
    ctx.lut = lut;
    ctx.sxs = a.K / 32;
    ctx.nb = nb;
    ctx.g = g;
    ctx.t = t;
    ctx.has_b = g < 2 * NV;

    for (int tb = blockIdx.x * groups; tb < ntiles; tb += gridDim.x * groups) {
        const int tile = tb + grp;
        float yA[kMats], yB[kMats];
#pragma unroll
        for (int mt = 0; mt < kMats; ++mt) yA[mt] = yB[mt] = 0.f;
        if (tile < ntiles) {
            const size_t rA = (size_t)min(tile * 16 + g, a.M - 1), rB = (size_t)min(tile * 16 + g + 8, a.M - 1);
            if constexpr (FUSED) {
                const uint8_t* const pa[2] = {a.w + rA * a.row_stride, a.w2 + rA * a.row_stride};
                const uint8_t* const pb[2] = {a.w + rB * a.row_stride, a.w2 + rB * a.row_stride};
                stream_tile<F, NV, 2>(pa, pb, kb0, kb1, ctx, yA, yB);
            } else {
                const uint8_t* const pa[1] = {a.w + rA * a.row_stride};
                const uint8_t* const pb[1] = {a.w + rB * a.row_stride};
                stream_tile<F, NV, 1>(pa, pb, kb0, kb1, ctx, yA, yB);
            }
        }
        if (t < NV) {
#pragma unroll
            for (int mt = 0; mt < kMats; ++mt) {
                float* r = red + ((mt * 8 + warp) * NV + t) * 16;
                r[g] = yA[mt];
                r[g + 8] = yB[mt];
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < groups * NV * 16; i += blockDim.x) {
            const int r = i & 15, v = (i >> 4) % NV, gi = i / (16 * NV);
            const int tl = tb + gi, row = tl * 16 + r;
            if (tl < ntiles && row < a.M && v < nvec) {
                float s = 0.f;
                for (int w = 0; w < WK; ++w) s += red[((gi * WK + w) * NV + v) * 16 + r];
                if constexpr (FUSED) {
                    float s2 = 0.f;
                    for (int w = 0; w < WK; ++w) s2 += red[((8 + gi * WK + w) * NV + v) * 16 + r];
                    s = silu_mul(s, s2);
                }
                if (a.resid) s += a.resid[(size_t)v * a.ldr + row];
                a.y[(size_t)v * a.ldy + row] = s;
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ host launch
template <class F, int NV, bool FUSED>
static cudaError_t launch_one(const GemvArgs& a, int nvec, int num_sms, cudaStream_t stream) {
    const GemvSmem L = gemv_smem_layout<F>(a.K, NV, FUSED);
    const int smem = L.total();
    auto kern = gemv_mma_kernel<F, NV, FUSED>;
    static int configured_smem[64];  // per template instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && dev < 64 && configured_smem[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured_smem[dev] = smem;
    }
    int occ = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorInvalidConfiguration;
    const int groups = 8 / a.wk;
    const int ntiles = (a.M + 15) / 16;
    const int need = (ntiles + groups - 1) / groups;
    const int grid = need < num_sms * occ ? need : num_sms * occ;
    kern<<<grid, 256, smem, stream>>>(a, nvec);
    return cudaGetLastError();
}

template <class F>
static int pick_wk(int K) {
    const int nb = (K + F::kBlockElems - 1) / F::kBlockElems;
    int wk = 8;
    while (wk > 1 && nb < wk) wk >>= 1;
    return wk;
}

template <class F>
static int max_nv(int K, bool fused, int smem_limit) {
    for (int nv = 4; nv >= 1; nv >>= 1)
        if (gemv_smem_layout<F>(K, nv, fused).total() <= smem_limit) return nv;
    return 0;
}

template <class F>
static cudaError_t launch_fmt(GemvArgs a, int nvec, bool fused, int num_sms, int smem_limit, cudaStream_t stream) {
    a.wk = pick_wk<F>(a.K);
    const int cap = max_nv<F>(a.K, fused, smem_limit);
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
            e = fused ? launch_one<F, 4, true>(b, cnt, num_sms, stream) : launch_one<F, 4, false>(b, cnt, num_sms, stream);
        else if (nv == 2)
            e = fused ? launch_one<F, 2, true>(b, cnt, num_sms, stream) : launch_one<F, 2, false>(b, cnt, num_sms, stream);
        else
            e = fused ? launch_one<F, 1, true>(b, cnt, num_sms, stream) : launch_one<F, 1, false>(b, cnt, num_sms, stream);
        if (e != cudaSuccess) return e;
        v0 += cnt;
    }
    return cudaSuccess;
}

cudaError_t launch_gemv_mma(int type, const GemvArgs& a, int nvec, bool fused, int num_sms, int smem_limit,
                            cudaStream_t stream) {
    switch (type) {
        case T_Q4_K: return launch_fmt<FmtQ4K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q6_K: return launch_fmt<FmtQ6K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q8_0: return launch_fmt<FmtQ80>(a, nvec, fused, num_sms, smem_limit, stream);
        default: return cudaErrorInvalidValue;
    }
}

bool gemv_mma_supported(int type) { return type == T_Q4_K || type == T_Q6_K || type == T_Q8_0; }

}  // namespace hc
