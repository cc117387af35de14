// gemv_mma.cu -- dense Q4_K / Q6_K / Q8_0 GEMV and fused SwiGLU gate/up on mma.m16n8k16,
// scheduled as warp-level stream-K with a per-warp cp.async pipeline.
//
// Reference semantics: gemv_q4_k (crates/hayai-model/src/q4k.rs:206-256), gemv_q6_k
// (crates/hayai-model/src/q6k.rs:59-90), gemv_q8_0 (crates/hayai-model/src/quant.rs:598-615)
// and the host SwiGLU combine (crates/hayai-core/src/stream_infer.rs:3836-3840).  Summation
// order differs from the reference's sequential sums (tensor-core tiles + tree reduction);
// results agree within the f32 tolerance of the parity contract and are deterministic.
//
// Schedule.  The work is the set of units (16-row tile, one kernel block of K); unit u is
// tile u / nbk, block u % nbk.  The T units are split into W = gridDim.x * 8 contiguous,
// equal ranges, one per warp, so every warp streams the same number of bytes (+-1 unit)
// whatever the matrix shape.  A tile whose units belong to one warp is finished in
// registers; a tile split between warps stores each warp's partial sums in slot order in a
// workspace and the last warp to arrive (atomic counter) adds the slots in order, applies
// the epilogue and re-arms the counter.  No CTA-wide barrier exists in the main loop.
//
// Memory pipeline.  Each warp owns an S-stage ring in shared memory.  For every unit a lane
// issues cp.async copies of exactly the 16-byte pieces it will dequantise (piece-major
// layout: conflict-free reads), so S-1 units are in flight while one is computed.
#include "gemv_launch.h"
#include "gemv_mma.cuh"
#include "gemv_mma_impl.cuh"

namespace hc {

// ------------------------------------------------------------------ pieces per format
// Byte offsets (within a row of the GPU layout) of the 16-byte pieces lane t copies for
// kernel block kb of one row.
template <class F>
struct Pieces;

template <>
struct Pieces<FmtQ4K> {
    static constexpr int kN = 3;  // header (d, dmin, scales), codes 32t..32t+15, 32t+16..32t+31
    __device__ static void offsets(int kb, int t, int /*nb*/, int (&o)[kN]) {
        o[0] = kb * 144;
        o[1] = kb * 144 + 16 + 32 * t;
        o[2] = kb * 144 + 32 + 32 * t;
    }
    __device__ static void fetch(const uint4 (&p)[kN], int /*kb*/, Q4KBlk& b) {
        b.h = p[0];
        b.q0 = p[1];
        b.q1 = p[2];
    }
};

template <>
struct Pieces<FmtQ6K> {
    static constexpr int kN = 5;  // ql (2), qh, scales, the 16-byte d-plane chunk holding d[kb]
    __device__ static void offsets(int kb, int t, int nb, int (&o)[kN]) {
        o[0] = kb * 208 + 32 * t;
        o[1] = kb * 208 + 32 * t + 16;
        o[2] = kb * 208 + 128 + 16 * t;
        o[3] = kb * 208 + 192;
        o[4] = nb * 208 + (kb >> 3) * 16;
    }
    __device__ static void fetch(const uint4 (&p)[kN], int kb, Q6KBlk& b) {
        b.l0 = p[0];
        b.l1 = p[1];
        b.qh = p[2];
        b.sc = p[3];
        const int i = (kb & 7) >> 1;
        const uint32_t w = i == 0 ? p[4].x : (i == 1 ? p[4].y : (i == 2 ? p[4].z : p[4].w));
        b.d = (uint16_t)(w >> (16 * (kb & 1)));
    }
};

template <>
struct Pieces<FmtQ80> {
    static constexpr int kN = 3;  // codes (2), the group's 4 f16 scales (8 bytes)
    __device__ static void offsets(int kg, int t, int ng, int (&o)[kN]) {
        o[0] = kg * 128 + 32 * t;
        o[1] = kg * 128 + 32 * t + 16;
        o[2] = ng * 128 + kg * 8;
    }
    __device__ static void fetch(const uint4 (&p)[kN], int /*kg*/, Q80Blk& b) {
        b.q0 = p[0];
        b.q1 = p[1];
        b.d = make_uint2(p[2].x, p[2].y);
    }
};

// bytes of one pipeline stage of one warp
template <class F>
__host__ __device__ constexpr int stage_bytes(int mats) {
    return mats * 2 * Pieces<F>::kN * 32 * 16;
}

// ------------------------------------------------------------------ kernel
constexpr int kWarps = 16;  // warps per CTA (one CTA per SM: the ring fills shared memory)
constexpr int kThreads = kWarps * 32;

// Units [0, T) are dealt to Weff = min(W, T) warps as equal contiguous ranges (every
// active warp owns at least one unit); unit u belongs to warp ((u + 1) * Weff - 1) / T.
__host__ __device__ __forceinline__ int sk_owner(int u, int Weff, int T) {
    return (int)(((long long)(u + 1) * Weff - 1) / T);
}
__host__ __device__ __forceinline__ int sk_begin(int w, int Weff, int T) { return (int)((long long)w * T / Weff); }

template <class F, int NV, bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) gemv_sk_kernel(GemvArgs a, int nvec) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int kMats = FUSED ? 2 : 1;
    constexpr int kP = Pieces<F>::kN;
    const GemvSmem L = gemv_smem_layout<F>(a.K, NV, FUSED);
    uint2* xt = reinterpret_cast<uint2*>(smem);
    float* sx = reinterpret_cast<float*>(smem + L.table_bytes);
    uint2* lut = reinterpret_cast<uint2*>(smem + L.table_bytes + L.sx_bytes);
    uint8_t* ring = smem + L.table_bytes + L.sx_bytes + L.lut_bytes + L.red_bytes;

    __shared__ float s_red[32];
    const NormArgs nrm{a.norm_w, a.norm_len, a.norm_eps};
    build_prologue<F, NV>(xt, sx, a.x, a.ldx, a.K, nvec, nrm, s_red, a.err);
    if constexpr (F::kType == T_Q4_K) build_q4k_lut(lut);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    const int ntiles = (a.M + 15) / 16;
    const int T = ntiles * nbk;
    const int W = gridDim.x * kWarps;
    const int Weff = W < T ? W : T;
    const int w = blockIdx.x * kWarps + warp;
    if (w >= Weff) return;  // no unit for this warp (only for matrices smaller than the machine)
    const int u0 = sk_begin(w, Weff, T), u1 = sk_begin(w + 1, Weff, T);
    const int S = a.stages;
    const int sbytes = stage_bytes<F>(kMats);
    const uint32_t ring_base = smem_addr(ring + (size_t)warp * S * sbytes) + lane * 16;
    const uint8_t* ring_gen = ring + (size_t)warp * S * sbytes + lane * 16;

    LaneCtx<NV> ctx;
    ctx.xt = xt + g * 4 + t;
    ctx.sx = sx;
    ctx.lut = lut;
    ctx.sxs = a.K / 32;
    ctx.nb = nbk;
    ctx.g = g;
    ctx.t = t;
    ctx.has_b = g < 2 * NV;

    // producer iterator: next unit to copy
    int p_tile = u0 / nbk, p_kb = u0 - p_tile * nbk, p_left = u1 - u0, p_slot = 0;
    const uint8_t* pr[2 * kMats];
    auto set_rows = [&](int tile) {
        const size_t rA = (size_t)min(tile * 16 + g, a.M - 1), rB = (size_t)min(tile * 16 + g + 8, a.M - 1);
#pragma unroll
        for (int mt = 0; mt < kMats; ++mt) {
            const uint8_t* wm = mt == 0 ? a.w : a.w2;
            pr[2 * mt] = wm + rA * a.row_stride;
            pr[2 * mt + 1] = wm + rB * a.row_stride;
        }
    };
    set_rows(p_tile);
    auto issue_next = [&]() {
        if (p_left > 0) {
            int off[kP];
            Pieces<F>::offsets(p_kb, t, nbk, off);
            const uint32_t sb = ring_base + p_slot * sbytes;
#pragma unroll
            for (int r = 0; r < 2 * kMats; ++r) {
#pragma unroll
                for (int p = 0; p < kP; ++p) {
                    const uint32_t d = sb + (r * kP + p) * 512;
                    if (F::kType == T_Q8_0 && p == kP - 1) cp_async8(d, pr[r] + off[p]);
                    else cp_async16(d, pr[r] + off[p]);
                }
            }
            --p_left;
            if (++p_kb == nbk) {
                p_kb = 0;
                set_rows(++p_tile);
            }
        }
        cp_async_commit();  // one group per call keeps the wait count uniform
        if (++p_slot == S) p_slot = 0;
    };

    for (int s = 0; s < S - 1; ++s) issue_next();

    using Blk = typename BlkOf<F>::T;
    float yA[kMats], yB[kMats];
    float pA[kMats][NV], pB[kMats][NV];  // Q4_K: per-lane shares (see q4k_unit_dist)
#pragma unroll
    for (int mt = 0; mt < kMats; ++mt) {
        yA[mt] = yB[mt] = 0.f;
#pragma unroll
        for (int v = 0; v < NV; ++v) pA[mt][v] = pB[mt][v] = 0.f;
    }
    int c_tile = u0 / nbk, c_kb = u0 - c_tile * nbk, c_slot = 0;

    for (int u = u0; u < u1; ++u) {
        issue_next();
        cp_async_wait(S - 1);
        const uint8_t* sp = ring_gen + c_slot * sbytes;
        if constexpr (F::kType == T_Q4_K) {
            Q4KBlk A[kMats], B[kMats];
#pragma unroll
            for (int mt = 0; mt < kMats; ++mt) {
                uint4 pa[kP], pb[kP];
#pragma unroll
                for (int p = 0; p < kP; ++p) {
                    pa[p] = *reinterpret_cast<const uint4*>(sp + ((mt * 2 + 0) * kP + p) * 512);
                    pb[p] = *reinterpret_cast<const uint4*>(sp + ((mt * 2 + 1) * kP + p) * 512);
                }
                Pieces<F>::fetch(pa, c_kb, A[mt]);
                Pieces<F>::fetch(pb, c_kb, B[mt]);
            }
            q4k_unit_dist<NV, kMats>(A, B, c_kb, ctx, pA, pB);
        } else {
#pragma unroll
            for (int mt = 0; mt < kMats; ++mt) {
                uint4 pa[kP], pb[kP];
#pragma unroll
                for (int p = 0; p < kP; ++p) {
                    pa[p] = *reinterpret_cast<const uint4*>(sp + ((mt * 2 + 0) * kP + p) * 512);
                    pb[p] = *reinterpret_cast<const uint4*>(sp + ((mt * 2 + 1) * kP + p) * 512);
                }
                Blk A, B;
                Pieces<F>::fetch(pa, c_kb, A);
                Pieces<F>::fetch(pb, c_kb, B);
                float dA, dB;
                blk_compute<F, NV>(A, B, c_kb, ctx, dA, dB);
                yA[mt] += dA;
                yB[mt] += dB;
            }
        }
        if (++c_slot == S) c_slot = 0;

        if (c_kb == nbk - 1 || u == u1 - 1) {  // flush the tile
            if constexpr (F::kType == T_Q4_K) {
                // lane shares -> lane t holds vector t's sums (the convention below)
#pragma unroll
                for (int mt = 0; mt < kMats; ++mt)
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        float sa = pA[mt][v], sb = pB[mt][v];
                        sa += __shfl_xor_sync(kFull, sa, 1);
                        sb += __shfl_xor_sync(kFull, sb, 1);
                        sa += __shfl_xor_sync(kFull, sa, 2);
                        sb += __shfl_xor_sync(kFull, sb, 2);
                        if (t == v) {
                            yA[mt] = sa;
                            yB[mt] = sb;
                        }
                        pA[mt][v] = pB[mt][v] = 0.f;
                    }
            }
            const int tile = c_tile, tu0 = tile * nbk, tu1 = tu0 + nbk;
            const int rowA = tile * 16 + g, rowB = rowA + 8;
            const bool whole = tu0 >= u0 && tu1 <= u1;
            float fA[kMats], fB[kMats];
            bool last = whole;
            if (whole) {
#pragma unroll
                for (int mt = 0; mt < kMats; ++mt) {
                    fA[mt] = yA[mt];
                    fB[mt] = yB[mt];
                }
            } else {
                const int wf = sk_owner(tu0, Weff, T), wl = sk_owner(tu1 - 1, Weff, T);
                const int ncon = wl - wf + 1, myslot = w - wf;
                float* ws = a.sk_ws + (size_t)tile * a.sk_slots * kMats * NV * 16;
                if (t < NV) {
#pragma unroll
                    for (int mt = 0; mt < kMats; ++mt) {
                        float* p = ws + ((size_t)(myslot * kMats + mt) * NV + t) * 16;
                        p[g] = yA[mt];
                        p[g + 8] = yB[mt];
                    }
                }
                __threadfence();
                __syncwarp();
                int old = 0;
                if (lane == 0) old = atomicAdd(a.sk_cnt + tile, 1);
                old = __shfl_sync(kFull, old, 0);
                last = old == ncon - 1;
                if (last) {
                    __threadfence();
#pragma unroll
                    for (int mt = 0; mt < kMats; ++mt) fA[mt] = fB[mt] = 0.f;
                    if (t < NV) {
                        for (int sl = 0; sl < ncon; ++sl) {
#pragma unroll
                            for (int mt = 0; mt < kMats; ++mt) {
                                const float* p = ws + ((size_t)(sl * kMats + mt) * NV + t) * 16;
                                fA[mt] += __ldcg(p + g);
                                fB[mt] += __ldcg(p + g + 8);
                            }
                        }
                    }
                    if (lane == 0) a.sk_cnt[tile] = 0;  // re-arm for the next launch
                }
            }
            if (last && t < NV && t < nvec) {
                float vA = fA[0], vB = fB[0];
                if constexpr (FUSED) {
                    vA = silu_mul(fA[0], fA[kMats - 1]);
                    vB = silu_mul(fB[0], fB[kMats - 1]);
                }
                if (rowA < a.M) {
                    if (a.resid) vA += a.resid[(size_t)t * a.ldr + rowA];
                    a.y[(size_t)t * a.ldy + rowA] = vA;
                }
                if (rowB < a.M) {
                    if (a.resid) vB += a.resid[(size_t)t * a.ldr + rowB];
                    a.y[(size_t)t * a.ldy + rowB] = vB;
                }
            }
#pragma unroll
            for (int mt = 0; mt < kMats; ++mt) yA[mt] = yB[mt] = 0.f;
        }
        if (++c_kb == nbk) {
            c_kb = 0;
            ++c_tile;
        }
    }
    cp_async_wait(0);
}

// ------------------------------------------------------------------ host launch
template <class F>
static int ring_stages(int K, int nv, bool fused, int smem_limit) {
    const int base = gemv_smem_layout<F>(K, nv, fused).total() + 256;  // + static shared
    const int per = kWarps * stage_bytes<F>(fused ? 2 : 1);
    int s = (smem_limit - base) / per;
    return s > 6 ? 6 : s;
}

static int sk_grid(int M, int nbk, int num_sms) {
    const long long T = (long long)((M + 15) / 16) * nbk;
    long long grid = (T + kWarps - 1) / kWarps;
    if (grid > num_sms) grid = num_sms;
    return grid < 1 ? 1 : (int)grid;
}

template <class F, int NV, bool FUSED>
static cudaError_t launch_one(GemvArgs a, int nvec, int num_sms, int smem_limit, cudaStream_t stream) {
    const GemvSmem L = gemv_smem_layout<F>(a.K, NV, FUSED);
    const int S = ring_stages<F>(a.K, NV, FUSED, smem_limit);
    if (S < 2) return cudaErrorInvalidConfiguration;
    a.stages = S;
    const int smem = L.total() + kWarps * S * stage_bytes<F>(FUSED ? 2 : 1);
    auto kern = gemv_sk_kernel<F, NV, FUSED>;
    static int configured_smem[64];  // per template instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && dev < 64 && configured_smem[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured_smem[dev] = smem;
    }
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    kern<<<sk_grid(a.M, nbk, num_sms), kThreads, smem, stream>>>(a, nvec);
    return cudaGetLastError();
}

// Contributors per tile of the stream-K split (host mirror of the kernel's partition).
static int sk_slots(int M, int nbk, int grid) {
    const int T = ((M + 15) / 16) * nbk, W = grid * kWarps, Weff = W < T ? W : T;
    int best = 1;
    for (int tile = 0; tile * nbk < T; ++tile) {
        const int c = sk_owner(tile * nbk + nbk - 1, Weff, T) - sk_owner(tile * nbk, Weff, T) + 1;
        best = c > best ? c : best;
    }
    return best;
}

template <class F>
static int max_nv(int K, bool fused, int smem_limit) {
    // Q4_K keeps 2*NV*NMAT accumulator fragments live: cap the fused variant at 2 vectors
    const int top = (F::kType == T_Q4_K && fused) ? 2 : 4;
    for (int nv = top; nv >= 1; nv >>= 1)
        if (ring_stages<F>(K, nv, fused, smem_limit) >= 2) return nv;
    return 0;
}

template <class F>
static cudaError_t launch_fmt(GemvArgs a, int nvec, bool fused, int num_sms, int smem_limit, cudaStream_t stream) {
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
            e = fused ? launch_one<F, 4, true>(b, cnt, num_sms, smem_limit, stream)
                      : launch_one<F, 4, false>(b, cnt, num_sms, smem_limit, stream);
        else if (nv == 2)
            e = fused ? launch_one<F, 2, true>(b, cnt, num_sms, smem_limit, stream)
                      : launch_one<F, 2, false>(b, cnt, num_sms, smem_limit, stream);
        else
            e = fused ? launch_one<F, 1, true>(b, cnt, num_sms, smem_limit, stream)
                      : launch_one<F, 1, false>(b, cnt, num_sms, smem_limit, stream);
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
    const int slots = sk_slots(M, nbk, sk_grid(M, nbk, num_sms));
    *ws_floats = (size_t)((M + 15) / 16) * slots * (fused ? 2 : 1) * 4 * 16;
    *counters = (size_t)((M + 15) / 16);
}

cudaError_t launch_gemv_mma(int type, const GemvArgs& a0, int nvec, bool fused, int num_sms, int smem_limit,
                            cudaStream_t stream) {
    GemvArgs a = a0;
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nbk = (a.K + be - 1) / be;
    a.sk_slots = sk_slots(a.M, nbk, sk_grid(a.M, nbk, num_sms));
    switch (type) {
        case T_Q4_K: return launch_fmt<FmtQ4K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q6_K: return launch_fmt<FmtQ6K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q8_0: return launch_fmt<FmtQ80>(a, nvec, fused, num_sms, smem_limit, stream);
        default: return cudaErrorInvalidValue;
    }
}

bool gemv_mma_supported(int type) { return type == T_Q4_K || type == T_Q6_K || type == T_Q8_0; }

}  // namespace hc
