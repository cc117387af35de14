// moe.cu -- expert-routed SwiGLU FFN: exact router, exact top-k, routed tensor-core GEMV.
//
// Reference: forward_moe (crates/hayai-core/src/moe_infer.rs:221-264 router + routing,
// :342-376 per-expert SwiGLU, :449-455 weighted combine), route_experts (:868-935),
// top_k_indices (:852-862), gemv_f32 (crates/hayai-model/src/quant.rs:358-369).
//
// Bit-exactness of the selected experts rests on two facts: the router scores are
// produced by the same sequential f32 chain as gemv_f32 (one thread per (token,
// expert), sum += w*x with separate multiply and add), and the selection is the
// reference's stable descending sort (ties -> lower expert id first).
#include <string.h>

#include <algorithm>

#include <vector>

#include "../../include/hayai_cuda.h"
#include "engine.h"
#include "gemv_launch.h"
#include "gemv_mma_impl.cuh"
#include "gemv_tma.cuh"

using namespace hc;

namespace hc {

// ------------------------------------------------------------------ router
__global__ void __launch_bounds__(128) router_exact_kernel(const float* __restrict__ W, const float* __restrict__ x,
                                                           int E, int D, int T, float* __restrict__ scores) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= E * T) return;
    const int e = i % E, t = i / E;
    const float* w = W + (size_t)e * D;
    const float* xt = x + (size_t)t * D;
    float s = 0.0f;
    int c = 0;
    if (((((uintptr_t)w) | ((uintptr_t)xt)) & 15) == 0) {
        for (; c + 4 <= D; c += 4) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(w + c));
            const float4 b = __ldg(reinterpret_cast<const float4*>(xt + c));
            s = __fadd_rn(s, __fmul_rn(a.x, b.x));
            s = __fadd_rn(s, __fmul_rn(a.y, b.y));
            s = __fadd_rn(s, __fmul_rn(a.z, b.z));
            s = __fadd_rn(s, __fmul_rn(a.w, b.w));
        }
    }
    for (; c < D; ++c) s = __fadd_rn(s, __fmul_rn(__ldg(w + c), __ldg(xt + c)));
    scores[(size_t)t * E + e] = s;
}

// The same scores with the inputs staged in shared memory: a block takes 8 experts x 16
// tokens (thread = token * 8 + expert), copies their rows in coalesced, then every thread runs
// its chain from shared memory (rows padded by 4 floats so the 8 experts' float4 reads fall on
// distinct banks).  Summation order and rounding are those of router_exact_kernel.
constexpr int kRouterE = 8, kRouterT = 16;

__global__ void __launch_bounds__(kRouterE * kRouterT) router_staged_kernel(const float* __restrict__ W,
                                                                            const float* __restrict__ x, int E, int D,
                                                                            int T, float* __restrict__ scores,
                                                                            int* err) {
    extern __shared__ __align__(128) float rs[];
    __shared__ __align__(8) uint64_t s_bar;
    __shared__ int s_ok;
    const int ld = D + 4;
    float* ws = rs;                  // [kRouterE][ld]
    float* xs = rs + kRouterE * ld;  // [kRouterT][ld]
    const int e0 = blockIdx.x * kRouterE, t0 = blockIdx.y * kRouterT;
    const int ne = min(kRouterE, E - e0), nt = min(kRouterT, T - t0), d4 = D >> 2;
    const uint32_t bar = smem_addr(&s_bar);
    if (threadIdx.x == 0) {  // every row with one bulk copy (rows are 16-byte multiples, 16-byte aligned)
        mbar_init(bar, 1);
        mbar_fence_init();
        mbar_arrive_expect_tx(bar, (uint32_t)((ne + nt) * D * 4));
        for (int r = 0; r < ne; ++r) bulk_g2s(smem_addr(ws + r * ld), W + (size_t)(e0 + r) * D, (uint32_t)(D * 4), bar);
        for (int r = 0; r < nt; ++r) bulk_g2s(smem_addr(xs + r * ld), x + (size_t)(t0 + r) * D, (uint32_t)(D * 4), bar);
        s_ok = mbar_wait(bar, 0) ? 1 : 0;
        if (!s_ok) atomicOr(err, 2);
    }
    __syncthreads();
    if (!s_ok) return;
    const int e = threadIdx.x % kRouterE, t = threadIdx.x / kRouterE;
    if (e >= ne || t >= nt) return;
    const float4* w4 = reinterpret_cast<const float4*>(ws + e * ld);
    const float4* x4 = reinterpret_cast<const float4*>(xs + t * ld);
    float s = 0.0f;
#pragma unroll 4
    for (int c = 0; c < d4; ++c) {
        const float4 a = w4[c], b = x4[c];
        s = __fadd_rn(s, __fmul_rn(a.x, b.x));
        s = __fadd_rn(s, __fmul_rn(a.y, b.y));
        s = __fadd_rn(s, __fmul_rn(a.z, b.z));
        s = __fadd_rn(s, __fmul_rn(a.w, b.w));
    }
    scores[(size_t)(t0 + t) * E + e0 + e] = s;
}

// Router scores on the stream: the staged kernel when the rows fit shared memory.
static cudaError_t launch_router(const float* W, const float* x, int E, int D, int T, float* scores, int smem_limit,
                                 cudaStream_t stream, int* err) {
    const int smem = (kRouterE + kRouterT) * (D + 4) * 4 + 128;
    const bool aligned = ((((uintptr_t)W) | ((uintptr_t)x)) & 15) == 0 && (D & 3) == 0;
    if (aligned && smem <= smem_limit) {
        static int configured[64];
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 64 || configured[dev] < smem) {
            cudaError_t e = cudaFuncSetAttribute(router_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            if (dev < 64) configured[dev] = smem;
        }
        const dim3 grid((E + kRouterE - 1) / kRouterE, (T + kRouterT - 1) / kRouterT);
        router_staged_kernel<<<grid, kRouterE * kRouterT, smem, stream>>>(W, x, E, D, T, scores, err);
    } else {
        router_exact_kernel<<<(unsigned)(((size_t)E * T + 127) / 128), 128, 0, stream>>>(W, x, E, D, T, scores);
    }
    return cudaGetLastError();
}

// ------------------------------------------------------------------ routing
// "a ranks before b" in the reference's stable descending sort of indices.
__device__ __forceinline__ bool ranks_before(float va, int ia, float vb, int ib) {
    return va > vb || (!(va < vb) && ia < ib);
}

struct RouteMeta {
    int E, k, n_group, topk_group, gating, norm_topk_prob;
    float scale;
};

// softmax / sigmoid weights, renorm and scaling for the chosen ids (moe_infer.rs:906-932).
__device__ void route_weights(const float* sc, int E, const int32_t* ids, int k, const RouteMeta& m, float* w) {
    if (m.gating == 1) {
        for (int i = 0; i < k; ++i) w[i] = 1.0f / (1.0f + expf(-sc[ids[i]]));
    } else {
        float mx = -INFINITY;
        for (int i = 0; i < E; ++i) mx = fmaxf(mx, sc[i]);
        float sum = 0.0f;
        for (int i = 0; i < E; ++i) sum += expf(sc[i] - mx);
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (int i = 0; i < k; ++i) w[i] = expf(sc[ids[i]] - mx) * inv;
    }
    if (m.norm_topk_prob) {
        float s = 0.0f;
        for (int i = 0; i < k; ++i) s += w[i];
        if (s > 0.0f)
            for (int i = 0; i < k; ++i) w[i] /= s;
    }
    if (fabsf(m.scale - 1.0f) > 1e-9f)
        for (int i = 0; i < k; ++i) w[i] *= m.scale;
}

// One warp per token, no expert groups: k rounds of a warp arg-max over the
// not-yet-chosen experts, ties broken towards the lower id.
__global__ void route_topk_warp_kernel(const float* __restrict__ scores, const float* __restrict__ bias, int T,
                                       RouteMeta m, int32_t* __restrict__ ids, float* __restrict__ wout) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float* sc = scores + (size_t)t * m.E;
    int32_t* id = ids + (size_t)t * m.k;
    unsigned long long taken = 0ull;  // bit `slot` = expert lane + 32*slot already chosen (E <= 2048)
    for (int r = 0; r < m.k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int j = lane, slot = 0; j < m.E; j += 32, ++slot) {
            if ((taken >> slot) & 1ull) continue;
            const float v = bias ? sc[j] + bias[j] : sc[j];
            if (bi == 0x7fffffff || ranks_before(v, j, bv, bi)) {
                bv = v;
                bi = j;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ranks_before(ov, oi, bv, bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) id[r] = bi;
        if (bi != 0x7fffffff && (bi & 31) == lane) {
            taken |= 1ull << (bi >> 5);
        }
    }
    __syncwarp();
    if (lane == 0) route_weights(sc, m.E, id, m.k, m, wout + (size_t)t * m.k);
}

// General routing (expert groups): one thread per token, route_experts restated step by
// step with stable insertion sorts.  scratch: [T][4E] words.
__global__ void route_general_kernel(const float* __restrict__ scores, const float* __restrict__ bias, int T,
                                     RouteMeta m, int32_t* __restrict__ ids, float* __restrict__ wout,
                                     float* __restrict__ scratch) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const int E = m.E;
    const float* sc = scores + (size_t)t * E;
    float* choice = scratch + (size_t)t * 4 * E;
    float* gsc = choice + E;                                     // n_group group scores
    int32_t* gidx = reinterpret_cast<int32_t*>(choice + 2 * E);  // n_group sorted group ids
    int32_t* cbuf = reinterpret_cast<int32_t*>(choice + 3 * E);  // candidates
    for (int i = 0; i < E; ++i) choice[i] = bias ? sc[i] + bias[i] : sc[i];
    const int gs = E / m.n_group;
    for (int g = 0; g < m.n_group; ++g) {  // group score = sum of its 2 largest choices
        float a = -INFINITY, b = -INFINITY;
        for (int j = 0; j < gs; ++j) {
            const float v = choice[g * gs + j];
            if (v > a || j == 0) {
                b = j == 0 ? b : a;
                a = v;
            } else if (v > b || j == 1) {
                b = v;
            }
        }
        gsc[g] = gs >= 2 ? a + b : a;
        gidx[g] = g;
    }
    for (int i = 1; i < m.n_group; ++i) {
        const int v = gidx[i];
        int j = i;
        while (j > 0 && gsc[gidx[j - 1]] < gsc[v]) {
            gidx[j] = gidx[j - 1];
            --j;
        }
        gidx[j] = v;
    }
    const int keep = m.topk_group < m.n_group ? m.topk_group : m.n_group;
    int nc = 0;
    for (int q = 0; q < keep; ++q)
        for (int j = 0; j < gs; ++j) cbuf[nc++] = gidx[q] * gs + j;
    for (int i = 1; i < nc; ++i) {
        const int v = cbuf[i];
        int j = i;
        while (j > 0 && choice[cbuf[j - 1]] < choice[v]) {
            cbuf[j] = cbuf[j - 1];
            --j;
        }
        cbuf[j] = v;
    }
    int k = m.k < 1 ? 1 : m.k;
    if (k > nc) k = nc;
    int32_t* id = ids + (size_t)t * m.k;
    for (int i = 0; i < m.k; ++i) id[i] = i < k ? cbuf[i] : -1;
    route_weights(sc, E, id, k, m, wout + (size_t)t * m.k);
}

// ------------------------------------------------------------------ routed GEMV
struct MoeStage {
    const int32_t* ids;        // [P] expert of pair p
    const uint8_t* const* w;   // [E] expert matrix (gate or down), GPU layout
    const uint8_t* const* w2;  // [E] up matrix (fused stage)
    long long row_stride;  // bytes per 16-row tile of the tile-major layout
    int M, K;
    const float* x;  // rows: token (x_div = top_k) or pair (x_div = 1)
    int x_div, ldx;
    float* y;  // [P][ldy]
    int ldy;
    int items_per_pair, rows_per_item, wk;
    int* err;
    int e_lo, e_hi;  // experts held here: w[e - e_lo] (pairs routed elsewhere are skipped)
};

template <class F, bool FUSED>
__global__ void __launch_bounds__(256) moe_gemv_kernel(MoeStage s) {
    extern __shared__ __align__(16) uint8_t smem[];
    const GemvSmem L = gemv_smem_layout<F>(s.K, 1, FUSED);
    uint2* xt = reinterpret_cast<uint2*>(smem);
    uint2* zero = reinterpret_cast<uint2*>(smem + L.table_bytes);
    float* sx = reinterpret_cast<float*>(smem + L.table_bytes + L.zero_bytes);
    float* red = reinterpret_cast<float*>(smem + L.table_bytes + L.zero_bytes + L.sx_bytes);

    const int p = blockIdx.x / s.items_per_pair, j = blockIdx.x % s.items_per_pair;
    const int e = s.ids[p];
    if (e < s.e_lo || e >= s.e_hi) return;  // no expert, or one held by another rank (uniform per CTA)
    const float* x = s.x + (size_t)(p / s.x_div) * s.ldx;
    __shared__ float s_red[32];
    const NormArgs nrm{nullptr, 0, 0.f};
    for (int i = threadIdx.x; i < table_entries_per_block<F>(1); i += blockDim.x) zero[i] = make_uint2(0u, 0u);
    build_prologue<F, 1>(xt, sx, x, s.ldx, s.K, 1, nrm, s_red, s.err);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int WK = s.wk, groups = 8 / WK, grp = warp / WK, wk = warp % WK;
    const int nb = (s.K + F::kBlockElems - 1) / F::kBlockElems;
    const int nbw = (nb + WK - 1) / WK;
    const int kb0 = min(nb, wk * nbw), kb1 = min(nb, kb0 + nbw);
    const int r0 = j * s.rows_per_item, r1 = min(s.M, r0 + s.rows_per_item);
    const int ntiles = (r1 - r0 + 15) / 16;
    const uint8_t* W = s.w[e - s.e_lo];
    const uint8_t* W2 = FUSED ? s.w2[e - s.e_lo] : nullptr;
    float* y = s.y + (size_t)p * s.ldy;
    constexpr int kMats = FUSED ? 2 : 1;
    const LaneCtx<1> ctx = make_ctx<F, 1>(xt, zero, sx, s.K, lane);
    for (int tb = 0; tb < ntiles; tb += groups) {
        const int tile = tb + grp;
        float yA[kMats], yB[kMats];
#pragma unroll
        for (int mt = 0; mt < kMats; ++mt) yA[mt] = yB[mt] = 0.f;
        if (tile < ntiles) {
            const size_t toff = (size_t)(r0 / 16 + tile) * s.row_stride;  // r0 is a multiple of 16
            if constexpr (FUSED) {
                const uint8_t* const tb[2] = {W + toff, W2 + toff};
                stream_tile<F, 1, 2>(tb, kb0, kb1, ctx, yA, yB);
            } else {
                const uint8_t* const tb[1] = {W + toff};
                stream_tile<F, 1, 1>(tb, kb0, kb1, ctx, yA, yB);
            }
        }
        if (t == 0) {
#pragma unroll
            for (int mt = 0; mt < kMats; ++mt) {
                float* r = red + (mt * 8 + warp) * 16;
                r[g] = yA[mt];
                r[g + 8] = yB[mt];
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < groups * 16; i += blockDim.x) {
            const int r = i & 15, gi = i >> 4;
            const int row = r0 + (tb + gi) * 16 + r;
            if (tb + gi < ntiles && row < r1) {
                float v = 0.f;
                for (int w = 0; w < WK; ++w) v += red[(gi * WK + w) * 16 + r];
                if constexpr (FUSED) {
                    float v2 = 0.f;
                    for (int w = 0; w < WK; ++w) v2 += red[(8 + gi * WK + w) * 16 + r];
                    v = silu_mul(v, v2);
                }
                y[row] = v;
            }
        }
        __syncthreads();
    }
}

// Expert parallelism: this rank's pairs are all in every region; count the phase in this
// rank's epoch and tell every rank (release, system scope, after a system fence).  The epoch
// lives on the device so that a captured graph replays with the right targets.
__global__ void ep_signal_kernel(char* const* regions, int n, unsigned* epoch) {
    __threadfence_system();
    if (threadIdx.x == 0) *epoch += 1u;
    if ((int)threadIdx.x < n)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(regions[threadIdx.x] + kPeerEpBar) : "memory");
}

// The combine of expert parallelism: wait (bounded, one second; error bit 1) until every rank
// has signalled this phase (epoch e: the counter reaches e * world), then the top-k-ordered
// weighted sum of the rows exchanged in buffer (e - 1) & 1, plus the optional residual.
__global__ void moe_combine_wait_kernel(const char* region, size_t buf_bytes, const float* __restrict__ w, int T,
                                        int k, int dm, const float* resid, float* y, int world, int* err) {
    __shared__ int s_ok;
    const unsigned epoch = __ldcg(reinterpret_cast<const unsigned*>(region + kPeerEpEpoch));
    const unsigned target = epoch * (unsigned)world;
    const unsigned* bar = reinterpret_cast<const unsigned*>(region + kPeerEpBar);
    const float* D = reinterpret_cast<const float*>(region + kPeerEpData + ((epoch - 1u) & 1u) * buf_bytes);
    if (threadIdx.x == 0) {
        unsigned long long t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        int ok = 1;
        while (true) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if ((int)(v - target) >= 0) break;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > 1000000000ull) {
                ok = 0;
                if (err) atomicOr(err, 2);
                break;
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const size_t n = (size_t)T * dm;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / dm), j = (int)(i % dm);
        float acc = 0.0f;
        for (int q = 0; q < k; ++q)
            acc = __fadd_rn(acc, __fmul_rn(w[t * k + q], __ldcg(D + ((size_t)t * k + q) * dm + j)));
        y[i] = resid ? __fadd_rn(resid[i], acc) : acc;  // resid may alias y: read, then written, here
    }
}

// y[t][j] = [resid +] sum_i w[t,i] * D[t*k+i][j], in top-k order (moe_infer.rs:449-455; the
// residual add is the caller's, stream_infer.rs:2166-2170)
__global__ void moe_combine_kernel(const float* __restrict__ D, const float* __restrict__ w, int T, int k, int dm,
                                   const float* resid, float* y) {
    const size_t n = (size_t)T * dm;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / dm), j = (int)(i % dm);
        float acc = 0.0f;
        for (int q = 0; q < k; ++q) acc = __fadd_rn(acc, __fmul_rn(w[t * k + q], D[((size_t)t * k + q) * dm + j]));
        y[i] = resid ? __fadd_rn(resid[i], acc) : acc;  // resid may alias y: read, then written, here
    }
}

// ------------------------------------------------------------------ expert-grouped TMA GEMV
// The routed pairs (token, slot) are grouped by expert into segments of up to kMoeNV pairs
// (moe_group_kernel, pairs in index order); a segment is one GEMV of its expert's matrix over
// kMoeNV vectors, so an expert's weights are streamed once per segment, not once per pair.
// The segments' 16-row tiles are concatenated and cut statically over the CTAs in whole tiles
// (no cross-CTA reduction).  Each CTA runs the warp-specialised TMA pipeline of the dense GEMV
// (gemv_tma.cuh): a stage holds as many whole tiles of one segment as fit its 16 units (8 per
// matrix when fused), one bulk copy per matrix (the tiles of an expert are contiguous in the
// tile-major layout); every consumer warp takes one unit, drops its partial into the stage's
// shared-memory slot, and the last warp to arrive adds the tiles' units in block order and
// writes the rows.  Crossing into a new segment, the consumers rebuild the fragment table.
constexpr int kMoeNV = 4;

struct MoeSeg {
    int expert;         // expert id
    int nv;             // pairs in the segment, 1..kMoeNV
    int pair[kMoeNV];   // pair = token * top_k + slot
};

// Relative cost of one tile of a segment by its table columns (1, 2 or 4 vectors): the
// dequantisation is shared, the MMAs and fragment loads grow with the vectors (instruction
// counts of the Q4_K unit: about 1 : 1.26 : 1.78).
__host__ __device__ constexpr int moe_tile_cost(int nv) { return nv == 1 ? 4 : nv == 2 ? 5 : 7; }

// Block-wide inclusive scan of v (blockDim.x a multiple of 32, s_warp[32] scratch).
__device__ __forceinline__ int block_scan_incl(int v, int* s_warp) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int tv = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += tv;
    }
    __syncthreads();  // s_warp may still be read by a previous scan
    if (lane == 31) s_warp[wid] = v;
    __syncthreads();
    if (wid == 0) {
        const int nw = (int)(blockDim.x >> 5);
        int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int tv = __shfl_up_sync(kFull, w, o);
            if (lane >= o) w += tv;
        }
        if (lane < nw) s_warp[lane] = w;  // inclusive totals per warp
    }
    __syncthreads();
    return v + (wid > 0 ? s_warp[wid - 1] : 0);
}

// First tile (in the concatenation of S segments of tps tiles) at cost position q, where
// segment s starts at cost wcum[s] * tps and costs w[s] per tile.
__device__ int moe_cost_to_tile(long long q, const int* wcum, const int* w, int S, int tps) {
    if (S == 0 || q >= (long long)wcum[S] * tps) return S * tps;
    int lo = 0, hi = S - 1;  // last segment starting at or before q
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((long long)wcum[mid] * tps <= q) lo = mid;
        else hi = mid - 1;
    }
    return lo * tps + (int)((q - (long long)wcum[lo] * tps + w[lo] - 1) / w[lo]);
}

// Group the routed pairs sid[0..P) (in shared memory) into segments of <= kMoeNV pairs of
// one expert, experts in id order and each expert's pairs in pair order, then cut both GEMVs'
// tile sequences into C ranges of equal cost: ranges[0..C] over tps_a tiles per segment
// (gate/up), ranges[C+1..2C+1] over tps_b (down).  nseg[0] = segments.
// Every pair finds its own place in O(P / 32 + 1) steps: warp w takes pairs [32w, 32w + 32)
// in rounds; __match_any_sync gives a pair's rank among the same expert's pairs of its group
// of 32 and the group's count per expert (hist, one byte per (group, expert)); the expert's
// total, its rank offset from the earlier groups and, after two block scans over the experts,
// its first segment and cost follow.  The result equals a sequential pass over the pairs.
// Scratch in shared memory: wcum [P + 1], wseg [P], hist [ceil(P / 32) x nE] bytes, sbase and
// swbase [nE] each.  Every thread of the block calls it (blockDim.x a multiple of 32).
__device__ void group_pairs(const int* sid, int P, int e_lo, int e_hi, MoeSeg* __restrict__ segs, int* __restrict__ nseg,
                            int C, int tps_a, int tps_b, int* __restrict__ ranges, int* wcum, int* wseg, uint8_t* hist,
                            int* sbase, int* swbase, int* s_warp, int* s_tot) {
    const int nE = e_hi - e_lo, nG = (P + 31) >> 5;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (int)(blockDim.x >> 5);
    for (int i = threadIdx.x; i < ((nG * nE + 3) >> 2); i += blockDim.x) reinterpret_cast<uint32_t*>(hist)[i] = 0u;
    __syncthreads();
    // counts per (group, expert)
    for (int g = warp; g < nG; g += nw) {
        const int p = 32 * g + lane;
        int e = p < P ? sid[p] - e_lo : -1;
        const bool held = e >= 0 && e < nE;  // (expert parallelism: other ranks' experts are skipped)
        if (!held) e = -1 - lane;            // distinct keys for the pairs not grouped here
        const unsigned same = __match_any_sync(kFull, e);
        if (held && (same & ((1u << lane) - 1u)) == 0u) hist[g * nE + e] = (uint8_t)__popc(same);
    }
    __syncthreads();
    // per expert: pairs, segments and cost; block scans give each expert its first segment
    int base_s = 0, base_w = 0;
    for (int e0 = 0; e0 < nE; e0 += blockDim.x) {
        const int e = e0 + (int)threadIdx.x;
        int n = 0;
        if (e < nE)
            for (int g = 0; g < nG; ++g) n += hist[g * nE + e];
        const int ns = (n + kMoeNV - 1) / kMoeNV;
        const int full = n / kMoeNV, rem = n - full * kMoeNV;
        const int wexp = full * moe_tile_cost(kMoeNV) + (rem ? moe_tile_cost(rem > 2 ? kMoeNV : rem) : 0);
        const int sincl = block_scan_incl(ns, s_warp);
        const int wincl = block_scan_incl(wexp, s_warp);
        if (e < nE) {
            sbase[e] = base_s + sincl - ns;
            swbase[e] = base_w + wincl - wexp;
        }
        if (threadIdx.x == blockDim.x - 1) {
            s_tot[0] = base_s + sincl;
            s_tot[1] = base_w + wincl;
        }
        __syncthreads();
        base_s = s_tot[0];
        base_w = s_tot[1];
        __syncthreads();
    }
    // every pair to its slot
    for (int g = warp; g < nG; g += nw) {
        const int p = 32 * g + lane;
        int e = p < P ? sid[p] - e_lo : -1;
        const bool held = e >= 0 && e < nE;
        if (!held) e = -1 - lane;
        const unsigned same = __match_any_sync(kFull, e);
        if (held) {
            int r = __popc(same & ((1u << lane) - 1u)), n = 0;
            for (int h = 0; h < nG; ++h) {
                const int c = hist[h * nE + e];
                n += c;
                if (h < g) r += c;
            }
            const int si = sbase[e] + r / kMoeNV;
            MoeSeg& sg = segs[si];
            sg.pair[r % kMoeNV] = p;
            if (r % kMoeNV == 0) {
                const int nv = min(kMoeNV, n - r);
                sg.expert = e_lo + e;
                sg.nv = nv;
                wcum[si] = swbase[e] + (r / kMoeNV) * moe_tile_cost(kMoeNV);
                wseg[si] = moe_tile_cost(nv > 2 ? kMoeNV : nv);
            }
        }
    }
    __syncthreads();
    const int S = base_s;
    if (threadIdx.x == 0) {
        wcum[S] = base_w;
        *nseg = S;
    }
    __syncthreads();
    for (int c = threadIdx.x; c <= C; c += blockDim.x) {
        const long long ca = (long long)wcum[S] * tps_a, cb = (long long)wcum[S] * tps_b;
        ranges[c] = moe_cost_to_tile(ca * c / C, wcum, wseg, S, tps_a);
        ranges[C + 1 + c] = moe_cost_to_tile(cb * c / C, wcum, wseg, S, tps_b);
    }
}

// Shared memory of the grouping step for P pairs over nE experts (ids, then group_pairs'
// scratch), in bytes.
__host__ __device__ constexpr size_t group_smem_bytes(int P, int nE) {
    return (size_t)(3 * P + 1) * 4 + (((size_t)((P + 31) / 32) * nE + 3) / 4) * 4 + 2 * (size_t)nE * 4;
}

__global__ void moe_group_kernel(const int32_t* __restrict__ ids, int P, int e_lo, int e_hi, MoeSeg* __restrict__ segs,
                                 int* __restrict__ nseg, int C, int tps_a, int tps_b, int* __restrict__ ranges) {
    extern __shared__ int sh[];  // [P] ids | group_pairs' scratch (group_smem_bytes)
    __shared__ int s_warp[32];
    __shared__ int s_tot[2];
    for (int p = threadIdx.x; p < P; p += blockDim.x) sh[p] = ids[p];
    __syncthreads();
    const int nE = e_hi - e_lo;
    uint8_t* hist = reinterpret_cast<uint8_t*>(sh + 3 * P + 1);
    int* sb = reinterpret_cast<int*>(hist + (((size_t)((P + 31) / 32) * nE + 3) / 4) * 4);
    group_pairs(sh, P, e_lo, e_hi, segs, nseg, C, tps_a, tps_b, ranges, sh + P, sh + 2 * P + 1, hist, sb, sb + nE,
                s_warp, s_tot);
}

// Routing and grouping in one block for up to 32 tokens and 256 experts (the decode-batch
// case): warp t routes token t with its scores in registers (k rounds of a warp arg-max over
// the experts not yet chosen, ties to the lower id: the reference's stable descending sort,
// moe_infer.rs:852-862; softmax or sigmoid weights, renorm and scaling, :906-932, with
// warp-tree max and sum), the ids go to shared memory, then the block groups the pairs.
constexpr int kRouteRegs = 8;  // scores per lane: E <= 256

__global__ void route_group_kernel(const float* __restrict__ scores, const float* __restrict__ bias, int T, RouteMeta m,
                                   int32_t* __restrict__ ids, float* __restrict__ wout, int e_lo, int e_hi,
                                   MoeSeg* __restrict__ segs, int* __restrict__ nseg, int C, int tps_a, int tps_b,
                                   int* __restrict__ ranges) {
    extern __shared__ int sh[];  // [P] ids | group_pairs' scratch (group_smem_bytes)
    __shared__ int s_warp[32];
    __shared__ int s_tot[2];
    const int P = T * m.k;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < T) {
        const float* sc = scores + (size_t)warp * m.E;
        float v[kRouteRegs], b[kRouteRegs];
#pragma unroll
        for (int q = 0; q < kRouteRegs; ++q) {
            const int j = lane + 32 * q;
            v[q] = j < m.E ? sc[j] : -INFINITY;
            b[q] = j < m.E ? (bias ? v[q] + bias[j] : v[q]) : -INFINITY;
        }
        unsigned taken = 0u;
        int myid[16];  // chosen ids (k <= 16 here), replicated in every lane
        for (int r = 0; r < m.k; ++r) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int q = 0; q < kRouteRegs; ++q) {
                const int j = lane + 32 * q;
                if (j < m.E && !((taken >> q) & 1u) && (bi == 0x7fffffff || ranks_before(b[q], j, bv, bi))) {
                    bv = b[q];
                    bi = j;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(kFull, bv, o);
                const int oi = __shfl_xor_sync(kFull, bi, o);
                if (oi != 0x7fffffff && (bi == 0x7fffffff || ranks_before(ov, oi, bv, bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            myid[r] = bi;
            if (lane == 0) {
                ids[(size_t)warp * m.k + r] = bi;
                sh[warp * m.k + r] = bi;
            }
        }
        // weights of the chosen ids from the raw scores
        float w[16];
        float mx = -INFINITY, sum = 0.f;
        if (m.gating != 1) {
#pragma unroll
            for (int q = 0; q < kRouteRegs; ++q) mx = fmaxf(mx, v[q]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
#pragma unroll
            for (int q = 0; q < kRouteRegs; ++q)
                if (lane + 32 * q < m.E) sum += expf(v[q] - mx);
            sum = warp_sum(sum);
        }
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        float wsum = 0.f;
        for (int r = 0; r < m.k; ++r) {
            const int id = myid[r];
            float sv = 0.f;  // the chosen expert's raw score, from the lane that holds it
#pragma unroll
            for (int q = 0; q < kRouteRegs; ++q)
                if (id == lane + 32 * q) sv = v[q];
            sv = __shfl_sync(kFull, sv, id & 31);
            w[r] = m.gating == 1 ? 1.0f / (1.0f + expf(-sv)) : expf(sv - mx) * inv;
            wsum += w[r];
        }
        if (lane == 0) {
            for (int r = 0; r < m.k; ++r) {
                float x = w[r];
                if (m.norm_topk_prob && wsum > 0.0f) x /= wsum;
                if (fabsf(m.scale - 1.0f) > 1e-9f) x *= m.scale;
                wout[(size_t)warp * m.k + r] = x;
            }
        }
    }
    __syncthreads();
    const int nE = e_hi - e_lo;
    uint8_t* hist = reinterpret_cast<uint8_t*>(sh + 3 * P + 1);
    int* sb = reinterpret_cast<int*>(hist + (((size_t)((P + 31) / 32) * nE + 3) / 4) * 4);
    group_pairs(sh, P, e_lo, e_hi, segs, nseg, C, tps_a, tps_b, ranges, sh + P, sh + 2 * P + 1, hist, sb, sb + nE,
                s_warp, s_tot);
}

struct MoeTmaArgs {
    const MoeSeg* segs;
    const int* nseg;
    const int* ranges;  // [gridDim.x + 1] first tile of every CTA (cost-balanced)
    const uint8_t* const* w;   // [experts held] gate (fused) or down matrices, tile-major
    const uint8_t* const* w2;  // [experts held] up matrices (fused)
    int e_lo;                  // expert id of w[0]
    long long tstride;         // bytes per 16-row tile
    int M, K;
    const float* x;  // input row of pair p: x + (p / x_div) * ldx
    int x_div, ldx;
    float* y;  // output row of pair p: y + p * ldy (or region_off in every region)
    int ldy;
    // expert parallelism: output rows go to every rank's region at region_base + buffer
    // (epoch & 1) * buf_bytes, epoch = this rank's signalled phases (read on the device)
    char* const* regions;
    int n_regions;
    size_t region_base, buf_bytes;
    const unsigned* epoch;
    int stages;
    int* err;
};

struct MoeSmem {
    int table, zero, sx, red, ring;
};

template <class F>
__host__ __device__ inline MoeSmem moe_smem_layout(int K, int stages) {
    const GemvSmem g = gemv_smem_layout<F>(K, kMoeNV, false);
    MoeSmem s;
    s.table = 128;
    s.zero = s.table + g.table_bytes;
    s.sx = s.zero + g.zero_bytes;
    s.red = s.sx + g.sx_bytes;
    s.ring = (s.red + (stages + 2) * tile_slot_bytes(kMoeNV) + 127) & ~127;
    return s;
}

// Stages of a CTA's tile range: runs of whole tiles inside one segment, at most tps_stage.
struct MoeStageIt {
    int gt, t1, tps, tps_stage;
    __device__ bool next(int& sg, int& tile, int& nt) {
        if (gt >= t1) return false;
        sg = gt / tps;
        tile = gt - sg * tps;
        nt = min(min(tps_stage, tps - tile), t1 - gt);
        gt += nt;
        return true;
    }
};

// One consumer warp's unit of a stage for a segment of class NVC (1, 2 or 4 vectors): the
// tensor-core unit (skipped when tb is null: the warp has no unit in this stage) and the
// warp's partials into red_w.  The fragment-table context is the same struct for every NV.
template <class F, int NVC>
__device__ __forceinline__ void moe_unit(const uint8_t* tb, int kbj, const LaneCtx<kMoeNV>& c, float* red_w) {
    const LaneCtx<NVC> ctx{c.xb0, c.xstride, c.sx, c.sxs, c.g, c.t};
    float yA = 0.f, yB = 0.f;
    float pA[1][NVC], pB[1][NVC];
#pragma unroll
    for (int v = 0; v < NVC; ++v) pA[0][v] = pB[0][v] = 0.f;
    if (tb) stage_unit<F, NVC>(tb, kbj, ctx, yA, yB, pA, pB);
    warp_partials<F, NVC>(red_w, c.g, c.t, yA, yB, pA, pB);
}

// Fragment table and lane context for a segment of class NVC.
template <class F, int NVC>
__device__ __forceinline__ LaneCtx<kMoeNV> moe_table(uint2* xt, uint2* zero, float* sx, int K, const float* const* rows,
                                                     float* scratch, int* err, int lane) {
    const NormArgs nrm{nullptr, 0, 0.f};
    build_prologue<F, NVC, kLdcg>(xt, sx, nullptr, 0, K, NVC, nrm, scratch, err, kCW * 32, kBarPro,
                                  XAccum{nullptr, 0, nullptr, 0, 0}, rows);
    const LaneCtx<NVC> c = make_ctx<F, NVC>(xt, zero, sx, K, lane);
    return LaneCtx<kMoeNV>{c.xb0, c.xstride, c.sx, c.sxs, c.g, c.t};
}

// A stage as the producer remembers it until it reduces it.
struct MoeStageRec {
    int tile, nt, nv;
    int pair[kMoeNV];
};

template <class F, bool FUSED>
__global__ void __launch_bounds__(kTThreads, 1) moe_tma_kernel(MoeTmaArgs a) {
    constexpr int NV = kMoeNV, kMats = FUSED ? 2 : 1, SB = stage_blocks(FUSED);
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[32];
    __shared__ const float* s_rows[NV];
    __shared__ int s_nv;
    __shared__ MoeStageRec s_rec[kMaxStages];  // producer: the stage in each ring slot
    const int S = a.stages;
    const MoeSmem L = moe_smem_layout<F>(a.K, S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring r;
    r.full0 = smem_addr(smem);
    r.empty0 = r.full0 + 8 * kMaxStages;
    r.base = smem + L.ring;
    r.base_s = smem_addr(r.base);
    r.S = S;
    r.slot_bytes = tma_stage_bytes<F>(FUSED);
    r.slot = r.round = 0;
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;  // <= SB (checked at launch)
    const int tps = (a.M + 15) / 16;
    const int NT = S + 2;  // partial slots (stage m -> m % NT)
    float* red = reinterpret_cast<float*>(smem + L.red);
    MoeStageIt it{__ldcg(a.ranges + blockIdx.x), __ldcg(a.ranges + blockIdx.x + 1), tps, SB / nbk};

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(r.full0 + 8 * s, 1);
            mbar_init(r.empty0 + 8 * s, kCW);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kCW) {
        // Producer: stream the stages, and reduce each stage once its slot comes back (the
        // consumers release a slot only after writing their partials): tile t of the stage,
        // row, vector v = sum over the tile's blocks (and matrices) in block order.
        size_t region_off = 0;
        if (a.regions) region_off = a.region_base + (size_t)(__ldcg(a.epoch) & 1u) * a.buf_bytes;
        auto reduce = [&](int m) {  // stage m, its record in s_rec[m % S]
            const MoeStageRec& d = s_rec[m % S];
            const float* rr = red + (size_t)(m % NT) * kCW * NV * 16;
            const int outs = d.nt * 16 * d.nv;
            for (int o = lane; o < outs; o += 32) {
                const int v = o % d.nv, rowi = o / d.nv, i = rowi >> 4, row = rowi & 15;
                const int grow = (d.tile + i) * 16 + row;
                float f[kMats];
#pragma unroll
                for (int mm = 0; mm < kMats; ++mm) {
                    float acc = 0.f;
                    for (int b = 0; b < nbk; ++b) acc += rr[((mm * SB + i * nbk + b) * NV + v) * 16 + row];
                    f[mm] = acc;
                }
                if (grow < a.M) {
                    float val = f[0];
                    if constexpr (FUSED) val = silu_mul(f[0], f[kMats - 1]);
                    const size_t off = (size_t)d.pair[v] * a.ldy + grow;
                    if (a.regions) {
                        for (int q2 = 0; q2 < a.n_regions; ++q2)
                            reinterpret_cast<float*>(a.regions[q2] + region_off)[off] = val;
                    } else {
                        a.y[off] = val;
                    }
                }
            }
        };
        bool ok = true;
        int sg, tile, nt, cur_sg = -1, nv = 0, m = 0;  // m = stages issued
        int pr[NV] = {0, 0, 0, 0};
        const uint8_t* wbase = nullptr;  // this lane's matrix of the current segment's expert
        while (ok && it.next(sg, tile, nt)) {
            if (sg != cur_sg) {  // once per segment: expert, its matrices, the pairs
                const MoeSeg& sgd = a.segs[sg];
                const int e = __ldg(&sgd.expert) - a.e_lo;
                nv = __ldg(&sgd.nv);
#pragma unroll
                for (int v = 0; v < NV; ++v) pr[v] = __ldg(&sgd.pair[v]);
                if (lane < kMats) wbase = lane ? a.w2[e] : a.w[e];
                cur_sg = sg;
            }
            if (r.round > 0 && !mbar_wait(r.empty0 + 8 * r.slot, (r.round - 1) & 1)) {
                ok = false;
                break;
            }
            const uint32_t bytes = (uint32_t)(nt * nbk * F::kTile), full = r.full0 + 8 * r.slot;
            if (lane == 0) mbar_arrive_expect_tx(full, kMats * bytes);
            __syncwarp();
            if (lane < kMats)
                bulk_g2s(r.base_s + r.slot * r.slot_bytes + lane * SB * F::kTile, wbase + (size_t)tile * a.tstride,
                         bytes, full);
            if (m >= S) reduce(m - S);  // the slot's previous stage, consumed and flushed
            __syncwarp();
            if (lane == 0) {
                MoeStageRec& rec = s_rec[r.slot];
                rec.tile = tile;
                rec.nt = nt;
                rec.nv = nv;
#pragma unroll
                for (int v = 0; v < NV; ++v) rec.pair[v] = pr[v];
            }
            __syncwarp();
            r.advance();
            ++m;
        }
        // the last stages: wait until consumed (their copies landed), then reduce
        for (int q = m - S < 0 ? 0 : m - S; q < m; ++q) {
            if (!mbar_wait(r.empty0 + 8 * (q % S), (q / S) & 1)) {
                ok = false;
                break;
            }
            if (ok) reduce(q);
        }
        if (!ok && lane == 0 && a.err) atomicOr(a.err, 2);
        if (a.regions) __threadfence_system();  // the peer stores, before the rank's signal kernel
        return;
    }

    uint2* xt = reinterpret_cast<uint2*>(smem + L.table);
    uint2* zero = reinterpret_cast<uint2*>(smem + L.zero);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    for (int i = threadIdx.x; i < table_entries_per_block<F>(NV); i += kCW * 32) zero[i] = make_uint2(0u, 0u);
    const int mt = warp_matrix(warp, FUSED), j = warp % SB;  // this warp's matrix and unit
    int cur = -1, m = 0, nvc = NV;
    bool aborted = false;
    LaneCtx<NV> ctx{};
    int sg, tile, nt;
    while (it.next(sg, tile, nt)) {
        if (sg != cur) {  // new segment: rebuild the fragment table for its pairs
            named_bar_sync(kBarPro, kCW * 32);  // every warp is done with the old table
            if (threadIdx.x < NV) {
                const MoeSeg& sgd = a.segs[sg];
                const int nv = sgd.nv, p = sgd.pair[threadIdx.x];
                s_rows[threadIdx.x] = (int)threadIdx.x < nv ? a.x + (size_t)(p / a.x_div) * a.ldx : nullptr;
                if (threadIdx.x == 0) s_nv = nv;
            }
            named_bar_sync(kBarPro, kCW * 32);
            // the segment's vectors as 1, 2 or 4 table columns (the MMA work grows with them)
            const int nv = s_nv;
            nvc = nv == 1 ? 1 : nv == 2 ? 2 : NV;
            if (nvc == 1)
                ctx = moe_table<F, 1>(xt, zero, sx, a.K, s_rows, s_red, a.err, lane);
            else if (nvc == 2)
                ctx = moe_table<F, 2>(xt, zero, sx, a.K, s_rows, s_red, a.err, lane);
            else
                ctx = moe_table<F, NV>(xt, zero, sx, a.K, s_rows, s_red, a.err, lane);
            named_bar_sync(kBarPro, kCW * 32);
            cur = sg;
        }
        if (!aborted && !mbar_wait(r.full0 + 8 * r.slot, r.round & 1)) {
            aborted = true;
            if (lane == 0 && a.err) atomicOr(a.err, 2);
        }
        // this warp's unit and its partials (vector stride 16 floats), then the slot goes back
        const uint8_t* tb =
            !aborted && j < nt * nbk ? r.base + r.slot * r.slot_bytes + (mt * SB + j) * F::kTile : nullptr;
        float* red_w = red + (size_t)((m % NT) * kCW + warp) * NV * 16;
        if (nvc == 1)
            moe_unit<F, 1>(tb, j % nbk, ctx, red_w);
        else if (nvc == 2)
            moe_unit<F, 2>(tb, j % nbk, ctx, red_w);
        else
            moe_unit<F, NV>(tb, j % nbk, ctx, red_w);
        __syncwarp();
        if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
        r.advance();
        ++m;
    }
}

template <class F, bool FUSED>
static cudaError_t launch_moe_tma_t(const MoeTmaArgs& a0, int num_sms, int smem_limit, cudaStream_t stream) {
    MoeTmaArgs a = a0;
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    if (nbk > stage_blocks(FUSED)) return cudaErrorInvalidConfiguration;  // a tile must fit one stage
    const int fixed = moe_smem_layout<F>(a.K, 0).ring + 512;
    int S = (smem_limit - fixed) / (tma_stage_bytes<F>(FUSED) + tile_slot_bytes(kMoeNV));
    if (S > kMaxStages) S = kMaxStages;
    if (S < 2) return cudaErrorInvalidConfiguration;
    a.stages = S;
    const int smem = moe_smem_layout<F>(a.K, S).ring + S * tma_stage_bytes<F>(FUSED);
    auto kern = moe_tma_kernel<F, FUSED>;
    static int configured[64];  // per instantiation and device: set once (not inside a graph capture)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || configured[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev] = smem;
    }
    kern<<<num_sms, kTThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

static cudaError_t launch_moe_tma(int type, bool fused, const MoeTmaArgs& a, int num_sms, int smem_limit,
                                  cudaStream_t stream) {
    switch (type) {
        case T_Q4_K: return fused ? launch_moe_tma_t<FmtQ4K, true>(a, num_sms, smem_limit, stream)
                                  : launch_moe_tma_t<FmtQ4K, false>(a, num_sms, smem_limit, stream);
        case T_Q6_K: return fused ? launch_moe_tma_t<FmtQ6K, true>(a, num_sms, smem_limit, stream)
                                  : launch_moe_tma_t<FmtQ6K, false>(a, num_sms, smem_limit, stream);
        case T_Q8_0: return fused ? launch_moe_tma_t<FmtQ80, true>(a, num_sms, smem_limit, stream)
                                  : launch_moe_tma_t<FmtQ80, false>(a, num_sms, smem_limit, stream);
        default: return cudaErrorInvalidValue;
    }
}

static bool moe_tma_fits(int type, bool fused, int K) {
    const int be = type == T_Q8_0 ? 128 : 256;
    return (K + be - 1) / be <= stage_blocks(fused);
}

template <class F, bool FUSED>
static cudaError_t launch_stage(const MoeStage& s, int P, int smem_limit, cudaStream_t stream) {
    const int smem = gemv_smem_layout<F>(s.K, 1, FUSED).total();
    if (smem > smem_limit) return cudaErrorInvalidConfiguration;
    auto kern = moe_gemv_kernel<F, FUSED>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
    }
    kern<<<P * s.items_per_pair, 256, smem, stream>>>(s);
    return cudaGetLastError();
}

static cudaError_t launch_moe_stage(int type, bool fused, const MoeStage& s, int P, int smem_limit,
                                    cudaStream_t stream) {
    switch (type) {
        case T_Q4_K: return fused ? launch_stage<FmtQ4K, true>(s, P, smem_limit, stream) : launch_stage<FmtQ4K, false>(s, P, smem_limit, stream);
        case T_Q6_K: return fused ? launch_stage<FmtQ6K, true>(s, P, smem_limit, stream) : launch_stage<FmtQ6K, false>(s, P, smem_limit, stream);
        case T_Q8_0: return fused ? launch_stage<FmtQ80, true>(s, P, smem_limit, stream) : launch_stage<FmtQ80, false>(s, P, smem_limit, stream);
        default: return cudaErrorInvalidValue;
    }
}

static int stage_wk(int type, int K) {
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nb = (K + be - 1) / be;
    int wk = 8;
    while (wk > 1 && nb < wk) wk >>= 1;
    return wk;
}

}  // namespace hc

// ------------------------------------------------------------------ C ABI

extern "C" int hc_router_scores_dev(hc_engine* e, const float* W, size_t E, size_t D, const float* x, size_t T,
                                    float* scores) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!W || !x || !scores || E == 0 || D == 0) return hc_set_error(HC_ERR_INVALID, "router: bad argument");
    if (T == 0) return HC_OK;
    HC_CUDA(launch_router(W, x, (int)E, (int)D, (int)T, scores, e->smem_optin, e->stream, e->d_err));
    return HC_OK;
}

static int route_dev(hc_engine* e, const float* scores, const float* bias, size_t T, size_t E, size_t k,
                     size_t n_group, size_t topk_group, int gating, int norm, float scale, int32_t* ids, float* w) {
    if (!scores || !ids || !w || E == 0 || k == 0) return hc_set_error(HC_ERR_INVALID, "route_experts: bad argument");
    if (k > E) return hc_set_error(HC_ERR_INVALID, "route_experts: top_k=%zu > n_expert=%zu", k, E);
    if (E > 2048) return hc_set_error(HC_ERR_INVALID, "route_experts: n_expert=%zu > 2048", E);
    if (T == 0) return HC_OK;
    RouteMeta m{(int)E, (int)k, (int)n_group, (int)topk_group, gating, norm, scale};
    const bool grouped = n_group > 0 && topk_group > 0 && E % n_group == 0;
    if (!grouped) {
        route_topk_warp_kernel<<<(unsigned)((T + 3) / 4), 128, 0, e->stream>>>(scores, bias, (int)T, m, ids, w);
    } else {
        int rc = e->ws_misc.ensure(T * E * 16 + 64);
        if (rc) return rc;
        route_general_kernel<<<(unsigned)((T + 63) / 64), 64, 0, e->stream>>>(scores, bias, (int)T, m, ids, w,
                                                                              (float*)e->ws_misc.p);
    }
    HC_CUDA(cudaGetLastError());
    return HC_OK;
}

extern "C" int hc_route_experts_dev(hc_engine* e, const float* scores, const float* bias, size_t T, size_t E,
                                    size_t k, size_t n_group, size_t topk_group, int gating, int norm, float scale,
                                    int32_t* ids, float* w) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    return route_dev(e, scores, bias, T, E, k, n_group, topk_group, gating, norm, scale, ids, w);
}

// Device table of expert base pointers, cached per weight set.
static int expert_table(hc_engine* e, const hc_weights* const* ws, size_t E, const uint8_t* const** out) {
    uint64_t key = 1469598103934665603ull;
    for (size_t i = 0; i < E; ++i) key = (key ^ (uint64_t)(uintptr_t)ws[i]->dev) * 1099511628211ull;
    key ^= E;
    auto it = e->ptr_tables.find(key);
    if (it == e->ptr_tables.end()) {
        std::vector<const void*> host(E);
        for (size_t i = 0; i < E; ++i) host[i] = ws[i]->dev;
        void* d = nullptr;
        HC_CUDA(cudaMalloc(&d, E * sizeof(void*)));
        cudaError_t ce = cudaMemcpy(d, host.data(), E * sizeof(void*), cudaMemcpyHostToDevice);
        if (ce != cudaSuccess) {
            cudaFree(d);
            return hc_cuda_error(ce, "expert table upload");
        }
        it = e->ptr_tables.emplace(key, d).first;
    }
    *out = (const uint8_t* const*)it->second;
    return HC_OK;
}

// Expert parallelism of one call: experts [lo, lo + n) are held here; the down rows of their
// pairs are stored into every rank's exchange region and combined after a cross-GPU signal.
struct EpRun {
    size_t lo, n;
};

// Bytes of moe_run's workspace for T tokens, top-k, E experts.
static size_t moe_ws_bytes(size_t T, size_t E, size_t k, size_t dm, size_t ff, size_t* off_ids, size_t* off_w,
                           size_t* off_h, size_t* off_d, size_t* off_seg, size_t* off_nseg) {
    const size_t P = T * k;
    *off_ids = T * E * 4;
    *off_w = *off_ids + P * 4;
    *off_h = (*off_w + P * 4 + 255) / 256 * 256;
    *off_d = *off_h + P * ff * 4;
    *off_seg = (*off_d + P * dm * 4 + 255) / 256 * 256;
    *off_nseg = *off_seg + P * sizeof(MoeSeg);
    return *off_nseg + 256 + 2 * (1024 + 1) * 4;  // count | cost-balanced CTA ranges of both GEMVs
}

// y = [resid +] MoE(x); resid may alias y (the residual stream updated in place).
static int moe_run(hc_engine* e, const float* router_w, size_t E, size_t k, int norm, float scale,
                   const hc_weights* const* gate, const hc_weights* const* up, const hc_weights* const* down,
                   const float* x, size_t T, float* y, int32_t* ids_out, float* w_out, const EpRun* ep,
                   const float* resid = nullptr) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!router_w || !gate || !up || !down || !x || !y || E == 0 || k == 0 || k > E)
        return hc_set_error(HC_ERR_INVALID, "moe_ffn: bad argument");
    const size_t n_held = ep ? ep->n : E, lo = ep ? ep->lo : 0;
    if (n_held == 0 || lo + n_held > E) return hc_set_error(HC_ERR_INVALID, "moe_ffn: experts [%zu, %zu) of %zu", lo, lo + n_held, E);
    const hc_weights *g0 = gate[0], *u0 = up[0], *d0 = down[0];
    if (!g0 || !u0 || !d0) return hc_set_error(HC_ERR_INVALID, "moe_ffn: null expert weights");
    for (size_t i = 0; i < n_held; ++i) {
        const hc_weights *g = gate[i], *u = up[i], *d = down[i];
        if (!g || !u || !d || g->type != g0->type || u->type != g0->type || d->type != d0->type || g->m != g0->m ||
            g->n != g0->n || u->m != g0->m || u->n != g0->n || d->m != d0->m || d->n != d0->n)
            return hc_set_error(HC_ERR_INVALID, "moe_ffn: expert %zu differs in type or shape from expert %zu", lo + i, lo);
        if (g->device != e->device || u->device != e->device || d->device != e->device)
            return hc_set_error(HC_ERR_INVALID, "moe_ffn: expert %zu lives on another device", lo + i);
    }
    const size_t dm = g0->n, ff = g0->m;
    if (d0->n != ff || d0->m != dm) return hc_set_error(HC_ERR_INVALID, "moe_ffn: down must be d_model x d_ff");
    auto routed = [](int t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0; };
    if (!routed(g0->type) || !routed(d0->type))
        return hc_set_error(HC_ERR_UNSUPPORTED, "moe_ffn: expert format %s/%s has no routed kernel",
                            hc_type_label(g0->type), hc_type_label(d0->type));
    if (((uintptr_t)x & 15) || (dm & 3)) return hc_set_error(HC_ERR_INVALID, "moe_ffn: x must be 16-byte aligned");
    const size_t P = T * k;
    PeerState& pe = e->peer;
    if (ep) {
        if (!pe.connected) return hc_set_error(HC_ERR_INVALID, "expert-parallel MoE without a connected peer group");
        // the EP rows must stay inside their own area: the batched tensor-parallel exchange
        // owns the bytes after it
        if (2 * P * dm * 4 > kPeerEpDataBytes || pe.bytes < kPeerEpData + 2 * P * dm * 4)
            return hc_set_error(HC_ERR_INVALID,
                                "expert-parallel MoE: %zu tokens x top-%zu x %zu need %zu exchange bytes; the EP area "
                                "holds %zu",
                                T, k, dm, 2 * P * dm * 4, (size_t)kPeerEpDataBytes);
    }
    if (T == 0) return HC_OK;
    // workspace: scores [T][E] | ids [P] | w [P] | h [P][ff] | D [P][dm] | segments [P] | count
    size_t off_ids, off_w, off_h, off_d, off_seg, off_nseg;
    const size_t total = moe_ws_bytes(T, E, k, dm, ff, &off_ids, &off_w, &off_h, &off_d, &off_seg, &off_nseg);
    rc = e->ws_h.ensure(total);
    if (rc) return rc;
    uint8_t* base = (uint8_t*)e->ws_h.p;
    float* scores = (float*)base;
    int32_t* ids = ids_out ? ids_out : (int32_t*)(base + off_ids);
    float* wts = w_out ? w_out : (float*)(base + off_w);
    float* h = (float*)(base + off_h);
    float* D = (float*)(base + off_d);
    const uint8_t* const* tg;
    const uint8_t* const* tu;
    const uint8_t* const* td;
    rc = expert_table(e, gate, n_held, &tg);
    if (!rc) rc = expert_table(e, up, n_held, &tu);
    if (!rc) rc = expert_table(e, down, n_held, &td);
    if (rc) return rc;

    // router and top-k: on every rank alike (x and the router are replicated)
    HC_CUDA(launch_router(router_w, x, (int)E, (int)dm, (int)T, scores, e->smem_optin, e->stream, e->d_err));
    const bool tma = moe_tma_fits(g0->type, true, (int)dm) && moe_tma_fits(d0->type, false, (int)ff) && n_held <= 1024 &&
                     group_smem_bytes((int)P, (int)n_held) <= 48 * 1024 && ff % 4 == 0 && e->num_sms <= 1024;
    // decode batches: routing and grouping in one block
    const bool fused_route = tma && T <= 32 && E <= 32 * kRouteRegs && k <= 16;
    if (!fused_route) {
        rc = route_dev(e, scores, nullptr, T, E, k, 0, 0, 0, norm, scale, ids, wts);
        if (rc) return rc;
    }
    if (ep && !tma)
        return hc_set_error(HC_ERR_UNSUPPORTED, "expert-parallel MoE: expert shapes need the grouped pipeline "
                                                "(gate/up K <= 8 and down K <= 16 kernel blocks)");
    if (tma) {
        // expert-grouped pipeline: segments of <= 4 pairs per expert, then the two GEMVs
        MoeSeg* segs = (MoeSeg*)(base + off_seg);
        int* nseg = (int*)(base + off_nseg);
        int* ranges = nseg + 64;
        const int C = e->num_sms;
        if (fused_route) {
            const RouteMeta rm{(int)E, (int)k, 0, 0, 0, norm, scale};
            const size_t nthr = std::max<size_t>(32 * T, (n_held + 31) / 32 * 32);
            route_group_kernel<<<1, (unsigned)nthr, group_smem_bytes((int)P, (int)n_held), e->stream>>>(
                scores, nullptr, (int)T, rm, ids, wts, (int)lo, (int)(lo + n_held), segs, nseg, C, (int)((ff + 15) / 16),
                (int)((dm + 15) / 16), ranges);
        } else {
            const unsigned gthreads = (unsigned)std::min<size_t>(1024, std::max<size_t>(P, n_held) + 31) / 32 * 32;
            moe_group_kernel<<<1, gthreads, group_smem_bytes((int)P, (int)n_held), e->stream>>>(ids, (int)P, (int)lo, (int)(lo + n_held),
                                                                         segs, nseg, C, (int)((ff + 15) / 16),
                                                                         (int)((dm + 15) / 16), ranges);
        }
        HC_CUDA(cudaGetLastError());
        MoeTmaArgs a1{};
        a1.segs = segs;
        a1.nseg = nseg;
        a1.ranges = ranges;
        a1.w = tg;
        a1.w2 = tu;
        a1.e_lo = (int)lo;
        a1.tstride = (long long)g0->stride;
        a1.M = (int)ff;
        a1.K = (int)dm;
        a1.x = x;
        a1.x_div = (int)k;
        a1.ldx = (int)dm;
        a1.y = h;
        a1.ldy = (int)ff;
        a1.err = e->d_err;
        cudaError_t ce = launch_moe_tma(g0->type, true, a1, e->num_sms, e->smem_optin, e->stream);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "moe gate/up launch");
        MoeTmaArgs a2 = a1;
        a2.ranges = ranges + C + 1;
        a2.w = td;
        a2.w2 = nullptr;
        a2.tstride = (long long)d0->stride;
        a2.M = (int)dm;
        a2.K = (int)ff;
        a2.x = h;
        a2.x_div = 1;
        a2.ldx = (int)ff;
        a2.y = D;
        a2.ldy = (int)dm;
        if (ep) {
            a2.regions = reinterpret_cast<char* const*>(pe.d_peer);
            a2.n_regions = pe.world;
            a2.region_base = kPeerEpData;
            a2.buf_bytes = P * dm * 4;
            a2.epoch = reinterpret_cast<const unsigned*>(static_cast<char*>(pe.region) + kPeerEpEpoch);
        }
        ce = launch_moe_tma(d0->type, false, a2, e->num_sms, e->smem_optin, e->stream);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "moe down launch");
    } else {
    MoeStage s1{};
    s1.ids = ids;
    s1.w = tg;
    s1.w2 = tu;
    s1.row_stride = (long long)g0->stride;
    s1.M = (int)ff;
    s1.K = (int)dm;
    s1.x = x;
    s1.x_div = (int)k;
    s1.ldx = (int)dm;
    s1.y = h;
    s1.ldy = (int)ff;
    s1.rows_per_item = 128;
    s1.items_per_pair = (int)((ff + 127) / 128);
    s1.wk = stage_wk(g0->type, (int)dm);
    s1.err = e->d_err;
    s1.e_lo = (int)lo;
    s1.e_hi = (int)(lo + n_held);
    cudaError_t ce = launch_moe_stage(g0->type, true, s1, (int)P, e->smem_optin, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "moe gate/up launch");

    MoeStage s2{};
    s2.ids = ids;
    s2.w = td;
    s2.w2 = nullptr;
    s2.row_stride = (long long)d0->stride;
    s2.M = (int)dm;
    s2.K = (int)ff;
    s2.x = h;
    s2.x_div = 1;
    s2.ldx = (int)ff;
    s2.y = D;
    s2.ldy = (int)dm;
    s2.rows_per_item = 128;
    s2.items_per_pair = (int)((dm + 127) / 128);
    s2.wk = stage_wk(d0->type, (int)ff);
    s2.err = e->d_err;
    s2.e_lo = (int)lo;
    s2.e_hi = (int)(lo + n_held);
    ce = launch_moe_stage(d0->type, false, s2, (int)P, e->smem_optin, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "moe down launch");
    }

    const size_t n = T * dm;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    if (ep) {
        char* mine = static_cast<char*>(pe.region);
        ep_signal_kernel<<<1, 32, 0, e->stream>>>(reinterpret_cast<char* const*>(pe.d_peer), pe.world,
                                                  reinterpret_cast<unsigned*>(mine + kPeerEpEpoch));
        HC_CUDA(cudaGetLastError());
        moe_combine_wait_kernel<<<blocks, 256, 0, e->stream>>>(mine, P * dm * 4, wts, (int)T, (int)k, (int)dm, resid, y,
                                                               pe.world, e->d_err);
        HC_CUDA(cudaGetLastError());
    } else {
        moe_combine_kernel<<<blocks, 256, 0, e->stream>>>(D, wts, (int)T, (int)k, (int)dm, resid, y);
        HC_CUDA(cudaGetLastError());
    }
    return HC_OK;
}

// A stack of MoE layers, x <- x + MoE_l(x) (the residual of moe_infer.rs:222-223 callers),
// replayed as one captured CUDA graph per (x, shapes, weights): 5-6 launches per layer go out
// as one graph launch.  Under expert parallelism the exchange epochs live on the device, so
// replays stay in step across the ranks.
static int moe_stack(hc_engine* e, size_t L, const float* const* routers, size_t E, size_t k, int norm, float scale,
                     const hc_weights* const* gate, const hc_weights* const* up, const hc_weights* const* down,
                     size_t lo, size_t n_held, bool ep, float* x, size_t T) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!routers || !gate || !up || !down || !x || L == 0 || n_held == 0)
        return hc_set_error(HC_ERR_INVALID, "moe_stack: bad argument");
    if (!ep && (lo != 0 || n_held != E)) return hc_set_error(HC_ERR_INVALID, "moe_stack: all experts must be held");
    if (T == 0) return HC_OK;
    for (size_t l = 0; l < L * n_held; ++l)
        if (!gate[l] || !up[l] || !down[l]) return hc_set_error(HC_ERR_INVALID, "moe_stack: null expert weights");
    const EpRun run{lo, n_held};
    const size_t dm = gate[0]->n, ff = gate[0]->m;
    size_t o1, o2, o3, o4, o5, o6;
    rc = e->ws_h.ensure(moe_ws_bytes(T, E, k, dm, ff, &o1, &o2, &o3, &o4, &o5, &o6));
    if (rc) return rc;
    const uint8_t* const* tab;
    for (size_t l = 0; l < L && !rc; ++l) {  // device tables exist before any capture
        rc = expert_table(e, gate + l * n_held, n_held, &tab);
        if (!rc) rc = expert_table(e, up + l * n_held, n_held, &tab);
        if (!rc) rc = expert_table(e, down + l * n_held, n_held, &tab);
    }
    if (rc) return rc;
    auto enqueue = [&]() -> int {
        for (size_t l = 0; l < L; ++l) {
            const size_t o = l * n_held;
            int r = moe_run(e, routers[l], E, k, norm, scale, gate + o, up + o, down + o, x, T, x, nullptr, nullptr,
                            ep ? &run : nullptr, x);
            if (r) return r;
        }
        return HC_OK;
    };
    if (!e->use_graphs) return enqueue();
    uint64_t key = 0x4D4F4553ull;  // "MOES"
    auto mixin = [&key](uint64_t v) { key = (key ^ v) * 0x100000001B3ull + 0x9E3779B97F4A7C15ull; };
    mixin((uint64_t)(uintptr_t)x);
    mixin(T);
    mixin(L);
    mixin(E);
    mixin(k);
    mixin((uint64_t)norm);
    uint32_t sb;
    memcpy(&sb, &scale, 4);
    mixin(sb);
    mixin(lo);
    mixin(n_held);
    mixin(ep);
    mixin((uint64_t)(uintptr_t)e->ws_h.p);
    for (size_t l = 0; l < L; ++l) mixin((uint64_t)(uintptr_t)routers[l]);
    for (size_t i = 0; i < L * n_held; ++i) {
        mixin((uint64_t)(uintptr_t)gate[i]->dev);
        mixin((uint64_t)(uintptr_t)up[i]->dev);
        mixin((uint64_t)(uintptr_t)down[i]->dev);
    }
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t graph;
        cudaStream_t caller = e->stream;
        e->stream = e->own_stream;
        cudaError_t ce = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeRelaxed);
        if (ce != cudaSuccess) {
            e->stream = caller;
            return hc_cuda_error(ce, "moe stack capture begin");
        }
        rc = enqueue();
        ce = cudaStreamEndCapture(e->stream, &graph);
        e->stream = caller;
        if (rc) {
            if (ce == cudaSuccess) cudaGraphDestroy(graph);
            return rc;
        }
        if (ce != cudaSuccess) return hc_cuda_error(ce, "moe stack capture");
        cudaGraphExec_t exec;
        ce = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "moe stack graph instantiate");
        it = e->graphs.emplace(key, exec).first;
    }
    HC_CUDA(cudaGraphLaunch(it->second, e->stream));
    return HC_OK;
}

extern "C" int hc_moe_ffn_dev(hc_engine* e, const float* router_w, size_t E, size_t k, int norm, float scale,
                              const hc_weights* const* gate, const hc_weights* const* up,
                              const hc_weights* const* down, const float* x, size_t T, float* y, int32_t* ids_out,
                              float* w_out) {
    return moe_run(e, router_w, E, k, norm, scale, gate, up, down, x, T, y, ids_out, w_out, nullptr);
}

extern "C" int hc_moe_stack_dev(hc_engine* e, size_t n_layers, const float* const* router_w, size_t E, size_t k,
                                int norm, float scale, const hc_weights* const* gate, const hc_weights* const* up,
                                const hc_weights* const* down, float* x, size_t T) {
    return moe_stack(e, n_layers, router_w, E, k, norm, scale, gate, up, down, 0, E, false, x, T);
}

extern "C" int hc_moe_stack_ep_dev(hc_engine* e, size_t n_layers, const float* const* router_w, size_t E, size_t k,
                                   int norm, float scale, const hc_weights* const* gate, const hc_weights* const* up,
                                   const hc_weights* const* down, size_t expert_lo, size_t n_local, float* x,
                                   size_t T) {
    return moe_stack(e, n_layers, router_w, E, k, norm, scale, gate, up, down, expert_lo, n_local, true, x, T);
}

extern "C" int hc_moe_ffn_ep_dev(hc_engine* e, const float* router_w, size_t E, size_t k, int norm, float scale,
                                 const hc_weights* const* gate, const hc_weights* const* up,
                                 const hc_weights* const* down, size_t expert_lo, size_t n_local, const float* x,
                                 size_t T, float* y, int32_t* ids_out, float* w_out) {
    const EpRun ep{expert_lo, n_local};
    return moe_run(e, router_w, E, k, norm, scale, gate, up, down, x, T, y, ids_out, w_out, &ep);
}
