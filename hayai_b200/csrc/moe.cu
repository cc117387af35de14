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

#include <vector>

#include "../../include/hayai_cuda.h"
#include "engine.h"
#include "gemv_launch.h"
#include "gemv_mma_impl.cuh"

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
    const float* x = s.x + (size_t)(p / s.x_div) * s.ldx;
    __shared__ float s_red[32];
    const NormArgs nrm{nullptr, 0, 0.f};
    for (int i = threadIdx.x; i < table_entries_per_block<F>(1); i += blockDim.x) zero[i] = make_uint2(0u, 0u);
    build_prologue<F, 1>(xt, sx, x, s.ldx, s.K, 1, nrm, s_red, s.err);
    __syncthreads();
    if (e < 0) return;  // no expert (cannot happen for validated routing)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int WK = s.wk, groups = 8 / WK, grp = warp / WK, wk = warp % WK;
    const int nb = (s.K + F::kBlockElems - 1) / F::kBlockElems;
    const int nbw = (nb + WK - 1) / WK;
    const int kb0 = min(nb, wk * nbw), kb1 = min(nb, kb0 + nbw);
    const int r0 = j * s.rows_per_item, r1 = min(s.M, r0 + s.rows_per_item);
    const int ntiles = (r1 - r0 + 15) / 16;
    const uint8_t* W = s.w[e];
    const uint8_t* W2 = FUSED ? s.w2[e] : nullptr;
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

// y[t][j] = resid + sum_i w[t,i] * D[t*k+i][j], in top-k order (moe_infer.rs:449-455)
__global__ void moe_combine_kernel(const float* __restrict__ D, const float* __restrict__ w, int T, int k, int dm,
                                   float* __restrict__ y) {
    const size_t n = (size_t)T * dm;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / dm), j = (int)(i % dm);
        float acc = 0.0f;
        for (int q = 0; q < k; ++q) acc = __fadd_rn(acc, __fmul_rn(w[t * k + q], D[((size_t)t * k + q) * dm + j]));
        y[i] = acc;
    }
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
#define HC_CUDA(call)                                              \
    do {                                                           \
        cudaError_t _e = (call);                                   \
        if (_e != cudaSuccess) return hc_cuda_error(_e, #call);    \
    } while (0)

extern "C" int hc_router_scores_dev(hc_engine* e, const float* W, size_t E, size_t D, const float* x, size_t T,
                                    float* scores) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!W || !x || !scores || E == 0 || D == 0) return hc_set_error(HC_ERR_INVALID, "router: bad argument");
    if (T == 0) return HC_OK;
    const size_t n = E * T;
    router_exact_kernel<<<(unsigned)((n + 127) / 128), 128, 0, e->stream>>>(W, x, (int)E, (int)D, (int)T, scores);
    HC_CUDA(cudaGetLastError());
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

extern "C" int hc_moe_ffn_dev(hc_engine* e, const float* router_w, size_t E, size_t k, int norm, float scale,
                              const hc_weights* const* gate, const hc_weights* const* up,
                              const hc_weights* const* down, const float* x, size_t T, float* y, int32_t* ids_out,
                              float* w_out) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!router_w || !gate || !up || !down || !x || !y || E == 0 || k == 0 || k > E)
        return hc_set_error(HC_ERR_INVALID, "moe_ffn: bad argument");
    const hc_weights *g0 = gate[0], *u0 = up[0], *d0 = down[0];
    if (!g0 || !u0 || !d0) return hc_set_error(HC_ERR_INVALID, "moe_ffn: null expert weights");
    for (size_t i = 0; i < E; ++i) {
        const hc_weights *g = gate[i], *u = up[i], *d = down[i];
        if (!g || !u || !d || g->type != g0->type || u->type != g0->type || d->type != d0->type || g->m != g0->m ||
            g->n != g0->n || u->m != g0->m || u->n != g0->n || d->m != d0->m || d->n != d0->n)
            return hc_set_error(HC_ERR_INVALID, "moe_ffn: expert %zu differs in type or shape from expert 0", i);
        if (g->device != e->device || u->device != e->device || d->device != e->device)
            return hc_set_error(HC_ERR_INVALID, "moe_ffn: expert %zu lives on another device", i);
    }
    const size_t dm = g0->n, ff = g0->m;
    if (d0->n != ff || d0->m != dm) return hc_set_error(HC_ERR_INVALID, "moe_ffn: down must be d_model x d_ff");
    if (!gemv_mma_supported(g0->type) || !gemv_mma_supported(d0->type))
        return hc_set_error(HC_ERR_UNSUPPORTED, "moe_ffn: expert format %s/%s has no routed kernel",
                            hc_type_label(g0->type), hc_type_label(d0->type));
    if (((uintptr_t)x & 15) || (dm & 3)) return hc_set_error(HC_ERR_INVALID, "moe_ffn: x must be 16-byte aligned");
    if (T == 0) return HC_OK;
    const size_t P = T * k;
    // workspace: scores [T][E] | ids [P] | w [P] | h [P][ff] | D [P][dm]
    const size_t off_ids = T * E * 4, off_w = off_ids + P * 4, off_h = (off_w + P * 4 + 255) / 256 * 256,
                 off_d = off_h + P * ff * 4, total = off_d + P * dm * 4;
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
    rc = expert_table(e, gate, E, &tg);
    if (!rc) rc = expert_table(e, up, E, &tu);
    if (!rc) rc = expert_table(e, down, E, &td);
    if (rc) return rc;

    router_exact_kernel<<<(unsigned)((E * T + 127) / 128), 128, 0, e->stream>>>(router_w, x, (int)E, (int)dm, (int)T,
                                                                                 scores);
    HC_CUDA(cudaGetLastError());
    rc = route_dev(e, scores, nullptr, T, E, k, 0, 0, 0, norm, scale, ids, wts);
    if (rc) return rc;

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
    ce = launch_moe_stage(d0->type, false, s2, (int)P, e->smem_optin, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "moe down launch");

    const size_t n = T * dm;
    moe_combine_kernel<<<(unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, e->stream>>>(
        D, wts, (int)T, (int)k, (int)dm, y);
    HC_CUDA(cudaGetLastError());
    return HC_OK;
}
