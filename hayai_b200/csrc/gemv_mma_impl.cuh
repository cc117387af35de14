// gemv_mma_impl.cuh -- device building blocks of the tensor-core GEMV, shared by the
// dense kernel (gemv_tma.cu) and the expert-routed kernels (moe.cu).
//
//  1. prologue: the activation rows (optionally RMS-normalised) are turned into the
//     B-fragment table in shared memory.  Every thread issues all its float4 loads up
//     front (no dependent load chain), maps each 4-element chunk to its table slot with
//     the format's inverse index, and writes the hi and lo f16 halves.
//  2. per kernel block: a warp takes rows g and g+8 of one tile-block image (from shared
//     memory, or streamed from global memory one block ahead) and dequantises them
//     straight into mma.m16n8k16 A fragments.
#pragma once

#include "gemv_mma.cuh"

namespace hc {

constexpr uint32_t kFull = 0xffffffffu;
constexpr float kLoScale = 1.0f / 2048.0f;

// ------------------------------------------------------------------ inverse maps
// Element offset within a kernel block -> (mma index mi, lane-in-group t) such that
// F::base(mi, t) == offset.  Offsets are multiples of 4.
__device__ __forceinline__ void inv_q4k(int e, int& mi, int& t) {
    t = e >> 6;  // 64t + 4wi + 32part
    const int r = e & 63;
    mi = 2 * ((r & 31) >> 2) + (r >> 5);
}
__device__ __forceinline__ void inv_q6k(int e, int& mi, int& t) {
    const int h = e >> 7, r = e & 127, q = r >> 5, r2 = r & 31, lh = r2 >> 4;
    t = (r2 & 15) >> 2;  // 128h + 32q + 16lh + 4t
    mi = 8 * h + 4 * lh + q;
}
__device__ __forceinline__ void inv_q80(int e, int& mi, int& t) {
    mi = e >> 4;  // 16mi + 4t
    t = (e & 15) >> 2;
}

template <class F>
__device__ __forceinline__ void inv_map(int e, int& mi, int& t) {
    if constexpr (F::kType == T_Q4_K) inv_q4k(e, mi, t);
    else if constexpr (F::kType == T_Q6_K) inv_q6k(e, mi, t);
    else inv_q80(e, mi, t);
}

// ------------------------------------------------------------------ prologue
// Optional RMSNorm of the activation rows, applied while the fragment table is built:
// xn[i] = (x[i] * inv[v]) * w[i] for i < len (rms_norm, crates/hayai-cpu/src/attention.rs:142-147).
struct NormArgs {
    const float* w;  // [len] norm weight, nullptr = no normalization
    int len;         // normalized length (<= K, multiple of 4; elements beyond it are zero padding)
    float eps;
};

// Sum over the first nthr threads of the CTA (whole warps), synchronised on named barrier
// `bar` (bar 0 with nthr == blockDim.x is __syncthreads).
__device__ __forceinline__ float block_sum(float s, float* scratch, int nthr, int bar) {
    s = warp_sum(s);
    named_bar_sync(bar, nthr);  // scratch may still be read by a previous call
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = s;
    named_bar_sync(bar, nthr);
    float t = 0.f;
    const int nw = nthr >> 5;
    for (int i = 0; i < nw; ++i) t += scratch[i];
    return t;
}

// Builds the B-fragment table (entry e = ((block * kMmaPerBlock + mi) * 2NV + g) * 4 + t holds
// {pack(x[e0], x[e2]), pack(x[e1], x[e3])} of vector g/2, part g&1 (hi / lo*2^11), with
// e_j = block*kBlockElems + F::base(mi, t) + j) and, for Q4_K, the 32-element sub-block sums.
// Run by threads [0, nthr) of the CTA (all of it by default); `bar` is the named barrier they
// synchronise on.
template <class F, int NV>
__device__ void build_prologue(uint2* __restrict__ xt, float* __restrict__ sx, const float* __restrict__ x, int ldx,
                               int K, int nvec, const NormArgs& nrm, float* scratch, int* err, int nthr, int bar) {
    const int nb = (K + F::kBlockElems - 1) / F::kBlockElems;
    const int nchunk = K >> 2;                         // real float4 chunks
    const int ntab = (nb * F::kBlockElems) >> 2;       // chunks covered by the table (zero padded)
    const int rounds = (ntab + nthr - 1) / nthr;
    bool bad = false;
    for (int v = 0; v < NV; ++v) {
        const float* xv = x + (size_t)v * ldx;
        const bool live = v < nvec;
        float inv = 1.0f;
        if (nrm.w) {
            float s = 0.f;
            if (live) {
                const int nc = nrm.len >> 2;
#pragma unroll 4
                for (int c = threadIdx.x; c < nc; c += nthr) {
                    const float4 a = __ldg(reinterpret_cast<const float4*>(xv) + c);
                    s += (a.x * a.x + a.y * a.y) + (a.z * a.z + a.w * a.w);
                }
            }
            const float tot = block_sum(s, scratch, nthr, bar);
            inv = 1.0f / sqrtf(tot / (float)nrm.len + nrm.eps);
        }
#pragma unroll 4
        for (int r = 0; r < rounds; ++r) {
            const int c = threadIdx.x + r * nthr;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            if (live && c < nchunk) {
                a = __ldg(reinterpret_cast<const float4*>(xv) + c);
                if (nrm.w) {
                    if (4 * c < nrm.len) {
                        const float4 w = __ldg(reinterpret_cast<const float4*>(nrm.w) + c);
                        a.x = a.x * inv * w.x;
                        a.y = a.y * inv * w.y;
                        a.z = a.z * inv * w.z;
                        a.w = a.w * inv * w.w;
                    } else {
                        a = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
            }
            if (c < ntab) {
                const float xs[4] = {a.x, a.y, a.z, a.w};
                __half hi[4], lo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (fabsf(xs[j]) >= 65504.0f && isfinite(xs[j])) bad = true;
                    split_f16(xs[j], hi[j], lo[j]);
                }
                const int e = 4 * c, kb = e / F::kBlockElems;
                int mi, t;
                inv_map<F>(e - kb * F::kBlockElems, mi, t);
                const int base = ((kb * F::kMmaPerBlock + mi) * 2 * NV + 2 * v) * 4 + t;
                xt[base] = make_uint2(h2_as_u32(__halves2half2(hi[0], hi[2])), h2_as_u32(__halves2half2(hi[1], hi[3])));
                xt[base + 4] =
                    make_uint2(h2_as_u32(__halves2half2(lo[0], lo[2])), h2_as_u32(__halves2half2(lo[1], lo[3])));
            }
            if constexpr (F::kNeedSx) {
                // 8 consecutive chunks (= consecutive lanes) form one 32-element sub-block
                float s = (a.x + a.y) + (a.z + a.w);
                s += __shfl_xor_sync(kFull, s, 1);
                s += __shfl_xor_sync(kFull, s, 2);
                s += __shfl_xor_sync(kFull, s, 4);
                if ((threadIdx.x & 7) == 0 && c < ntab) sx[v * (ntab >> 3) + (c >> 3)] = s;
            }
        }
    }
    if (bad && err) atomicOr(err, 1);
}

template <class F, int NV>
__device__ void build_prologue(uint2* __restrict__ xt, float* __restrict__ sx, const float* __restrict__ x, int ldx,
                               int K, int nvec, const NormArgs& nrm, float* scratch, int* err) {
    build_prologue<F, NV>(xt, sx, x, ldx, K, nvec, nrm, scratch, err, (int)blockDim.x, 0);
}

// Q4_K scale LUT: [sc] -> {mul (sc,sc), add (-1024 sc)} for low nibbles (value 1024+n),
// [64+sc] -> {mul (sc/16), add (-64 sc)} for high nibbles (value 1024+16n).  All exact in f16.
__device__ inline void build_q4k_lut(uint2* lut) {
    for (int i = threadIdx.x; i < 64; i += blockDim.x) {
        const float sc = (float)i;
        lut[i] = make_uint2(pack_h2(sc, sc), pack_h2(-1024.f * sc, -1024.f * sc));
        lut[64 + i] = make_uint2(pack_h2(sc * 0.0625f, sc * 0.0625f), pack_h2(-64.f * sc, -64.f * sc));
    }
}

// Per-lane context of the main loop.
template <int NV>
struct LaneCtx {
    const uint2* xt;   // table + g*4 + t
    const float* sx;   // Q4_K sub-block sums
    const uint2* lut;  // Q4_K scale LUT
    int sxs;           // Q4_K: K/32
    int nb;            // kernel blocks per row (Q6_K/Q8_0: d plane offset)
    int g, t;
    bool has_b;
};

// ------------------------------------------------------------------ Q4_K
// 6-bit (scale, min) pairs of sub-blocks 2t and 2t+1 (get_scale_min_k4, q4k.rs:34-43),
// from the 12 scale bytes held in h.y, h.z, h.w.
__device__ __forceinline__ void q4k_scales(const uint4& h, int t, int& sc0, int& m0, int& sc1, int& m1) {
    const int sh = 16 * (t & 1);
    const uint32_t Y = h.y >> sh, Z = h.z >> sh, W = h.w >> sh;
    if (t < 2) {
        sc0 = Y & 63;
        m0 = Z & 63;
        sc1 = (Y >> 8) & 63;
        m1 = (Z >> 8) & 63;
    } else {
        sc0 = (W & 0xF) | ((Y >> 2) & 0x30);
        m0 = ((W >> 4) & 0xF) | ((Z >> 2) & 0x30);
        sc1 = ((W >> 8) & 0xF) | ((Y >> 10) & 0x30);
        m1 = ((W >> 12) & 0xF) | ((Z >> 10) & 0x30);
    }
}

struct Q4KBlk {
    uint4 h, q0, q1;
};

// Contribution of one super-block to rows g (dA) and g+8 (dB), for vector t (lanes t < NV).
template <int NV>
__device__ __forceinline__ void q4k_block(const Q4KBlk& A, const Q4KBlk& B, int kb, const LaneCtx<NV>& c,
                                          float& dA, float& dB) {
    constexpr int kEnt = 16 * 2 * NV * 4;
    const int t = c.t;
    int scA0, mA0, scA1, mA1, scB0, mB0, scB1, mB1;
    q4k_scales(A.h, t, scA0, mA0, scA1, mA1);
    q4k_scales(B.h, t, scB0, mB0, scB1, mB1);
    const uint2 loA = c.lut[scA0], hiA = c.lut[64 + scA1], loB = c.lut[scB0], hiB = c.lut[64 + scB1];
    const uint2* xb = c.xt + kb * kEnt;
    const uint32_t wA[8] = {A.q0.x, A.q0.y, A.q0.z, A.q0.w, A.q1.x, A.q1.y, A.q1.z, A.q1.w};
    const uint32_t wB[8] = {B.q0.x, B.q0.y, B.q0.z, B.q0.w, B.q1.x, B.q1.y, B.q1.z, B.q1.w};
    // two accumulator chains (low / high nibbles) halve the dependent MMA latency
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int wi = 0; wi < 8; ++wi) {
        const uint32_t a = wA[wi], b = wB[wi], a8 = a >> 8, b8 = b >> 8;
        const uint2 fl = c.has_b ? xb[(2 * wi) * (2 * NV * 4)] : make_uint2(0u, 0u);
        const uint2 fh = c.has_b ? xb[(2 * wi + 1) * (2 * NV * 4)] : make_uint2(0u, 0u);
        mma16816(acc, hfma2_u32(lop3_and_or(a, 0x000F000Fu, 0x64006400u), loA.x, loA.y),
                 hfma2_u32(lop3_and_or(b, 0x000F000Fu, 0x64006400u), loB.x, loB.y),
                 hfma2_u32(lop3_and_or(a8, 0x000F000Fu, 0x64006400u), loA.x, loA.y),
                 hfma2_u32(lop3_and_or(b8, 0x000F000Fu, 0x64006400u), loB.x, loB.y), fl.x, fl.y);
        mma16816(acc2, hfma2_u32(lop3_and_or(a, 0x00F000F0u, 0x64006400u), hiA.x, hiA.y),
                 hfma2_u32(lop3_and_or(b, 0x00F000F0u, 0x64006400u), hiB.x, hiB.y),
                 hfma2_u32(lop3_and_or(a8, 0x00F000F0u, 0x64006400u), hiA.x, hiA.y),
                 hfma2_u32(lop3_and_or(b8, 0x00F000F0u, 0x64006400u), hiB.x, hiB.y), fh.x, fh.y);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += acc2[i];
    const float2 ddA = __half22float2(u32_as_h2(A.h.x));
    const float2 ddB = __half22float2(u32_as_h2(B.h.x));
    float mpA = 0.f, mpB = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        const float s0 = c.sx[v * c.sxs + kb * 8 + 2 * t], s1 = c.sx[v * c.sxs + kb * 8 + 2 * t + 1];
        float pa = (float)mA0 * s0 + (float)mA1 * s1;
        float pb = (float)mB0 * s0 + (float)mB1 * s1;
        pa += __shfl_xor_sync(kFull, pa, 1);
        pb += __shfl_xor_sync(kFull, pb, 1);
        pa += __shfl_xor_sync(kFull, pa, 2);
        pb += __shfl_xor_sync(kFull, pb, 2);
        if (t == v) {
            mpA = pa;
            mpB = pb;
        }
    }
    dA = ddA.x * (acc[0] + acc[1] * kLoScale) - ddA.y * mpA;
    dB = ddB.x * (acc[2] + acc[3] * kLoScale) - ddB.y * mpB;
}

// Q4_K, scale-per-lane variant.  Lane t's codes are chunk t of the super-block: the low
// nibbles are sub-block 2t, the high nibbles sub-block 2t+1.  B holds lane t's x only in
// columns 2t (hi part) and 2t+1 (lo part), so in every MMA lane t's k-slots meet only its
// own columns and the accumulator comes back per sub-block, already distributed over the
// lanes: C[row][2t] = sum over sub-block (2t+G) of A * x_hi.  Codes enter as
// f16(1 + n/64) (magic 0x3C00, nibble at bits 4-7: one LOP3 per two codes), so
//     sum n*x = 64 * (C - Sx_j)
// and the 6-bit scale, d, dmin and the min term are applied once per sub-block per lane in
// f32.  pA/pB receive lane t's share of rows g / g+8 (summed over t at the end of a tile).
template <int NV, int NMAT>
__device__ __forceinline__ void q4k_unit_dist(const Q4KBlk (&A)[NMAT], const Q4KBlk (&B)[NMAT], int kb,
                                              const LaneCtx<NV>& c, float (&pA)[NMAT][NV], float (&pB)[NMAT][NV]) {
    constexpr int kEnt = 16 * 2 * NV * 4;  // table entries of one super-block
    const int t = c.t, g = c.g;
    const bool mine = (g >> 1) == t;
    // entry ((mma * 2NV + 2v + part) * 4 + t); c.xt points at g*4 + t, rebase to part*4 + t
    const uint2* xb = c.xt - g * 4 + (g & 1) * 4 + kb * kEnt;
    float acc[NMAT][NV][2][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[m][v][0][i] = acc[m][v][1][i] = 0.f;
#pragma unroll
    for (int wi = 0; wi < 8; ++wi) {
        uint2 blo[NV], bhi[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            blo[v] = mine ? xb[((2 * wi) * 2 * NV + 2 * v) * 4] : make_uint2(0u, 0u);
            bhi[v] = mine ? xb[((2 * wi + 1) * 2 * NV + 2 * v) * 4] : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            const uint32_t qa[8] = {A[m].q0.x, A[m].q0.y, A[m].q0.z, A[m].q0.w, A[m].q1.x, A[m].q1.y, A[m].q1.z, A[m].q1.w};
            const uint32_t qb[8] = {B[m].q0.x, B[m].q0.y, B[m].q0.z, B[m].q0.w, B[m].q1.x, B[m].q1.y, B[m].q1.z, B[m].q1.w};
            const uint32_t a = qa[wi], b = qb[wi];
            const uint32_t lo02a = lop3_and_or(a << 4, 0x00F000F0u, 0x3C003C00u);
            const uint32_t lo13a = lop3_and_or(a >> 4, 0x00F000F0u, 0x3C003C00u);
            const uint32_t hi02a = lop3_and_or(a, 0x00F000F0u, 0x3C003C00u);
            const uint32_t hi13a = lop3_and_or(a >> 8, 0x00F000F0u, 0x3C003C00u);
            const uint32_t lo02b = lop3_and_or(b << 4, 0x00F000F0u, 0x3C003C00u);
            const uint32_t lo13b = lop3_and_or(b >> 4, 0x00F000F0u, 0x3C003C00u);
            const uint32_t hi02b = lop3_and_or(b, 0x00F000F0u, 0x3C003C00u);
            const uint32_t hi13b = lop3_and_or(b >> 8, 0x00F000F0u, 0x3C003C00u);
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                mma16816(acc[m][v][0], lo02a, lo02b, lo13a, lo13b, blo[v].x, blo[v].y);
                mma16816(acc[m][v][1], hi02a, hi02b, hi13a, hi13b, bhi[v].x, bhi[v].y);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        int scA0, mA0, scA1, mA1, scB0, mB0, scB1, mB1;
        q4k_scales(A[m].h, t, scA0, mA0, scA1, mA1);
        q4k_scales(B[m].h, t, scB0, mB0, scB1, mB1);
        const float2 ddA = __half22float2(u32_as_h2(A[m].h.x));  // (d, dmin)
        const float2 ddB = __half22float2(u32_as_h2(B[m].h.x));
        const float cA0 = 64.f * ddA.x * (float)scA0, cA1 = 64.f * ddA.x * (float)scA1;
        const float cB0 = 64.f * ddB.x * (float)scB0, cB1 = 64.f * ddB.x * (float)scB1;
        const float kA0 = cA0 + ddA.y * (float)mA0, kA1 = cA1 + ddA.y * (float)mA1;
        const float kB0 = cB0 + ddB.y * (float)mB0, kB1 = cB1 + ddB.y * (float)mB1;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const float s0 = c.sx[v * c.sxs + kb * 8 + 2 * t], s1 = c.sx[v * c.sxs + kb * 8 + 2 * t + 1];
            const float* a0 = acc[m][v][0];
            const float* a1 = acc[m][v][1];
            pA[m][v] += cA0 * (a0[0] + a0[1] * kLoScale) - s0 * kA0 + cA1 * (a1[0] + a1[1] * kLoScale) - s1 * kA1;
            pB[m][v] += cB0 * (a0[2] + a0[3] * kLoScale) - s0 * kB0 + cB1 * (a1[2] + a1[3] * kLoScale) - s1 * kB1;
        }
    }
}

// ------------------------------------------------------------------ Q6_K (GPU layout)
// Row: nb blocks of 208 B {ql_perm[4 lanes][8 words] | qh_perm[4 lanes][4 words] | sc[16]},
// then the f16 d plane (nb entries, padded to 16 B).  ql word wq = 4h + 2qq + lh of lane t
// holds original ql bytes 64h + 32qq + 16lh + 4t..+3; qh word wh = 2h + lh holds
// qh bytes 32h + 16lh + 4t..+3 (q6k.rs:26-57 layout).
__device__ __forceinline__ float i8_to_f32(uint32_t word, int byte) {
    const uint32_t b = (uint32_t)byte;
    const uint32_t sel = b | ((0x8u | b) << 4) | ((0x8u | b) << 8) | ((0x8u | b) << 12);
    return (float)(int)prmt(word, 0u, sel);
}

struct Q6KBlk {
    uint4 l0, l1, qh, sc;
    uint16_t d;
};

template <int NV>
__device__ __forceinline__ void q6k_block(const Q6KBlk& A, const Q6KBlk& B, int kb, const LaneCtx<NV>& c,
                                          float& dA, float& dB) {
    constexpr int kEnt = 16 * 2 * NV * 4;
    const uint32_t kOff = 0x64206420u;  // (1056, 1056) in f16: 1024 magic + 32 code offset
    const float fdA = h2f(A.d), fdB = h2f(B.d);
    const uint32_t LA[8] = {A.l0.x, A.l0.y, A.l0.z, A.l0.w, A.l1.x, A.l1.y, A.l1.z, A.l1.w};
    const uint32_t LB[8] = {B.l0.x, B.l0.y, B.l0.z, B.l0.w, B.l1.x, B.l1.y, B.l1.z, B.l1.w};
    const uint32_t QHA[4] = {A.qh.x, A.qh.y, A.qh.z, A.qh.w};
    const uint32_t QHB[4] = {B.qh.x, B.qh.y, B.qh.z, B.qh.w};
    const uint32_t SA[4] = {A.sc.x, A.sc.y, A.sc.z, A.sc.w};
    const uint32_t SB[4] = {B.sc.x, B.sc.y, B.sc.z, B.sc.w};
    const uint2* xb = c.xt + kb * kEnt;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            const uint32_t QA = QHA[2 * h + lh], QB = QHB[2 * h + lh];
            const uint32_t qa[4] = {(QA << 4) & 0x30303030u, (QA << 2) & 0x30303030u, QA & 0x30303030u,
                                    (QA >> 2) & 0x30303030u};
            const uint32_t qb[4] = {(QB << 4) & 0x30303030u, (QB << 2) & 0x30303030u, QB & 0x30303030u,
                                    (QB >> 2) & 0x30303030u};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int qq = q & 1;
                const uint32_t la = LA[4 * h + 2 * qq + lh], lb = LB[4 * h + 2 * qq + lh];
                const uint32_t ua = lop3_and_or(q < 2 ? la : (la >> 4), 0x0F0F0F0Fu, qa[q]);
                const uint32_t ub = lop3_and_or(q < 2 ? lb : (lb >> 4), 0x0F0F0F0Fu, qb[q]);
                const int m = 8 * h + 4 * lh + q;
                const uint2 f = c.has_b ? xb[m * (2 * NV * 4)] : make_uint2(0u, 0u);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(acc, hsub2_u32(prmt(ua, 0x64646464u, 0x4240u), kOff),
                         hsub2_u32(prmt(ub, 0x64646464u, 0x4240u), kOff),
                         hsub2_u32(prmt(ua, 0x64646464u, 0x4341u), kOff),
                         hsub2_u32(prmt(ub, 0x64646464u, 0x4341u), kOff), f.x, f.y);
                const int si = 8 * h + 2 * q + lh;  // scale index = element / 16
                sumA += i8_to_f32(SA[si >> 2], si & 3) * (acc[0] + acc[1] * kLoScale);
                sumB += i8_to_f32(SB[si >> 2], si & 3) * (acc[2] + acc[3] * kLoScale);
            }
        }
    }
    dA = fdA * sumA;
    dB = fdB * sumB;
}

// ------------------------------------------------------------------ Q8_0 (GPU layout)
// Row: ng groups of 128 B {qs_perm[4 lanes][8 words]} (group = 4 Q8_0 blocks = 128
// elements), then the f16 d plane (4 entries per group, padded to 16 B).  Word w of
// lane t holds codes 16*(w&1) + 4t..+3 of block w/2 of the group.
struct Q80Blk {
    uint4 q0, q1;
    uint2 d;
};

template <int NV>
__device__ __forceinline__ void q80_block(const Q80Blk& A, const Q80Blk& B, int kg, const LaneCtx<NV>& c, float& dA,
                                          float& dB) {
    constexpr int kEnt = 8 * 2 * NV * 4;
    const uint32_t kOff = 0x64806480u;  // (1152, 1152): 1024 magic + 128 sign flip
    const uint32_t WA[8] = {A.q0.x, A.q0.y, A.q0.z, A.q0.w, A.q1.x, A.q1.y, A.q1.z, A.q1.w};
    const uint32_t WB[8] = {B.q0.x, B.q0.y, B.q0.z, B.q0.w, B.q1.x, B.q1.y, B.q1.z, B.q1.w};
    const float2 dA01 = __half22float2(u32_as_h2(A.d.x)), dA23 = __half22float2(u32_as_h2(A.d.y));
    const float2 dB01 = __half22float2(u32_as_h2(B.d.x)), dB23 = __half22float2(u32_as_h2(B.d.y));
    const float fa[4] = {dA01.x, dA01.y, dA23.x, dA23.y};
    const float fb[4] = {dB01.x, dB01.y, dB23.x, dB23.y};
    const uint2* xb = c.xt + kg * kEnt;
    float sA = 0.f, sB = 0.f;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int w = 2 * blk + half;
            const uint32_t ua = WA[w] ^ 0x80808080u, ub = WB[w] ^ 0x80808080u;
            const uint2 f = c.has_b ? xb[w * (2 * NV * 4)] : make_uint2(0u, 0u);
            mma16816(acc, hsub2_u32(prmt(ua, 0x64646464u, 0x4240u), kOff),
                     hsub2_u32(prmt(ub, 0x64646464u, 0x4240u), kOff),
                     hsub2_u32(prmt(ua, 0x64646464u, 0x4341u), kOff),
                     hsub2_u32(prmt(ub, 0x64646464u, 0x4341u), kOff), f.x, f.y);
        }
        sA += fa[blk] * (acc[0] + acc[1] * kLoScale);
        sB += fb[blk] * (acc[2] + acc[3] * kLoScale);
    }
    dA = sA;
    dB = sB;
}

// ------------------------------------------------------------------ tile streaming
template <class F>
struct BlkOf;
template <>
struct BlkOf<FmtQ4K> {
    using T = Q4KBlk;
};
template <>
struct BlkOf<FmtQ6K> {
    using T = Q6KBlk;
};
template <>
struct BlkOf<FmtQ80> {
    using T = Q80Blk;
};

template <bool kShared>
__device__ __forceinline__ uint4 ld_piece(const uint8_t* p) {
    if constexpr (kShared) return *reinterpret_cast<const uint4*>(p);
    else return ldg_stream128(p);
}

// Rows g (A) and g+8 (B) of one tile-block image (see repack.cu for the layout), from
// shared memory (kShared) or streamed from global memory.
template <class F, bool kShared>
__device__ __forceinline__ void tile_load(typename BlkOf<F>::T& A, typename BlkOf<F>::T& B, const uint8_t* tb, int g,
                                          int t) {
    const int pa = 16 * (4 * g + t), pb = pa + 512;
    if constexpr (F::kType == T_Q4_K) {
        A.h = ld_piece<kShared>(tb + F::kHdr + 16 * g);
        B.h = ld_piece<kShared>(tb + F::kHdr + 16 * (g + 8));
        A.q0 = ld_piece<kShared>(tb + F::kQ0 + pa);
        B.q0 = ld_piece<kShared>(tb + F::kQ0 + pb);
        A.q1 = ld_piece<kShared>(tb + F::kQ1 + pa);
        B.q1 = ld_piece<kShared>(tb + F::kQ1 + pb);
    } else if constexpr (F::kType == T_Q6_K) {
        A.l0 = ld_piece<kShared>(tb + F::kL0 + pa);
        B.l0 = ld_piece<kShared>(tb + F::kL0 + pb);
        A.l1 = ld_piece<kShared>(tb + F::kL1 + pa);
        B.l1 = ld_piece<kShared>(tb + F::kL1 + pb);
        A.qh = ld_piece<kShared>(tb + F::kQh + pa);
        B.qh = ld_piece<kShared>(tb + F::kQh + pb);
        A.sc = ld_piece<kShared>(tb + F::kSc + 16 * g);
        B.sc = ld_piece<kShared>(tb + F::kSc + 16 * (g + 8));
        if constexpr (kShared) {
            A.d = *reinterpret_cast<const uint16_t*>(tb + F::kD + 2 * g);
            B.d = *reinterpret_cast<const uint16_t*>(tb + F::kD + 2 * (g + 8));
        } else {
            A.d = ldg_u16(tb + F::kD + 2 * g);
            B.d = ldg_u16(tb + F::kD + 2 * (g + 8));
        }
    } else {
        A.q0 = ld_piece<kShared>(tb + F::kQ0 + pa);
        B.q0 = ld_piece<kShared>(tb + F::kQ0 + pb);
        A.q1 = ld_piece<kShared>(tb + F::kQ1 + pa);
        B.q1 = ld_piece<kShared>(tb + F::kQ1 + pb);
        if constexpr (kShared) {
            A.d = *reinterpret_cast<const uint2*>(tb + F::kD + 8 * g);
            B.d = *reinterpret_cast<const uint2*>(tb + F::kD + 8 * (g + 8));
        } else {
            A.d = ldg_u2(tb + F::kD + 8 * g);
            B.d = ldg_u2(tb + F::kD + 8 * (g + 8));
        }
    }
}

template <class F, int NV>
__device__ __forceinline__ void blk_compute(const typename BlkOf<F>::T& A, const typename BlkOf<F>::T& B, int kb,
                                            const LaneCtx<NV>& c, float& dA, float& dB) {
    if constexpr (F::kType == T_Q4_K) q4k_block<NV>(A, B, kb, c, dA, dB);
    else if constexpr (F::kType == T_Q6_K) q6k_block<NV>(A, B, kb, c, dA, dB);
    else q80_block<NV>(A, B, kb, c, dA, dB);
}

// Streams blocks [kb0, kb1) of one 16-row tile of NMAT matrices (tile images at tb[m])
// through the tensor cores, one block ahead: yA[m] / yB[m] accumulate the outputs of rows
// g / g+8 for vector t.
template <class F, int NV, int NMAT>
__device__ __forceinline__ void stream_tile(const uint8_t* const (&tb)[NMAT], int kb0, int kb1, const LaneCtx<NV>& c,
                                            float (&yA)[NMAT], float (&yB)[NMAT]) {
    using B = typename BlkOf<F>::T;
    const int nk = kb1 - kb0;
    const int total = NMAT * nk;
    if (total <= 0) return;
    B curA, curB, nxtA, nxtB;
    tile_load<F, false>(curA, curB, tb[0] + (size_t)kb0 * F::kTile, c.g, c.t);
#pragma unroll 1
    for (int i = 0; i < total; ++i) {
        const int m = NMAT == 1 ? 0 : i / nk;
        const int kb = kb0 + (i - m * nk);
        if (i + 1 < total) {
            const int m1 = NMAT == 1 ? 0 : (i + 1) / nk;
            const int kbn = kb0 + (i + 1 - m1 * nk);
            tile_load<F, false>(nxtA, nxtB, tb[m1] + (size_t)kbn * F::kTile, c.g, c.t);
        }
        float dA, dB;
        blk_compute<F, NV>(curA, curB, kb, c, dA, dB);
        if (NMAT == 1 || m == 0) {
            yA[0] += dA;
            yB[0] += dB;
        } else {
            yA[NMAT - 1] += dA;
            yB[NMAT - 1] += dB;
        }
        curA = nxtA;
        curB = nxtB;
    }
}

}  // namespace hc
