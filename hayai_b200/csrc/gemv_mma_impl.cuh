// gemv_mma_impl.cuh -- device building blocks of the tensor-core GEMV, shared by the
// dense kernels (gemv_mma.cu) and the expert-routed kernels (moe.cu).
#pragma once

#include "gemv_mma.cuh"

namespace hc {

constexpr uint32_t kFull = 0xffffffffu;
constexpr float kLoScale = 1.0f / 2048.0f;

// ------------------------------------------------------------------ prologue
// B-fragment table: entry e = ((block * kMmaPerBlock + mi) * 2NV + g) * 4 + t holds
// {pack(x[e0], x[e2]), pack(x[e1], x[e3])} of vector g/2, part g&1 (hi / lo*2^11),
// where e_j = block*kBlockElems + F::base(mi, t) + j.
template <class F, int NV>
__device__ void build_table(uint2* __restrict__ xt, const float* __restrict__ x, int ldx, int K, int nvec,
                            int* err) {
    const int nb = (K + F::kBlockElems - 1) / F::kBlockElems;
    const int total = nb * F::kMmaPerBlock * 2 * NV * 4;
    bool bad = false;
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
        const int t = e & 3;
        const int g = (e >> 2) % (2 * NV);
        const int mall = e / (8 * NV);
        const int kb = mall / F::kMmaPerBlock, mi = mall % F::kMmaPerBlock;
        const int v = g >> 1, part = g & 1;
        const int b = kb * F::kBlockElems + F::base(mi, t);
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (v < nvec && b < K) xv = __ldg(reinterpret_cast<const float4*>(x + (size_t)v * ldx + b));
        float xs[4] = {xv.x, xv.y, xv.z, xv.w};
        __half p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (fabsf(xs[j]) >= 65504.0f && isfinite(xs[j])) bad = true;
            __half hi, lo;
            split_f16(xs[j], hi, lo);
            p[j] = part ? lo : hi;
        }
        xt[e] = make_uint2(h2_as_u32(__halves2half2(p[0], p[2])), h2_as_u32(__halves2half2(p[1], p[3])));
    }
    if (bad && err) atomicOr(err, 1);
}

// Sub-block sums of x (for the Q4_K min term), [NV][K/32].
template <int NV>
__device__ void build_sx(float* __restrict__ sx, const float* __restrict__ x, int ldx, int K, int nvec) {
    const int ns = K / 32;
    for (int i = threadIdx.x; i < NV * ns; i += blockDim.x) {
        const int v = i / ns, j = i % ns;
        float s = 0.f;
        if (v < nvec) {
            const float4* p = reinterpret_cast<const float4*>(x + (size_t)v * ldx + 32 * j);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 a = __ldg(p + q);
                s += (a.x + a.y) + (a.z + a.w);
            }
        }
        sx[i] = s;
    }
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

template <int NV>
__device__ __forceinline__ void q4k_rows(const uint8_t* __restrict__ pA, const uint8_t* __restrict__ pB, int kb0,
                                         int kb1, const uint2* __restrict__ xt, const float* __restrict__ sx, int sxs,
                                         const uint2* __restrict__ lut, int g, int t, float& yA, float& yB) {
    constexpr int kEnt = 16 * 2 * NV * 4;
    const bool has_b = g < 2 * NV;
#pragma unroll 1
    for (int kb = kb0; kb < kb1; ++kb) {
        const uint8_t* bA = pA + kb * 144;
        const uint8_t* bB = pB + kb * 144;
        const uint4 hA = ldg_stream128(bA), hB = ldg_stream128(bB);
        const uint4 qA0 = ldg_stream128(bA + 16 + 32 * t), qA1 = ldg_stream128(bA + 32 + 32 * t);
        const uint4 qB0 = ldg_stream128(bB + 16 + 32 * t), qB1 = ldg_stream128(bB + 32 + 32 * t);
        int scA0, mA0, scA1, mA1, scB0, mB0, scB1, mB1;
        q4k_scales(hA, t, scA0, mA0, scA1, mA1);
        q4k_scales(hB, t, scB0, mB0, scB1, mB1);
        const uint2 loA = lut[scA0], hiA = lut[64 + scA1], loB = lut[scB0], hiB = lut[64 + scB1];
        const uint2* xb = xt + kb * kEnt + g * 4 + t;
        const uint32_t wA[8] = {qA0.x, qA0.y, qA0.z, qA0.w, qA1.x, qA1.y, qA1.z, qA1.w};
        const uint32_t wB[8] = {qB0.x, qB0.y, qB0.z, qB0.w, qB1.x, qB1.y, qB1.z, qB1.w};
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int wi = 0; wi < 8; ++wi) {
            const uint32_t a = wA[wi], b = wB[wi], a8 = a >> 8, b8 = b >> 8;
            const uint2 fl = has_b ? xb[(2 * wi) * (2 * NV * 4)] : make_uint2(0u, 0u);
            const uint2 fh = has_b ? xb[(2 * wi + 1) * (2 * NV * 4)] : make_uint2(0u, 0u);
            mma16816(c, hfma2_u32(lop3_and_or(a, 0x000F000Fu, 0x64006400u), loA.x, loA.y),
                     hfma2_u32(lop3_and_or(b, 0x000F000Fu, 0x64006400u), loB.x, loB.y),
                     hfma2_u32(lop3_and_or(a8, 0x000F000Fu, 0x64006400u), loA.x, loA.y),
                     hfma2_u32(lop3_and_or(b8, 0x000F000Fu, 0x64006400u), loB.x, loB.y), fl.x, fl.y);
            mma16816(c, hfma2_u32(lop3_and_or(a, 0x00F000F0u, 0x64006400u), hiA.x, hiA.y),
                     hfma2_u32(lop3_and_or(b, 0x00F000F0u, 0x64006400u), hiB.x, hiB.y),
                     hfma2_u32(lop3_and_or(a8, 0x00F000F0u, 0x64006400u), hiA.x, hiA.y),
                     hfma2_u32(lop3_and_or(b8, 0x00F000F0u, 0x64006400u), hiB.x, hiB.y), fh.x, fh.y);
        }
        const float2 ddA = __half22float2(u32_as_h2(hA.x));
        const float2 ddB = __half22float2(u32_as_h2(hB.x));
        float mpA = 0.f, mpB = 0.f;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const float s0 = sx[v * sxs + kb * 8 + 2 * t], s1 = sx[v * sxs + kb * 8 + 2 * t + 1];
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
        yA += ddA.x * (c[0] + c[1] * kLoScale) - ddA.y * mpA;
        yB += ddB.x * (c[2] + c[3] * kLoScale) - ddB.y * mpB;
    }
}

// ------------------------------------------------------------------ Q6_K (GPU layout)
// Row: nb blocks of 208 B {ql_perm[4 lanes][8 words] | qh_perm[4 lanes][4 words] | sc[16]},
// then the f16 d plane (nb entries, padded to 16 B).  ql word wq = 4h + 2qq + lh of lane t
// holds original ql bytes 64h + 32qq + 16lh + 4t..+3; qh word wh = 2h + lh holds
// qh bytes 32h + 16lh + 4t..+3 (q6k.rs:26-57 layout).
__device__ __forceinline__ float i8_to_f32(uint32_t word, int byte) {
    const uint32_t sel = 0x8880u | (uint32_t)byte | ((0x8u | (uint32_t)byte) << 4) | ((0x8u | (uint32_t)byte) << 8) |
                         ((0x8u | (uint32_t)byte) << 12);
    const int s = (int)prmt(word, 0u, sel & 0xFFFFu);
    return (float)s;
}

template <int NV>
__device__ __forceinline__ void q6k_rows(const uint8_t* __restrict__ pA, const uint8_t* __restrict__ pB, int kb0,
                                         int kb1, int nb, const uint2* __restrict__ xt, int g, int t, float& yA,
                                         float& yB) {
    constexpr int kEnt = 16 * 2 * NV * 4;
    const bool has_b = g < 2 * NV;
    const uint8_t* dpA = pA + (size_t)nb * 208;
    const uint8_t* dpB = pB + (size_t)nb * 208;
    const uint32_t kOff = 0x64206420u;  // (1056, 1056) in f16: 1024 magic + 32 code offset
#pragma unroll 1
    for (int kb = kb0; kb < kb1; ++kb) {
        const uint8_t* bA = pA + kb * 208;
        const uint8_t* bB = pB + kb * 208;
        const uint4 lA0 = ldg_stream128(bA + 32 * t), lA1 = ldg_stream128(bA + 32 * t + 16);
        const uint4 lB0 = ldg_stream128(bB + 32 * t), lB1 = ldg_stream128(bB + 32 * t + 16);
        const uint4 hA = ldg_stream128(bA + 128 + 16 * t), hB = ldg_stream128(bB + 128 + 16 * t);
        const uint4 sA = ldg_stream128(bA + 192), sB = ldg_stream128(bB + 192);
        const float dA = h2f(ldg_u16(dpA + 2 * kb)), dB = h2f(ldg_u16(dpB + 2 * kb));
        const uint32_t LA[8] = {lA0.x, lA0.y, lA0.z, lA0.w, lA1.x, lA1.y, lA1.z, lA1.w};
        const uint32_t LB[8] = {lB0.x, lB0.y, lB0.z, lB0.w, lB1.x, lB1.y, lB1.z, lB1.w};
        const uint32_t QHA[4] = {hA.x, hA.y, hA.z, hA.w};
        const uint32_t QHB[4] = {hB.x, hB.y, hB.z, hB.w};
        const uint32_t SA[4] = {sA.x, sA.y, sA.z, sA.w};
        const uint32_t SB[4] = {sB.x, sB.y, sB.z, sB.w};
        const uint2* xb = xt + kb * kEnt + g * 4 + t;
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
                    const uint2 f = has_b ? xb[m * (2 * NV * 4)] : make_uint2(0u, 0u);
                    float c[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(c, hsub2_u32(prmt(ua, 0x64646464u, 0x4240u), kOff),
                             hsub2_u32(prmt(ub, 0x64646464u, 0x4240u), kOff),
                             hsub2_u32(prmt(ua, 0x64646464u, 0x4341u), kOff),
                             hsub2_u32(prmt(ub, 0x64646464u, 0x4341u), kOff), f.x, f.y);
                    const int si = 8 * h + 2 * q + lh;  // scale index = element / 16
                    const float sa = dA * i8_to_f32(SA[si >> 2], si & 3);
                    const float sb = dB * i8_to_f32(SB[si >> 2], si & 3);
                    yA += sa * (c[0] + c[1] * kLoScale);
                    yB += sb * (c[2] + c[3] * kLoScale);
                }
            }
        }
    }
}

// ------------------------------------------------------------------ Q8_0 (GPU layout)
// Row: ng groups of 128 B {qs_perm[4 lanes][8 words]} (group = 4 Q8_0 blocks = 128
// elements), then the f16 d plane (4 entries per group, padded to 16 B).  Word w of
// lane t holds codes 16*(w&1) + 4t..+3 of block w/2 of the group.
template <int NV>
__device__ __forceinline__ void q80_rows(const uint8_t* __restrict__ pA, const uint8_t* __restrict__ pB, int kb0,
                                         int kb1, int ng, const uint2* __restrict__ xt, int g, int t, float& yA,
                                         float& yB) {
    constexpr int kEnt = 8 * 2 * NV * 4;
    const bool has_b = g < 2 * NV;
    const uint8_t* dpA = pA + (size_t)ng * 128;
    const uint8_t* dpB = pB + (size_t)ng * 128;
    const uint32_t kOff = 0x64806480u;  // (1152, 1152): 1024 magic + 128 sign flip
#pragma unroll 1
    for (int kg = kb0; kg < kb1; ++kg) {
        const uint4 qA0 = ldg_stream128(pA + kg * 128 + 32 * t), qA1 = ldg_stream128(pA + kg * 128 + 32 * t + 16);
        const uint4 qB0 = ldg_stream128(pB + kg * 128 + 32 * t), qB1 = ldg_stream128(pB + kg * 128 + 32 * t + 16);
        const uint2 dwA = ldg_u2(dpA + kg * 8), dwB = ldg_u2(dpB + kg * 8);
        const uint32_t WA[8] = {qA0.x, qA0.y, qA0.z, qA0.w, qA1.x, qA1.y, qA1.z, qA1.w};
        const uint32_t WB[8] = {qB0.x, qB0.y, qB0.z, qB0.w, qB1.x, qB1.y, qB1.z, qB1.w};
        const float2 dA01 = __half22float2(u32_as_h2(dwA.x)), dA23 = __half22float2(u32_as_h2(dwA.y));
        const float2 dB01 = __half22float2(u32_as_h2(dwB.x)), dB23 = __half22float2(u32_as_h2(dwB.y));
        const float dA[4] = {dA01.x, dA01.y, dA23.x, dA23.y};
        const float dB[4] = {dB01.x, dB01.y, dB23.x, dB23.y};
        const uint2* xb = xt + kg * kEnt + g * 4 + t;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
            float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int w = 2 * blk + half;
                const uint32_t ua = WA[w] ^ 0x80808080u, ub = WB[w] ^ 0x80808080u;
                const uint2 f = has_b ? xb[w * (2 * NV * 4)] : make_uint2(0u, 0u);
                mma16816(c, hsub2_u32(prmt(ua, 0x64646464u, 0x4240u), kOff),
                         hsub2_u32(prmt(ub, 0x64646464u, 0x4240u), kOff),
                         hsub2_u32(prmt(ua, 0x64646464u, 0x4341u), kOff),
                         hsub2_u32(prmt(ub, 0x64646464u, 0x4341u), kOff), f.x, f.y);
            }
            yA += dA[blk] * (c[0] + c[1] * kLoScale);
            yB += dB[blk] * (c[2] + c[3] * kLoScale);
        }
    }
}

template <class F, int NV>
__device__ __forceinline__ void rows_dispatch(const uint8_t* pA, const uint8_t* pB, int kb0, int kb1, int nb,
                                              const uint2* xt, const float* sx, int sxs, const uint2* lut, int g,
                                              int t, float& yA, float& yB) {
    if constexpr (F::kType == T_Q4_K) {
        q4k_rows<NV>(pA, pB, kb0, kb1, xt, sx, sxs, lut, g, t, yA, yB);
    } else if constexpr (F::kType == T_Q6_K) {
        q6k_rows<NV>(pA, pB, kb0, kb1, nb, xt, g, t, yA, yB);
    } else {
        q80_rows<NV>(pA, pB, kb0, kb1, nb, xt, g, t, yA, yB);
    }
}

}  // namespace hc
