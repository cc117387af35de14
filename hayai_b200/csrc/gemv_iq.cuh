// gemv_iq.cuh -- the IQ2 / IQ3 codebook formats on the tensor-core GEMV (batch 1..4).
//
// Reference semantics: the IQ2 block decoders (crates/hayai-model/src/iq2.rs:504-573, gemv
// :591-626) and the IQ3 ones (crates/hayai-model/src/iq3.rs:147-220, gemv :258-331): a
// 256-element super-block of 32-element groups; each group's elements are codebook grid points
// (8 elements for IQ2, 4 for IQ3) with per-element signs and a 4-bit group scale (IQ2_XS and
// IQ2_S: one per 16 elements).  Every weight is db * g * sign with db the group's scale.
//
// GPU layout (repack.cu): the tile-block image of 16 rows x one super-block is
//   [d of the 16 rows: 32 B][piece (r, t) at 32 + 16 (4r + t): 1024 B][extras]
// where lane t's piece holds its two groups 2t and 2t + 1 (IQ2_XXS / IQ2_XS / IQ3_XXS / IQ3_S:
// raw bytes 2 + 16t ..+16 of the block; IQ2_S: its 8 grid-index bytes, then its 8 sign bytes),
// and the extras hold the rest per row (IQ2_XS: scales; IQ2_S: qh then scales; IQ3_XXS: the
// scale-and-sign words; IQ3_S: sign bytes, qh, scales).  The images are whole multiples of 16
// rows x the block size: no padding.
//
// Compute: lane-distributed like Q4_K (same fragment table): lane t's k-slots are elements
// 64t + 32k + 4wi + j of the block (group 2t + k, wi < 8, j < 4), and B holds lane t's x only
// in its own two columns, so every accumulator is one group's (or half-group's) dot product on
// its own lane; the group scale is applied once per accumulator in f32.  Grid bytes enter the
// A fragment as f16(1024 + g) by one PRMT, minus 1024 (exact), and the element signs are
// XORed into the f16 sign bits: the sign bits of elements (0, 2) land on bits 15 / 31 by one
// multiply of (s & 5) by 0x20008000, those of (1, 3) by (s & 10) * 0x10004000.  The codebooks
// are read through the read-only cache (at most 8 KB each).
#pragma once

#include "gemv_mma_impl.cuh"

#define HC_IQ_QUAL static __device__ const
#include "_gen/iq_tables.h"

namespace hc {

template <int TYPE>
struct FmtIQ {
    static constexpr int kType = TYPE;
    static constexpr int kTile = TYPE == T_IQ2_XXS ? 1056
                                 : TYPE == T_IQ2_XS ? 1184
                                 : TYPE == T_IQ2_S  ? 1312
                                 : TYPE == T_IQ3_XXS ? 1568
                                                     : 1760;
    static constexpr int kD = 0, kP = 32, kX = 1056;
    static constexpr int kBlockElems = 256;
    static constexpr int kMmaPerBlock = 16;
    __device__ static int base(int mi, int t) { return FmtQ4K::base(mi, t); }
    static constexpr bool kNeedSx = false;
    static constexpr bool kLaneShares = true;
    template <int NV>
    __device__ static int tab(int mi, int v, int t) {
        return FmtQ4K::template tab<NV>(mi, v, t);
    }
    static constexpr int kLoOff = FmtQ4K::kLoOff;
    // accumulators per lane: one per group, or per half-group for the 16-element scales
    static constexpr int kAcc = (TYPE == T_IQ2_XS || TYPE == T_IQ2_S) ? 4 : 2;
};

// One row's share of a tile-block image for lane t.
struct IQBlk {
    uint4 p;      // the piece
    uint2 x;      // IQ3_XXS: the two scale-and-sign words; IQ3_S: the two groups' sign words
    uint32_t s;   // IQ2_XS: scale bytes (low 16 bits); IQ2_S: qh (low 16) | scales (high 16);
                  // IQ3_S: qh (low 16) | scale byte (bits 16-23)
    uint32_t d;   // f16 d in the low 16 bits
};

template <int TYPE>
__device__ __forceinline__ void iq_load(IQBlk& b, const uint8_t* tb, int r, int t) {
    using F = FmtIQ<TYPE>;
    b.p = *reinterpret_cast<const uint4*>(tb + F::kP + 16 * (4 * r + t));
    b.d = *reinterpret_cast<const uint16_t*>(tb + F::kD + 2 * r);
    b.x = make_uint2(0u, 0u);
    b.s = 0u;
    if constexpr (TYPE == T_IQ2_XS) {
        b.s = *reinterpret_cast<const uint16_t*>(tb + F::kX + 8 * r + 2 * t);
    } else if constexpr (TYPE == T_IQ2_S) {
        b.s = (uint32_t)*reinterpret_cast<const uint16_t*>(tb + F::kX + 16 * r + 2 * t) |
              ((uint32_t)*reinterpret_cast<const uint16_t*>(tb + F::kX + 16 * r + 8 + 2 * t) << 16);
    } else if constexpr (TYPE == T_IQ3_XXS) {
        b.x = *reinterpret_cast<const uint2*>(tb + F::kX + 32 * r + 8 * t);
    } else if constexpr (TYPE == T_IQ3_S) {
        b.x = *reinterpret_cast<const uint2*>(tb + F::kX + 32 * r + 8 * t);
        b.s = (uint32_t)*reinterpret_cast<const uint16_t*>(tb + F::kX + 512 + 8 * r + 2 * t) |
              ((uint32_t)tb[F::kX + 640 + 4 * r + t] << 16);
    }
}

__device__ __forceinline__ uint32_t iq_ksigns(uint32_t i) {  // iq2.rs:18-27
    i &= 127u;
    return i | ((__popc(i) & 1u) << 7);
}

__device__ __forceinline__ uint32_t byte_of(const uint4& p, int i) {
    const uint32_t w = i < 4 ? p.x : (i < 8 ? p.y : (i < 12 ? p.z : p.w));
    return (w >> (8 * (i & 3))) & 0xFFu;
}

// Grid point l of group k (8 elements for IQ2; for IQ3 the two 4-element points 2l, 2l+1) as
// 8 grid bytes (lo: elements 0-3, hi: 4-7) and the 8 sign bits (bit j: element j negative).
template <int TYPE>
__device__ __forceinline__ void iq_point(const IQBlk& b, int k, int l, uint32_t& lo, uint32_t& hi, uint32_t& s8) {
    if constexpr (TYPE == T_IQ2_XXS) {
        const uint32_t aux0 = k ? b.p.z : b.p.x, aux1 = k ? b.p.w : b.p.y;
        const uint2 g = __ldg(reinterpret_cast<const uint2*>(hc_iq2xxs_grid) + ((aux0 >> (8 * l)) & 0xFFu));
        lo = g.x;
        hi = g.y;
        s8 = iq_ksigns(aux1 >> (7 * l));
    } else if constexpr (TYPE == T_IQ2_XS) {
        const int i = 4 * k + l;  // u16 i of the piece
        const uint32_t w = i < 2 ? b.p.x : (i < 4 ? b.p.y : (i < 6 ? b.p.z : b.p.w));
        const uint32_t q = (w >> (16 * (i & 1))) & 0xFFFFu;
        const uint2 g = __ldg(reinterpret_cast<const uint2*>(hc_iq2xs_grid) + (q & 511u));
        lo = g.x;
        hi = g.y;
        s8 = iq_ksigns(q >> 9);
    } else if constexpr (TYPE == T_IQ2_S) {
        const uint32_t qh = (b.s >> (8 * k)) & 0xFFu;
        const uint32_t idx = byte_of(b.p, 4 * k + l) | (((qh >> (2 * l)) & 3u) << 8);
        const uint2 g = __ldg(reinterpret_cast<const uint2*>(hc_iq2s_grid) + idx);
        lo = g.x;
        hi = g.y;
        s8 = byte_of(b.p, 8 + 4 * k + l);
    } else if constexpr (TYPE == T_IQ3_XXS) {
        const uint32_t aux = k ? b.x.y : b.x.x;
        lo = __ldg(hc_iq3xxs_grid + byte_of(b.p, 8 * k + 2 * l));
        hi = __ldg(hc_iq3xxs_grid + byte_of(b.p, 8 * k + 2 * l + 1));
        s8 = iq_ksigns(aux >> (7 * l));
    } else {  // IQ3_S
        const uint32_t qh = (b.s >> (8 * k)) & 0xFFu;
        const uint32_t i0 = byte_of(b.p, 8 * k + 2 * l) | (((qh >> (2 * l)) & 1u) << 8);
        const uint32_t i1 = byte_of(b.p, 8 * k + 2 * l + 1) | (((qh >> (2 * l + 1)) & 1u) << 8);
        lo = __ldg(hc_iq3s_grid + i0);
        hi = __ldg(hc_iq3s_grid + i1);
        s8 = ((k ? b.x.y : b.x.x) >> (8 * l)) & 0xFFu;
    }
}

// Group scale db of accumulator a (group a / (kAcc / 2), half-group a % 2 for kAcc = 4).
template <int TYPE>
__device__ __forceinline__ float iq_scale(const IQBlk& b, int a) {
    const float d = h2f((uint16_t)b.d);
    if constexpr (TYPE == T_IQ2_XXS) {
        const uint32_t aux1 = a ? b.p.w : b.p.y;
        return d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
    } else if constexpr (TYPE == T_IQ2_XS || TYPE == T_IQ2_S) {
        const int k = a >> 1, h = a & 1;
        const uint32_t sc = TYPE == T_IQ2_XS ? (b.s >> (8 * k)) : (b.s >> (16 + 8 * k));
        return d * (0.5f + (float)((sc >> (4 * h)) & 0xFu)) * 0.25f;
    } else if constexpr (TYPE == T_IQ3_XXS) {
        const uint32_t aux = a ? b.x.y : b.x.x;
        return d * (0.5f + (float)(aux >> 28)) * 0.5f;
    } else {
        const uint32_t sc = (b.s >> (16 + 4 * a)) & 0xFu;
        return d * (1.0f + 2.0f * (float)sc);
    }
}

// 4 grid bytes and their 4 sign bits (at bit `sh` of s8) -> the A registers of elements (0, 2)
// and (1, 3), exact signed integers in f16.
__device__ __forceinline__ void iq_frag(uint32_t g4, uint32_t s8, int sh, uint32_t& a02, uint32_t& a13) {
    constexpr uint32_t k1024 = 0x64006400u;
    a02 = hsub2_u32(prmt(g4, 0x64646464u, 0x4240u), k1024);
    a13 = hsub2_u32(prmt(g4, 0x64646464u, 0x4341u), k1024);
    const uint32_t m02 = ((s8 & (5u << sh)) * (0x20008000u >> sh)) & 0x80008000u;
    const uint32_t m13 = ((s8 & (10u << sh)) * (0x10004000u >> sh)) & 0x80008000u;
    a02 ^= m02;
    a13 ^= m13;
}

// One IQ unit: rows g (A) and g+8 (B) of one tile-block image, lane shares into pA / pB.
template <int TYPE, int NV>
__device__ __forceinline__ void iq_unit(const IQBlk& A, const IQBlk& B, int kb, const LaneCtx<NV>& c,
                                        float (&pA)[1][NV], float (&pB)[1][NV]) {
    constexpr int NA = FmtIQ<TYPE>::kAcc;
    const uint4* xb = reinterpret_cast<const uint4*>(c.xb0 + kb * c.xstride);
    float acc[NA][NV][4];
#pragma unroll
    for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[a][v][i] = 0.f;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        uint32_t ga[2][2], gb[2][2], sa[2], sb[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            iq_point<TYPE>(A, k, l, ga[k][0], ga[k][1], sa[k]);
            iq_point<TYPE>(B, k, l, gb[k][0], gb[k][1], sb[k]);
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int wi = 2 * l + half;
            uint4 f[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) f[v] = xb[(wi * 2 * NV + 2 * v) * 4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                uint32_t a0, a2, b0, b2;
                iq_frag(ga[k][half], sa[k], 4 * half, a0, a2);
                iq_frag(gb[k][half], sb[k], 4 * half, b0, b2);
                const int ai = NA == 4 ? 2 * k + (l >> 1) : k;
#pragma unroll
                for (int v = 0; v < NV; ++v)
                    mma16816(acc[ai][v], a0, b0, a2, b2, k ? f[v].z : f[v].x, k ? f[v].w : f[v].y);
            }
        }
    }
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        const float da = iq_scale<TYPE>(A, a), db = iq_scale<TYPE>(B, a);
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            pA[0][v] += da * (acc[a][v][0] + acc[a][v][1] * kLoScale);
            pB[0][v] += db * (acc[a][v][2] + acc[a][v][3] * kLoScale);
        }
    }
}

// The stage_unit hook of the TMA pipeline for the IQ formats (rows g, g+8 from shared memory).
template <class F, int NV>
__device__ __forceinline__ void iq_stage_unit(const uint8_t* tb, int kbj, const LaneCtx<NV>& ctx,
                                              float (&pA)[1][NV], float (&pB)[1][NV]) {
    IQBlk A, B;
    iq_load<F::kType>(A, tb, ctx.g, ctx.t);
    iq_load<F::kType>(B, tb, ctx.g + 8, ctx.t);
    iq_unit<F::kType, NV>(A, B, kbj, ctx, pA, pB);
}

}  // namespace hc
