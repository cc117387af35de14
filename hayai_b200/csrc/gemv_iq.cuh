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
// its own lane; the group scale is applied once per accumulator in f32.  Grid values enter the
// A fragment as exact f16 (from the LUT below), and the element signs are XORed into the f16
// sign bits.
//
// Shared-memory LUTs.  Each CTA expands its format's codebook once, at kernel start, into a
// shared-memory table of ready A-fragment registers: per grid point the f16 pairs (e0, e2),
// (e1, e3) (and (e4, e6), (e5, e7) for the 8-element IQ2 points) of its exact small-integer
// values, 16 B per IQ2 point, 8 B per IQ3 point (IQ2_XXS 4 KB, IQ2_XS 8 KB, IQ2_S 16 KB,
// IQ3_XXS 2 KB, IQ3_S 4 KB).  A point then costs one shared-memory load instead of a gather
// through L1 plus the byte-to-f16 conversion.  The 8 sign bits s of a point (bit j: element j)
// become the f16 sign masks of its four registers by one multiply each: s * 0x20008000 puts
// s0 on bit 15 and s2 on bit 31 (the two shifted copies of s do not overlap, so no carries),
// s * 0x10004000 puts s1 / s3 there, s * 0x02000800 s4 / s6 and s * 0x01000400 s5 / s7.
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

// Bytes of format TYPE's shared-memory LUT (0 for the other formats).
__host__ __device__ constexpr int iq_lut_bytes(int type) {
    return type == T_IQ2_XXS ? 256 * 16
           : type == T_IQ2_XS ? 512 * 16
           : type == T_IQ2_S  ? 1024 * 16
           : type == T_IQ3_XXS ? 256 * 8
           : type == T_IQ3_S   ? 512 * 8
                               : 0;
}

// The f16 sign masks of the four registers of an 8-element point with sign bits s8 (a table of
// these masks in shared memory, one 16-byte load per point, measured 35-45 % slower: the loads
// compete with the grid lookups for shared-memory bandwidth).
__device__ __forceinline__ uint4 iq_sign_masks(uint32_t s8) {
    return make_uint4((s8 * 0x20008000u) & 0x80008000u, (s8 * 0x10004000u) & 0x80008000u,
                      (s8 * 0x02000800u) & 0x80008000u, (s8 * 0x01000400u) & 0x80008000u);
}

// 4 grid bytes -> the f16 pairs (e0, e2), (e1, e3) of their values: f16(1024 + g) by one PRMT
// under the exponent byte 0x64, minus 1024 (exact).
__device__ __forceinline__ uint2 iq_f16_pairs(uint32_t g4) {
    constexpr uint32_t k1024 = 0x64006400u;
    return make_uint2(hsub2_u32(prmt(g4, 0x64646464u, 0x4240u), k1024),
                      hsub2_u32(prmt(g4, 0x64646464u, 0x4341u), k1024));
}

// Expand the codebook of TYPE into the shared-memory LUT (threads [0, nthr) of the CTA; the
// caller synchronises before the first use).
template <int TYPE>
__device__ __forceinline__ void iq_fill_lut(uint8_t* lut, int tid, int nthr) {
    if constexpr (TYPE == T_IQ3_XXS || TYPE == T_IQ3_S) {
        const uint32_t* grid = TYPE == T_IQ3_XXS ? hc_iq3xxs_grid : hc_iq3s_grid;
        constexpr int n = TYPE == T_IQ3_XXS ? 256 : 512;
        for (int i = tid; i < n; i += nthr) reinterpret_cast<uint2*>(lut)[i] = iq_f16_pairs(grid[i]);
    } else {
        const uint64_t* grid = TYPE == T_IQ2_XXS ? hc_iq2xxs_grid : TYPE == T_IQ2_XS ? hc_iq2xs_grid : hc_iq2s_grid;
        constexpr int n = TYPE == T_IQ2_XXS ? 256 : TYPE == T_IQ2_XS ? 512 : 1024;
        for (int i = tid; i < n; i += nthr) {
            const uint2 lo = iq_f16_pairs((uint32_t)grid[i]), hi = iq_f16_pairs((uint32_t)(grid[i] >> 32));
            reinterpret_cast<uint4*>(lut)[i] = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
    }
}

// Point l of group k (8 elements: for IQ3 the two 4-element points 2l, 2l+1) as its four
// A-fragment registers (e0, e2), (e1, e3), (e4, e6), (e5, e7) from the LUT, signs applied.
template <int TYPE>
__device__ __forceinline__ void iq_point(const IQBlk& b, const uint8_t* lut, int k, int l, uint4& f) {
    uint32_t s8;  // sign byte, or the 7-bit sign index of the ksigns formats
    const uint4* lut4 = reinterpret_cast<const uint4*>(lut);
    const uint2* lut2 = reinterpret_cast<const uint2*>(lut);
    if constexpr (TYPE == T_IQ2_XXS) {
        const uint32_t aux0 = k ? b.p.z : b.p.x, aux1 = k ? b.p.w : b.p.y;
        f = lut4[(aux0 >> (8 * l)) & 0xFFu];
        s8 = (aux1 >> (7 * l)) & 127u;
    } else if constexpr (TYPE == T_IQ2_XS) {
        const int i = 4 * k + l;  // u16 i of the piece
        const uint32_t w = i < 2 ? b.p.x : (i < 4 ? b.p.y : (i < 6 ? b.p.z : b.p.w));
        const uint32_t q = (w >> (16 * (i & 1))) & 0xFFFFu;
        f = lut4[q & 511u];
        s8 = q >> 9;
    } else if constexpr (TYPE == T_IQ2_S) {
        const uint32_t qh = (b.s >> (8 * k)) & 0xFFu;
        f = lut4[byte_of(b.p, 4 * k + l) | (((qh >> (2 * l)) & 3u) << 8)];
        s8 = byte_of(b.p, 8 + 4 * k + l);
    } else if constexpr (TYPE == T_IQ3_XXS) {
        const uint32_t aux = k ? b.x.y : b.x.x;
        const uint2 p0 = lut2[byte_of(b.p, 8 * k + 2 * l)], p1 = lut2[byte_of(b.p, 8 * k + 2 * l + 1)];
        f = make_uint4(p0.x, p0.y, p1.x, p1.y);
        s8 = (aux >> (7 * l)) & 127u;
    } else {  // IQ3_S
        const uint32_t qh = (b.s >> (8 * k)) & 0xFFu;
        const uint2 p0 = lut2[byte_of(b.p, 8 * k + 2 * l) | (((qh >> (2 * l)) & 1u) << 8)];
        const uint2 p1 = lut2[byte_of(b.p, 8 * k + 2 * l + 1) | (((qh >> (2 * l + 1)) & 1u) << 8)];
        f = make_uint4(p0.x, p0.y, p1.x, p1.y);
        s8 = ((k ? b.x.y : b.x.x) >> (8 * l)) & 0xFFu;
    }
    constexpr bool kByte = TYPE == T_IQ2_S || TYPE == T_IQ3_S;
    const uint4 m = iq_sign_masks(kByte ? s8 : iq_ksigns(s8));
    f.x ^= m.x;
    f.y ^= m.y;
    f.z ^= m.z;
    f.w ^= m.w;
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
        uint4 ga[2], gb[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            iq_point<TYPE>(A, c.lut, k, l, ga[k]);
            iq_point<TYPE>(B, c.lut, k, l, gb[k]);
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int wi = 2 * l + half;
            uint4 f[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) f[v] = xb[(wi * 2 * NV + 2 * v) * 4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const uint32_t a0 = half ? ga[k].z : ga[k].x, a2 = half ? ga[k].w : ga[k].y;
                const uint32_t b0 = half ? gb[k].z : gb[k].x, b2 = half ? gb[k].w : gb[k].y;
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
