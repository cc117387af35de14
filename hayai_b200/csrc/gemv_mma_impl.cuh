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
    const int h = e >> 7, r = e & 127, q = r >> 5, s = (r >> 4) & 1, j = (r >> 2) & 3;
    t = 2 * h + s;  // 128h + 32q + 16s + 4j
    mi = 4 * q + j;
}
__device__ __forceinline__ void inv_q80(int e, int& mi, int& t) {
    mi = e >> 4;  // 16mi + 4t
    t = (e & 15) >> 2;
}

template <class F>
__device__ __forceinline__ void inv_map(int e, int& mi, int& t) {
    if constexpr (F::kType == T_Q6_K) inv_q6k(e, mi, t);
    else if constexpr (F::kType == T_Q8_0) inv_q80(e, mi, t);
    else inv_q4k(e, mi, t);  // Q4_K and the IQ formats (the same lane-distributed slots)
}

// Table slot (single vector) of the hi part of 4-element chunk c of the activation; the lo
// part sits F::kLoOff entries further on.
template <class F>
__device__ __forceinline__ int chunk_slot(int c) {
    const int e = 4 * c, kb = e / F::kBlockElems;
    int mi, t;
    inv_map<F>(e - kb * F::kBlockElems, mi, t);
    return kb * table_entries_per_block<F>(1) + F::template tab<1>(mi, 0, t);
}

// One chunk as its two table entries: f16 hi parts and 2^11-scaled lo parts, elements paired
// (0, 2) and (1, 3).  bad: an element outside the f16 range.
__device__ __forceinline__ void pack_chunk(const float (&xs)[4], uint2& hi2, uint2& lo2, bool& bad) {
    __half hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (fabsf(xs[j]) >= 65504.0f && isfinite(xs[j])) bad = true;
        split_f16(xs[j], hi[j], lo[j]);
    }
    hi2 = make_uint2(h2_as_u32(__halves2half2(hi[0], hi[2])), h2_as_u32(__halves2half2(hi[1], hi[3])));
    lo2 = make_uint2(h2_as_u32(__halves2half2(lo[0], lo[2])), h2_as_u32(__halves2half2(lo[1], lo[3])));
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
// Optional second source of the activation (batch 1, persistent FFN stack): the vector is
// x + the sum of `parts` partial vectors stored per 16-row tile as
// part[(tile * parts + p) * 16 + row], added in p order; the float4 chunks [c0, c1) of the
// completed vector are also stored to `out`.
struct XAccum {
    const float* part;  // nullptr: none
    int parts;
    float* out;
    int c0, c1;
};

// How the prologue reads the activation: kLdg = read-only path (the vector is constant for the
// kernel); kLdcg = coherent L2 loads (written earlier in the same kernel by other CTAs);
// kPlain = generic loads (a staging copy in shared memory).
enum XLoad { kLdg = 0, kLdcg = 1, kPlain = 2 };
constexpr int kMaxParts = 8;

// Activation chunk c (4 elements) of vector row xv, plus the partials of acc (all their loads
// are issued before the first add, then added in part order).
template <int LOAD>
__device__ __forceinline__ float4 load_x4(const float* xv, int c, const XAccum& acc) {
    const float4* p4 = reinterpret_cast<const float4*>(xv) + c;
    float4 a = LOAD == kLdg ? __ldg(p4) : (LOAD == kLdcg ? __ldcg(p4) : *p4);
    if (acc.part) {
        const float* pp = acc.part + (size_t)(c >> 2) * acc.parts * 16 + (c & 3) * 4;
        float4 d[kMaxParts];
#pragma unroll
        for (int p = 0; p < kMaxParts; ++p)
            if (p < acc.parts) d[p] = __ldcg(reinterpret_cast<const float4*>(pp + p * 16));
#pragma unroll
        for (int p = 0; p < kMaxParts; ++p) {
            if (p < acc.parts) {
                a.x += d[p].x;
                a.y += d[p].y;
                a.z += d[p].z;
                a.w += d[p].w;
            }
        }
    }
    return a;
}

// Run by threads [0, nthr) of the CTA (all of it by default); `bar` is the named barrier they
// synchronise on.
// rows: optional per-vector row pointers (gathered rows; nullptr rows are zero) instead of
// x + v * ldx.
template <class F, int NV, int LOAD = kLdg>
__device__ void build_prologue(uint2* __restrict__ xt, float* __restrict__ sx, const float* __restrict__ x, int ldx,
                               int K, int nvec, const NormArgs& nrm, float* scratch, int* err, int nthr, int bar,
                               const XAccum& acc = XAccum{nullptr, 0, nullptr, 0, 0},
                               const float* const* rows = nullptr) {
    const int nb = (K + F::kBlockElems - 1) / F::kBlockElems;
    const int nchunk = K >> 2;                         // real float4 chunks
    const int ntab = (nb * F::kBlockElems) >> 2;       // chunks covered by the table (zero padded)
    const int rounds = (ntab + nthr - 1) / nthr;
    bool bad = false;
    for (int v = 0; v < NV; ++v) {
        const float* xv = rows ? rows[v] : x + (size_t)v * ldx;
        const bool live = v < nvec && xv != nullptr;
        float inv = 1.0f;
        if (nrm.w) {
            float s = 0.f;
            if (live) {
                const int nc = nrm.len >> 2;
#pragma unroll 4
                for (int c = threadIdx.x; c < nc; c += nthr) {
                    const float4 a = load_x4<LOAD>(xv, c, acc);
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
                a = load_x4<LOAD>(xv, c, acc);
                if (acc.out && v == 0 && c >= acc.c0 && c < acc.c1) reinterpret_cast<float4*>(acc.out)[c] = a;
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
                const int e = 4 * c, kb = e / F::kBlockElems;
                int mi, t;
                inv_map<F>(e - kb * F::kBlockElems, mi, t);
                const int base = kb * table_entries_per_block<F>(NV) + F::template tab<NV>(mi, v, t);
                pack_chunk(xs, xt[base], xt[base + F::kLoOff], bad);
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

// Per-lane context of the main loop.  The B fragments of kernel block kb are read at
// xb0 + kb * xstride; a lane whose B columns are zero for the format (no vector there, or
// a Q4_K column owned by another lane) points at a zeroed block of the table instead
// (xstride 0), so every fragment load is unconditional.
template <int NV>
struct LaneCtx {
    const uint2* xb0;
    int xstride;      // table entries per kernel block, or 0
    const float* sx;  // Q4_K sub-block sums
    int sxs;          // Q4_K: K/32 (K/16 with sx16)
    int g, t;
    const uint8_t* lut = nullptr;  // IQ formats: the shared-memory codebook
    int sx16 = 0;     // Q4_K: sx holds sums over 16-element halves of the sub-blocks
};

// Lane context for format F: xt = fragment table, zero = a zeroed block of it.
template <class F, int NV>
__device__ __forceinline__ LaneCtx<NV> make_ctx(const uint2* xt, const uint2* zero, const float* sx, int K, int lane) {
    LaneCtx<NV> c;
    c.g = lane >> 2;
    c.t = lane & 3;
    c.sx = sx;
    c.sxs = K / 32;
    int off;
    bool live;
    if constexpr (F::kLaneShares) {
        off = ((c.g & 1) * 4 + c.t) * 2;  // part g&1 of owner lane g>>1, lane t
        live = (c.g >> 1) == c.t;
    } else {
        off = c.g * 4 + c.t;
        live = c.g < 2 * NV;
        if (!live) off = c.t;
    }
    c.xb0 = (live ? xt : zero) + off;
    c.xstride = live ? table_entries_per_block<F>(NV) : 0;
    return c;
}

// ------------------------------------------------------------------ Q4_K
struct Q4KBlk {
    uint4 h, q0, q1;
};

// Q4_K (sc, m) of sub-blocks 2t, 2t+1 of one row, folded into the per-sub-block factors
// c = 64 d sc and k = c + dmin m.  The header (repack.cu) holds lane t's four 6-bit fields as
// 24 bits at byte 4 + 3t: one funnel shift brings them down, and each field becomes f32 under
// the 2^23 magic (a LOP3 and an FADD; a field left at bits 6 or 12 comes out scaled by 64 or
// 4096, which the factor it multiplies absorbs exactly).
__device__ __forceinline__ void q4k_factors(const uint4& h, int t, float& c0, float& k0, float& c1, float& k1) {
    // bits 24t.. of the 96 bits (y, z, w): t = 0, 1 from (y, z), t = 2 from (z, w), t = 3 from w
    const uint32_t V = __funnelshift_r(t < 2 ? h.y : (t == 2 ? h.z : h.w), t < 2 ? h.z : h.w, (24 * t) & 31);
    const float2 dd = __half22float2(u32_as_h2(h.x));
    const float s0 = __uint_as_float((V & 0x3Fu) | 0x4B000000u) - 8388608.0f;               // sc(2t)
    const float s1 = __uint_as_float((V & 0xFC0u) | 0x4B000000u) - 8388608.0f;              // 64 sc(2t+1)
    const float m0 = __uint_as_float((V & 0x3F000u) | 0x4B000000u) - 8388608.0f;            // 4096 m(2t)
    const float m1 = __uint_as_float(((V >> 6) & 0x3F000u) | 0x4B000000u) - 8388608.0f;     // 4096 m(2t+1)
    c0 = (64.f * dd.x) * s0;
    c1 = dd.x * s1;
    const float dm = dd.y * (1.0f / 4096.0f);
    k0 = fmaf(dm, m0, c0);
    k1 = fmaf(dm, m1, c1);
}

// The 8 codes of one Q4_K word as four f16x2 registers, every code as f16(1 + n/64): low
// nibbles of bytes 0/2 (lo02) and 1/3 (lo13), high nibbles of bytes 0/2 (hi02) and 1/3 (hi13).
// High nibbles sit at mantissa bits 4-7 under the 0x3C00 magic (one LOP3 per register; bytes
// 1/3 after one shift by 8); low nibbles at mantissa bits 0-3 under the 0x6400 magic give
// f16(1024 + n), turned into 1 + n/64 = (1024 + n) / 64 - 15 by one exact HFMA2, so two of
// the four registers cost an FMA-pipe op instead of an ALU shift.
__device__ __forceinline__ void q4k_codes(uint32_t w, uint32_t& lo02, uint32_t& lo13, uint32_t& hi02,
                                          uint32_t& hi13) {
    constexpr uint32_t kInv64 = 0x24002400u, kMinus15 = 0xCB80CB80u;  // f16x2 (1/64, 1/64), (-15, -15)
    const uint32_t w8 = w >> 8;
    hi02 = lop3_and_or(w, 0x00F000F0u, 0x3C003C00u);
    hi13 = lop3_and_or(w8, 0x00F000F0u, 0x3C003C00u);
    lo02 = hfma2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), kInv64, kMinus15);
    lo13 = hfma2_u32(lop3_and_or(w8, 0x000F000Fu, 0x64006400u), kInv64, kMinus15);
}

// One Q4_K unit, lane-distributed sub-blocks.  Lane t's codes are chunk t of the super-block
// (q0, q1): the low nibbles are sub-block 2t, the high nibbles sub-block 2t+1.  B holds lane
// t's x only in columns 2t (hi part) and 2t+1 (lo part), so in every MMA lane t's k-slots
// meet only its own columns and the accumulator comes back per sub-block, already spread
// over the lanes: C[row][2t] = sum over the sub-block of A * x_hi.  Codes enter as
// f16(1 + n/64) (magic 0x3C00, nibble at bits 4-7: one LOP3 per two codes), so
//     sum n*x = 64 * (C - Sx_j)
// and the 6-bit scale, d, dmin and the min term (get_scale_min_k4, q4k.rs:34-43; the
// dequantisation q4k.rs:206-256) are applied once per sub-block per lane in f32.  pA/pB
// receive lane t's share of rows g / g+8 of each of the NMAT matrices (the caller sums the
// shares over t).  The table holds, per 8-code word wi, the lo-nibble and hi-nibble B
// fragments side by side, so one 128-bit load feeds both MMAs of every matrix.
template <int NV, int NMAT, bool SHARE_B = true>
__device__ __forceinline__ void q4k_unit(const Q4KBlk (&A)[NMAT], const Q4KBlk (&B)[NMAT], const int (&kbs)[NMAT],
                                         const LaneCtx<NV>& c, float (&pA)[NMAT][NV], float (&pB)[NMAT][NV]) {
    const uint4* xbm[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) xbm[m] = reinterpret_cast<const uint4*>(c.xb0 + kbs[SHARE_B ? 0 : m] * c.xstride);
    float lo[NMAT][NV][4], hi[NMAT][NV][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int i = 0; i < 4; ++i) lo[m][v][i] = hi[m][v][i] = 0.f;
#pragma unroll
    for (int wi = 0; wi < 8; ++wi) {
        uint4 f[NMAT][NV];
#pragma unroll
        for (int m = 0; m < (SHARE_B ? 1 : NMAT); ++m)
#pragma unroll
            for (int v = 0; v < NV; ++v) f[m][v] = xbm[m][(wi * 2 * NV + 2 * v) * 4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            const int fm = SHARE_B ? 0 : m;
            const uint32_t wA[8] = {A[m].q0.x, A[m].q0.y, A[m].q0.z, A[m].q0.w,
                                    A[m].q1.x, A[m].q1.y, A[m].q1.z, A[m].q1.w};
            const uint32_t wB[8] = {B[m].q0.x, B[m].q0.y, B[m].q0.z, B[m].q0.w,
                                    B[m].q1.x, B[m].q1.y, B[m].q1.z, B[m].q1.w};
            uint32_t lo02a, lo13a, hi02a, hi13a, lo02b, lo13b, hi02b, hi13b;
            q4k_codes(wA[wi], lo02a, lo13a, hi02a, hi13a);
            q4k_codes(wB[wi], lo02b, lo13b, hi02b, hi13b);
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                mma16816(lo[m][v], lo02a, lo02b, lo13a, lo13b, f[fm][v].x, f[fm][v].y);
                mma16816(hi[m][v], hi02a, hi02b, hi13a, hi13b, f[fm][v].z, f[fm][v].w);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const int kb = kbs[SHARE_B ? 0 : m];
        float2 s[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (c.sx16) {
                const float4 h = *reinterpret_cast<const float4*>(c.sx + v * c.sxs + kb * 16 + 4 * c.t);
                s[v] = make_float2(h.x + h.y, h.z + h.w);
            } else {
                s[v] = *reinterpret_cast<const float2*>(c.sx + v * c.sxs + kb * 8 + 2 * c.t);
            }
        }
        float cA0, kA0, cA1, kA1, cB0, kB0, cB1, kB1;
        q4k_factors(A[m].h, c.t, cA0, kA0, cA1, kA1);
        q4k_factors(B[m].h, c.t, cB0, kB0, cB1, kB1);
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            pA[m][v] += cA0 * (lo[m][v][0] + lo[m][v][1] * kLoScale) - s[v].x * kA0 +
                        cA1 * (hi[m][v][0] + hi[m][v][1] * kLoScale) - s[v].y * kA1;
            pB[m][v] += cB0 * (lo[m][v][2] + lo[m][v][3] * kLoScale) - s[v].x * kB0 +
                        cB1 * (hi[m][v][2] + hi[m][v][3] * kLoScale) - s[v].y * kB1;
        }
    }
}

// ------------------------------------------------------------------ Q6_K (GPU layout)
// Lane-distributed (repack.cu): lane t of a row owns half h = t >> 1 and l in [16s, 16s + 16),
// s = t & 1, i.e. the four scale groups 8h + 2q + s (q < 4) whole: elements 128h + 32q + 16s + i.
// Its pieces: l0 = ql bytes 64h + 16s + i (low nibble: q = 0, high: q = 2), l1 = ql bytes
// 64h + 32 + 16s + i (q = 1, 3), qh = qh bytes 32h + 16s + i (bits 2q..2q+1), sc = the int8
// scales of its groups (byte q), and d (q6k.rs:26-57).  MMA mi = 4q + j takes codes
// i = 4j..4j+3 of group q, bytes 0/2 in k-slots 2t, 2t+1 and bytes 1/3 in 2t+8, 2t+9 (the
// pairing of Q4_K); B holds lane t's x only in columns 2t (hi) and 2t+1 (lo), so each group's
// accumulator stays on its own lane and the scale is applied once per group (4 MMAs) in f32.
// pA/pB receive the lane's share of rows g / g+8 (summed over t by the caller).  The codes
// enter as f16(1024 + c) by one PRMT of the merged 6-bit bytes and one exact HSUB2 of 1056.
struct Q6KBlk {
    uint4 l0, l1, qh;
    uint32_t sc;
    uint16_t d;
};

template <int NV>
__device__ __forceinline__ void q6k_unit(const Q6KBlk& A, const Q6KBlk& B, int kb, const LaneCtx<NV>& c,
                                         float (&pA)[1][NV], float (&pB)[1][NV]) {
    const uint32_t kOff = 0x64206420u;  // (1056, 1056) in f16: 1024 magic + 32 code offset
    const uint32_t LA[2][4] = {{A.l0.x, A.l0.y, A.l0.z, A.l0.w}, {A.l1.x, A.l1.y, A.l1.z, A.l1.w}};
    const uint32_t LB[2][4] = {{B.l0.x, B.l0.y, B.l0.z, B.l0.w}, {B.l1.x, B.l1.y, B.l1.z, B.l1.w}};
    const uint32_t QA[4] = {A.qh.x, A.qh.y, A.qh.z, A.qh.w};
    const uint32_t QB[4] = {B.qh.x, B.qh.y, B.qh.z, B.qh.w};
    const uint4* xb = reinterpret_cast<const uint4*>(c.xb0 + kb * c.xstride);
    float acc[4][NV][4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[q][v][i] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
            uint4 f[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) f[v] = xb[((2 * q + jp) * 2 * NV + 2 * v) * 4];
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int j = 2 * jp + jj;
                const uint32_t la = LA[q & 1][j], lb = LB[q & 1][j];
                const int qs = 4 - 2 * q;  // qh bits 2q..2q+1 -> bits 4..5 of each byte
                const uint32_t ha = (qs >= 0 ? QA[j] << qs : QA[j] >> -qs) & 0x30303030u;
                const uint32_t hb = (qs >= 0 ? QB[j] << qs : QB[j] >> -qs) & 0x30303030u;
                const uint32_t ua = lop3_and_or(q < 2 ? la : (la >> 4), 0x0F0F0F0Fu, ha);
                const uint32_t ub = lop3_and_or(q < 2 ? lb : (lb >> 4), 0x0F0F0F0Fu, hb);
                const uint32_t a0 = hsub2_u32(prmt(ua, 0x64646464u, 0x4240u), kOff);
                const uint32_t a1 = hsub2_u32(prmt(ub, 0x64646464u, 0x4240u), kOff);
                const uint32_t a2 = hsub2_u32(prmt(ua, 0x64646464u, 0x4341u), kOff);
                const uint32_t a3 = hsub2_u32(prmt(ub, 0x64646464u, 0x4341u), kOff);
#pragma unroll
                for (int v = 0; v < NV; ++v)
                    mma16816(acc[q][v], a0, a1, a2, a3, jj ? f[v].z : f[v].x, jj ? f[v].w : f[v].y);
            }
        }
    }
    const uint32_t SA = A.sc ^ 0x80808080u, SB = B.sc ^ 0x80808080u;  // flipped for s8_to_f32_flipped
    const float dA = h2f(A.d), dB = h2f(B.d);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            sa += s8_to_f32_flipped(SA, q) * (acc[q][v][0] + acc[q][v][1] * kLoScale);
            sb += s8_to_f32_flipped(SB, q) * (acc[q][v][2] + acc[q][v][3] * kLoScale);
        }
        pA[0][v] += dA * sa;
        pB[0][v] += dB * sb;
    }
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
    const uint32_t kOff = 0x64806480u;  // (1152, 1152): 1024 magic + 128 sign flip
    const uint32_t WA[8] = {A.q0.x, A.q0.y, A.q0.z, A.q0.w, A.q1.x, A.q1.y, A.q1.z, A.q1.w};
    const uint32_t WB[8] = {B.q0.x, B.q0.y, B.q0.z, B.q0.w, B.q1.x, B.q1.y, B.q1.z, B.q1.w};
    const float2 dA01 = __half22float2(u32_as_h2(A.d.x)), dA23 = __half22float2(u32_as_h2(A.d.y));
    const float2 dB01 = __half22float2(u32_as_h2(B.d.x)), dB23 = __half22float2(u32_as_h2(B.d.y));
    const float fa[4] = {dA01.x, dA01.y, dA23.x, dA23.y};
    const float fb[4] = {dB01.x, dB01.y, dB23.x, dB23.y};
    const uint2* xb = c.xb0 + kg * c.xstride;
    float sA = 0.f, sB = 0.f;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int w = 2 * blk + half;
            const uint32_t ua = WA[w] ^ 0x80808080u, ub = WB[w] ^ 0x80808080u;
            const uint2 f = xb[w * (2 * NV * 4)];
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
        if constexpr (kShared) {
            A.sc = *reinterpret_cast<const uint32_t*>(tb + F::kSc + 16 * g + 4 * t);
            B.sc = *reinterpret_cast<const uint32_t*>(tb + F::kSc + 16 * (g + 8) + 4 * t);
            A.d = *reinterpret_cast<const uint16_t*>(tb + F::kD + 2 * g);
            B.d = *reinterpret_cast<const uint16_t*>(tb + F::kD + 2 * (g + 8));
        } else {
            A.sc = ldg_stream32(tb + F::kSc + 16 * g + 4 * t);
            B.sc = ldg_stream32(tb + F::kSc + 16 * (g + 8) + 4 * t);
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
    if constexpr (F::kLaneShares) {
        float pa[1][NV], pb[1][NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) pa[0][v] = pb[0][v] = 0.f;
        if constexpr (F::kType == T_Q4_K) {
            const Q4KBlk a1[1] = {A}, b1[1] = {B};
            const int k1[1] = {kb};
            q4k_unit<NV, 1>(a1, b1, k1, c, pa, pb);
        } else {
            q6k_unit<NV>(A, B, kb, c, pa, pb);
        }
        dA = dB = 0.f;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            float sa = pa[0][v], sb = pb[0][v];
            sa += __shfl_xor_sync(kFull, sa, 1);
            sb += __shfl_xor_sync(kFull, sb, 1);
            sa += __shfl_xor_sync(kFull, sa, 2);
            sb += __shfl_xor_sync(kFull, sb, 2);
            if (c.t == v) {
                dA = sa;
                dB = sb;
            }
        }
    }
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
