// gemv_simple.cu -- CUDA-core kernels on the raw GGUF layout: F32, F16, BF16, IQ4_NL / IQ4_XS,
// the other GGML block formats (Q4_0, Q4_1, Q5_0, Q5_1, Q8_1, Q2_K, Q3_K, Q5_K, Q8_K), the toy
// LUT-Q4 matmul, and the elementwise SwiGLU combine.  (The IQ2 / IQ3 codebook formats run on
// the tensor-core GEMV: gemv_iq.cuh.)
//
// Reference semantics: gemv_f32 (crates/hayai-model/src/quant.rs:358-369), IQ4_NL / IQ4_XS
// (iq4.rs:36-42, :121-138), Q4_0 / Q4_1 (quant.rs:538-596, :617-650), Q5_0 / Q5_1
// (q5.rs:26-158), Q2_K (q2k.rs:26-58), Q3_K (q3k.rs:10-30, :52-84), Q5_K (q5k.rs:10-66),
// gemv_f16 / gemv_bf16 / gemv_q8_1 / gemv_q8_k (quant.rs:371-395, :458-501),
// cpu_lut_matmul_q4 (crates/hayai-cpu/src/matmul.rs:48-82).
#include "common.cuh"
#include "gemv_launch.h"

#define HC_IQ_QUAL static __device__ const
#include "_gen/iq_tables.h"

namespace hc {

// Byte loads of a block; the group kernel stages blocks in shared memory, so these are
// generic loads (no read-only-path form, which only addresses global memory).
__device__ __forceinline__ uint32_t ldb(const uint8_t* p) { return *p; }
__device__ __forceinline__ uint32_t ld_u16u(const uint8_t* p) { return ldb(p) | (ldb(p + 1) << 8); }
__device__ __forceinline__ uint32_t ld_u32u(const uint8_t* p) { return ld_u16u(p) | (ld_u16u(p + 2) << 16); }
__device__ __forceinline__ float ld_f16u(const uint8_t* p) { return h2f((uint16_t)ld_u16u(p)); }

// get_scale_min_k4 (q4k.rs:34-43, q5k.rs:10-18): 6-bit scale and min j of a K-quant header.
__device__ __forceinline__ void scale_min_k4(const uint8_t* s, int j, float& sc, float& m) {
    if (j < 4) {
        sc = (float)(ldb(s + j) & 63u);
        m = (float)(ldb(s + j + 4) & 63u);
    } else {
        sc = (float)((ldb(s + j + 4) & 0x0Fu) | ((ldb(s + j - 4) >> 6) << 4));
        m = (float)((ldb(s + j + 4) >> 4) | ((ldb(s + j) >> 6) << 4));
    }
}

// Q3_K scale i (0..15) of the 12 packed bytes, as unpack_q3_k_scales (q3k.rs:10-30) lays
// them out: low 4 bits from byte i (i < 8) or the high nibble of byte i - 8, top 2 bits from
// byte 8 + i % 4 at bit 2 (i / 4); minus 32.
__device__ __forceinline__ float q3k_scale(const uint8_t* s12, int i) {
    const uint32_t lo = i < 8 ? (ldb(s12 + i) & 0x0Fu) : (ldb(s12 + i - 8) >> 4);
    const uint32_t hi = (ldb(s12 + 8 + (i & 3)) >> (2 * (i >> 2))) & 3u;
    return (float)((int)(lo | (hi << 4)) - 32);
}

// Elements e..e+3 (e a multiple of 4) of the 32-element group ib32 of a block, dotted with x4:
// the same values as group_dot, one quarter-octet at a time, so that 8 lanes share a group and
// a warp's activation loads are 512 contiguous bytes.
template <int TYPE>
__device__ __forceinline__ float group_dot4(const uint8_t* blk, int ib32, int e, const float4& x) {
    float w[4];
    if constexpr (TYPE == T_Q4_0 || TYPE == T_Q4_1 || TYPE == T_Q5_0 || TYPE == T_Q5_1 || TYPE == T_IQ4_NL) {
        // element j < 16: low nibble of qs[j]; j >= 16: high nibble of qs[j - 16]
        const float d = ld_f16u(blk);
        const float m = (TYPE == T_Q4_1 || TYPE == T_Q5_1) ? ld_f16u(blk + 2) : 0.f;
        const int qoff = TYPE == T_Q4_0 || TYPE == T_IQ4_NL ? 2 : TYPE == T_Q4_1 ? 4 : TYPE == T_Q5_0 ? 6 : 8;
        const uint32_t qh = TYPE == T_Q5_0 ? ld_u32u(blk + 2) : TYPE == T_Q5_1 ? ld_u32u(blk + 4) : 0u;
        const bool hi = e >= 16;
        const int j0 = hi ? e - 16 : e;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = j0 + i;
            const uint32_t q = ldb(blk + qoff + j);
            uint32_t c = hi ? q >> 4 : q & 0x0Fu;
            if constexpr (TYPE == T_Q5_0 || TYPE == T_Q5_1) c |= hi ? (qh >> (j + 12)) & 0x10u : ((qh >> j) << 4) & 0x10u;
            if constexpr (TYPE == T_Q4_0) w[i] = (float)((int)c - 8) * d;
            else if constexpr (TYPE == T_Q5_0) w[i] = (float)((int)c - 16) * d;
            else if constexpr (TYPE == T_IQ4_NL) w[i] = d * (float)hc_iq4nl_values[c];
            else w[i] = (float)c * d + m;
        }
    } else if constexpr (TYPE == T_Q2_K || TYPE == T_Q3_K) {
        // half n = ib32 / 4, shift 2 (ib32 % 4); elements 0-15 from q[l], 16-31 from q[16 + l]
        const int n = ib32 >> 2, jj = ib32 & 3, h = e >> 4, l0 = e & 15;
        const uint8_t* q = blk + (TYPE == T_Q2_K ? 16 : 32) + 32 * n + 16 * h;
        if constexpr (TYPE == T_Q2_K) {
            const uint32_t sc = ldb(blk + 8 * n + 2 * jj + h);
            const float dl = ld_f16u(blk + 80) * (float)(sc & 0xFu), ml = ld_f16u(blk + 82) * (float)(sc >> 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = dl * (float)((ldb(q + l0 + i) >> (2 * jj)) & 3u) - ml;
        } else {
            const float dl = ld_f16u(blk + 108) * q3k_scale(blk + 96, 8 * n + 2 * jj + h);
            const uint32_t mbit = 1u << (4 * n + jj);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int qv = (int)((ldb(q + l0 + i) >> (2 * jj)) & 3u);
                const int hm = (ldb(blk + 16 * h + l0 + i) & mbit) ? 0 : 4;
                w[i] = dl * (float)(qv - hm);
            }
        }
    } else if constexpr (TYPE == T_Q5_K) {
        const int c = ib32 >> 1, hi = ib32 & 1;
        float sc, mn;
        scale_min_k4(blk + 4, ib32, sc, mn);
        const float d1 = ld_f16u(blk) * sc, m1 = ld_f16u(blk + 2) * mn;
        const uint32_t u = (hi ? 2u : 1u) << (2 * c);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t ql = ldb(blk + 48 + 32 * c + e + i);
            const uint32_t v = (hi ? ql >> 4 : ql & 0x0Fu) + ((ldb(blk + 16 + e + i) & u) ? 16u : 0u);
            w[i] = d1 * (float)v - m1;
        }
    } else if constexpr (TYPE == T_Q8_1) {
        // {f16 d, f16 s, int8 qs[32]}: element j = qs[j] d (s is not read)
        const float d = ld_f16u(blk);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = (float)(int8_t)ldb(blk + 4 + e + i) * d;
    } else if constexpr (TYPE == T_Q8_K) {
        // {f32 d, int8 qs[256], int16 bsums[16]}: element j = qs[j] d (bsums are not read)
        const float d = __uint_as_float(ld_u32u(blk));
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = (float)(int8_t)ldb(blk + 4 + 32 * ib32 + e + i) * d;
    } else if constexpr (TYPE == T_IQ4_XS) {
        const uint32_t sh = ld_u16u(blk + 2);
        const int ls = (int)(((ldb(blk + 4 + ib32 / 2) >> (4 * (ib32 & 1))) & 0x0Fu) | (((sh >> (2 * ib32)) & 3u) << 4));
        const float dl = ld_f16u(blk) * (float)(ls - 32);
        const bool hi = e >= 16;
        const uint8_t* qs = blk + 8 + 16 * ib32 + (hi ? e - 16 : e);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t q = ldb(qs + i);
            w[i] = dl * (float)hc_iq4nl_values[hi ? q >> 4 : q & 0x0Fu];
        }
    }
    return w[0] * x.x + w[1] * x.y + w[2] * x.z + w[3] * x.w;
}

// One warp per (row, vector).  The warp first stages a segment of whole blocks of the row
// (<= kGroupSeg bytes) in its shared-memory buffer with coalesced 16-byte loads (the raw GGUF
// rows are byte-aligned only; the copy starts at the 16-byte boundary below the segment and
// may read up to 15 bytes past the row, inside the 16 bytes of padding every weight allocation
// carries), then decodes it with 4 lanes per 32-element group, 8 elements each (QK elements
// and BLK bytes per block, QK / 32 groups per block).  One lane per group made every
// activation load instruction touch 32 cache lines and ran at 0.04-0.09 of the HBM peak.
constexpr int kGroupSeg = 4096;

template <int TYPE, int QK, int BLK>
__global__ void __launch_bounds__(256, 4) gemv_group_kernel(const uint8_t* __restrict__ w, size_t row_bytes, int M,
                                                          int K, const float* __restrict__ x, int ldx,
                                                          float* __restrict__ y, int ldy, const float* resid, int ldr,
                                                          int nvec) {
    constexpr int G = QK / 32;
    constexpr int SEGB = kGroupSeg / BLK;  // blocks per segment
    __shared__ __align__(16) uint8_t sbuf[8][kGroupSeg + 32];
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int warp = blockIdx.x * 8 + wib, nwarps = gridDim.x * 8;
    uint8_t* buf = sbuf[wib];
    const int nb = K / QK;
    for (int rv = warp; rv < M * nvec; rv += nwarps) {
        const int row = rv % M, v = rv / M;
        const uint8_t* wr = w + (size_t)row * row_bytes;
        const float* xv = x + (size_t)v * ldx;
        float s = 0.f;
        for (int b0 = 0; b0 < nb; b0 += SEGB) {
            const int nbs = nb - b0 < SEGB ? nb - b0 : SEGB;
            const uintptr_t g0 = reinterpret_cast<uintptr_t>(wr + (size_t)b0 * BLK), a0 = g0 & ~(uintptr_t)15;
            const int lead = (int)(g0 - a0), nchunks = (lead + nbs * BLK + 15) >> 4;
            __syncwarp();  // the previous segment has been decoded
            for (int c = lane; c < nchunks; c += 32)
                *reinterpret_cast<uint4*>(buf + 16 * c) = ldg_stream128(reinterpret_cast<const void*>(a0 + 16 * c));
            __syncwarp();
            const uint8_t* sb = buf + lead;
            if constexpr (QK == 256) {
                // super-block formats: 4 lanes per group, 8 elements each (two 4-element slices
                // share one read of the block header); lanes 4g..4g+3 read the group's 128 B of x
                for (int gi = lane >> 2; gi < nbs * G; gi += 8) {
                    const int b = gi / G, ib32 = gi % G, e = 8 * (lane & 3);
                    const float4* xp = reinterpret_cast<const float4*>(xv + (size_t)(b0 + b) * QK + 32 * ib32 + e);
                    const float4 xa = __ldg(xp), xb = __ldg(xp + 1);
                    s += group_dot4<TYPE>(sb + b * BLK, ib32, e, xa) + group_dot4<TYPE>(sb + b * BLK, ib32, e + 4, xb);
                }
            } else {
                // 32-element blocks: 4 lanes per block, 8 elements each, elements e..e+3 and
                // e+16..e+19 (the low and high nibbles of the same 4 bytes, read once)
                for (int gi = lane >> 2; gi < nbs * G; gi += 8) {
                    const int b = gi / G, ib32 = gi % G, e = 4 * (lane & 3);
                    const float* xp = xv + (size_t)(b0 + b) * QK + 32 * ib32 + e;
                    const float4 xa = __ldg(reinterpret_cast<const float4*>(xp));
                    const float4 xb = __ldg(reinterpret_cast<const float4*>(xp + 16));
                    s += group_dot4<TYPE>(sb + b * BLK, ib32, e, xa) + group_dot4<TYPE>(sb + b * BLK, ib32, e + 16, xb);
                }
            }
        }
        s = warp_sum(s);
        if (lane == 0) y[(size_t)v * ldy + row] = (resid ? resid[(size_t)v * ldr + row] : 0.f) + s;
    }
}

__global__ void __launch_bounds__(256) gemv_f32_kernel(const float* __restrict__ w, size_t row_floats, int M, int K,
                                                        const float* __restrict__ x, int ldx, float* __restrict__ y,
                                                        int ldy, const float* resid, int ldr, int nvec) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int rv = warp; rv < M * nvec; rv += nwarps) {
        const int row = rv % M, v = rv / M;
        const float* wr = w + (size_t)row * row_floats;
        const float* xv = x + (size_t)v * ldx;
        float s = 0.f;
        for (int c = lane; c < K; c += 32) s += __ldg(wr + c) * __ldg(xv + c);
        s = warp_sum(s);
        if (lane == 0) y[(size_t)v * ldy + row] = (resid ? resid[(size_t)v * ldr + row] : 0.f) + s;
    }
}

// F16 / BF16 rows (quant.rs:371-395): one warp per (row, vector); with K a multiple of 8 every
// lane reads 16 bytes (8 elements) per step, the warp 512 contiguous bytes; otherwise one
// element per lane per step.  BF16 is the upper half of an f32 (exact widening).
template <bool BF>
__device__ __forceinline__ float half_to_f32(uint32_t h) {
    return BF ? __uint_as_float(h << 16) : h2f((uint16_t)h);
}

template <bool BF>
__global__ void __launch_bounds__(256) gemv_half_kernel(const uint16_t* __restrict__ w, size_t row_elems, int M, int K,
                                                        const float* __restrict__ x, int ldx, float* __restrict__ y,
                                                        int ldy, const float* resid, int ldr, int nvec) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const bool vec = (K & 7) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (ldx & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    for (int rv = warp; rv < M * nvec; rv += nwarps) {
        const int row = rv % M, v = rv / M;
        const uint16_t* wr = w + (size_t)row * row_elems;
        const float* xv = x + (size_t)v * ldx;
        float s = 0.f;
        if (vec) {
            for (int c = 8 * lane; c < K; c += 256) {
                const uint4 q = ldg_stream128(wr + c);
                const float4 xa = __ldg(reinterpret_cast<const float4*>(xv + c));
                const float4 xb = __ldg(reinterpret_cast<const float4*>(xv + c + 4));
                s += half_to_f32<BF>(q.x & 0xFFFFu) * xa.x;
                s += half_to_f32<BF>(q.x >> 16) * xa.y;
                s += half_to_f32<BF>(q.y & 0xFFFFu) * xa.z;
                s += half_to_f32<BF>(q.y >> 16) * xa.w;
                s += half_to_f32<BF>(q.z & 0xFFFFu) * xb.x;
                s += half_to_f32<BF>(q.z >> 16) * xb.y;
                s += half_to_f32<BF>(q.w & 0xFFFFu) * xb.z;
                s += half_to_f32<BF>(q.w >> 16) * xb.w;
            }
        } else {
            for (int c = lane; c < K; c += 32) s += half_to_f32<BF>(__ldg(wr + c)) * __ldg(xv + c);
        }
        s = warp_sum(s);
        if (lane == 0) y[(size_t)v * ldy + row] = (resid ? resid[(size_t)v * ldr + row] : 0.f) + s;
    }
}

static int grid_for(int work_warps) {
    int blocks = (work_warps + 7) / 8;
    return blocks < 1 ? 1 : (blocks > 65535 ? 65535 : blocks);
}

bool gemv_simple_supported(int type) {
    switch (type) {
        case T_F32: case T_Q4_0:
        case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q2_K: case T_Q3_K: case T_Q5_K: case T_IQ4_NL: case T_IQ4_XS:
        case T_F16: case T_BF16: case T_Q8_1: case T_Q8_K:
            return true;
        default:
            return false;
    }
}

cudaError_t launch_gemv_simple(int type, const uint8_t* w, size_t row_bytes, int M, int K, const float* x, int ldx,
                               float* y, int ldy, const float* resid, int ldr, int nvec, cudaStream_t stream) {
    const int grid = grid_for(M * nvec);
    switch (type) {
        case T_F32:
            gemv_f32_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float*>(w), row_bytes / 4, M, K, x, ldx,
                                                      y, ldy, resid, ldr, nvec);
            break;
        case T_F16:
            gemv_half_kernel<false><<<grid, 256, 0, stream>>>(reinterpret_cast<const uint16_t*>(w), row_bytes / 2, M, K,
                                                             x, ldx, y, ldy, resid, ldr, nvec);
            break;
        case T_BF16:
            gemv_half_kernel<true><<<grid, 256, 0, stream>>>(reinterpret_cast<const uint16_t*>(w), row_bytes / 2, M, K,
                                                            x, ldx, y, ldy, resid, ldr, nvec);
            break;
#define HC_GROUP_CASE(T, QK, BLK)                                                                       \
    case T:                                                                                             \
        gemv_group_kernel<T, QK, BLK><<<grid, 256, 0, stream>>>(w, row_bytes, M, K, x, ldx, y, ldy, resid, ldr, \
                                                                nvec);                                  \
        break;
        HC_GROUP_CASE(T_Q4_0, 32, 18)
        HC_GROUP_CASE(T_Q4_1, 32, 20)
        HC_GROUP_CASE(T_Q5_0, 32, 22)
        HC_GROUP_CASE(T_Q5_1, 32, 24)
        HC_GROUP_CASE(T_IQ4_NL, 32, 18)
        HC_GROUP_CASE(T_Q2_K, 256, 84)
        HC_GROUP_CASE(T_Q3_K, 256, 110)
        HC_GROUP_CASE(T_Q5_K, 256, 176)
        HC_GROUP_CASE(T_IQ4_XS, 256, 136)
        HC_GROUP_CASE(T_Q8_1, 32, 36)
        HC_GROUP_CASE(T_Q8_K, 256, 292)
#undef HC_GROUP_CASE
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ------------------------------------------------------------------ toy LUT-Q4
// cpu_lut_matmul_q4 (matmul.rs:48-82): y[m] = sum_c x[2c]*LUT[b&15] + x[2c+1]*LUT[b>>4];
// the 16-entry LUT lives in shared memory.
__global__ void __launch_bounds__(256) lut_q4_kernel(const uint8_t* __restrict__ w, int M, int N,
                                                      const float* __restrict__ lut16, const float* __restrict__ x,
                                                      float* __restrict__ y, bool stage_x, bool words) {
    __shared__ float lut[16];
    extern __shared__ __align__(16) float xs[];  // x, when staged (N floats)
    if (threadIdx.x < 16) lut[threadIdx.x] = lut16[threadIdx.x];
    if (stage_x)
        for (int i = threadIdx.x; i < N; i += blockDim.x) xs[i] = __ldg(x + i);
    __syncthreads();
    const float* xv = stage_x ? xs : x;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int pc = N / 2;
    for (int row = warp; row < M; row += nwarps) {
        const uint8_t* wr = w + (size_t)row * pc;
        float s = 0.f;
        if (words) {
            // 4 bytes (8 codes) per lane and step: byte k of word c holds elements 8c + 2k (low
            // nibble) and 8c + 2k + 1 (high nibble); x comes from shared memory
            const uint32_t* w4 = reinterpret_cast<const uint32_t*>(wr);
            for (int c = lane; c < pc / 4; c += 32) {
                const uint32_t b = __ldg(w4 + c);
                const float4 xa = *reinterpret_cast<const float4*>(xv + 8 * c);
                const float4 xb = *reinterpret_cast<const float4*>(xv + 8 * c + 4);
                s += xa.x * lut[b & 15] + xa.y * lut[(b >> 4) & 15] + xa.z * lut[(b >> 8) & 15] +
                     xa.w * lut[(b >> 12) & 15] + xb.x * lut[(b >> 16) & 15] + xb.y * lut[(b >> 20) & 15] +
                     xb.z * lut[(b >> 24) & 15] + xb.w * lut[b >> 28];
            }
        } else {
            for (int c = lane; c < pc; c += 32) {
                const uint32_t b = __ldg(wr + c);
                s += xv[2 * c] * lut[b & 15] + xv[2 * c + 1] * lut[b >> 4];
            }
        }
        s = warp_sum(s);
        if (lane == 0) y[row] = s;
    }
}

cudaError_t launch_lut_matmul_q4(const uint8_t* w, int M, int N, const float* lut16, const float* x, float* y,
                                 cudaStream_t stream) {
    // x is staged in shared memory when it fits the default 48 KB; the word path needs whole
    // 4-byte words per row (N a multiple of 8) on 4-byte aligned weights
    const bool stage_x = (size_t)N * 4 <= 48 * 1024;
    const bool words = stage_x && N % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 3) == 0;
    lut_q4_kernel<<<grid_for(M), 256, stage_x ? (size_t)N * 4 : 0, stream>>>(w, M, N, lut16, x, y, stage_x, words);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ RMSNorm rows
// out[v][i] = (x[v][i] * inv_v) * w[i] for i < len, zero padding up to K
// (rms_norm, crates/hayai-cpu/src/attention.rs:142-147; one CTA per row).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* __restrict__ x, int ldx,
                                                       const float* __restrict__ w, int len, int K, float eps,
                                                       float* __restrict__ out, int ldo) {
    __shared__ float red[8];
    const float* xr = x + (size_t)blockIdx.x * ldx;
    float s = 0.f;
    for (int i = threadIdx.x; i < len; i += blockDim.x) s += xr[i] * xr[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    const float inv = 1.0f / sqrtf(t / (float)len + eps);
    float* o = out + (size_t)blockIdx.x * ldo;
    for (int i = threadIdx.x; i < K; i += blockDim.x) o[i] = i < len ? xr[i] * inv * w[i] : 0.f;
}

cudaError_t launch_rms_norm(const float* x, int ldx, const float* w, int len, int K, float eps, float* out, int ldo,
                            int nvec, cudaStream_t stream) {
    rms_norm_kernel<<<nvec, 256, 0, stream>>>(x, ldx, w, len, K, eps, out, ldo);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ SwiGLU combine
__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ h,
                              size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        h[i] = silu_mul(g[i], u[i]);
}

cudaError_t launch_swiglu(const float* g, const float* u, float* h, size_t n, cudaStream_t stream) {
    size_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    swiglu_kernel<<<(unsigned)blocks, 256, 0, stream>>>(g, u, h, n);
    return cudaGetLastError();
}

}  // namespace hc
