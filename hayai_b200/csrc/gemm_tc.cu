// gemm_tc.cu -- batched Q8_0 GEMV (B >= 8 activation rows) on the 5th-generation tensor cores.
//
// Reference semantics: gemv_q8_0 (crates/hayai-model/src/quant.rs:598-615) applied to every row
// of a batch, the multi-row case of execute_quant_gemv_batched (crates/hayai-opencl/src/
// orchestrator.rs:240-267, which loops over rows on the CPU path).
//
// Y[t][m] = sum_k W[m][k] x[t][k] with W in Q8_0 (per 32-element block: int8 codes q and an f16
// scale d).  The block scale changes every 32 elements and every row, so it cannot ride on a
// TMEM accumulator; instead the weights are dequantised in shared memory into two exact f16
// operands: with w' = q * d * 2^8, A_hi = f16(w') (HMUL2) and A_lo = w' - A_hi (one HFMA2, exact:
// q has 8 significant bits and d 11, so the remainder has at most 8), and A_hi + A_lo = w'
// exactly.  The activations enter as two f16 columns per row, x = x_hi + x_lo * 2^-11 (rows
// [0, Bp) and [Bp, 2 Bp) of the B operand), so one tcgen05.mma with N = 2 Bp multiplies both,
// and D = A_hi X + A_lo X accumulates in f32 in TMEM; the epilogue forms
// y = (D[:, t] + D[:, Bp + t] * 2^-11) * 2^-8.
//
// CTA = 128 output rows (the MMA's M) over a K range (split K: partial outputs per split, added
// by the finishing kernel in split order, so results are deterministic), 10 warps:
//   warp 0    TMA producers: lane 0 per 128-element group one bulk copy per 16-row tile of
//             the tile-major weight layout (8 x 2176 B); lane 1 the activation chunks (64 K
//             each, prepared in the MMA's operand layout by tc_prep_kernel, one copy each);
//   warp 1    owns the TMEM columns; one elected lane issues the MMAs (4 K-steps x {hi, lo}
//             per 64-K chunk) and tcgen05.commit frees the operand buffers;
//   warps 2-9 dequantise each weight half-group into the A_hi / A_lo operand buffers (K-major,
//             128-byte swizzle: rows of 128 B, 16-byte chunks XOR-permuted by row), then warps
//             2-5 read the accumulator (tcgen05.ld, one TMEM lane quarter each) and write the
//             partial outputs.
// Every wait is bounded (~1 s; error bit 1), and the TMEM columns are freed on every path.
#include <cuda_fp16.h>

#include <cmath>

#include "common.cuh"
#include "gemv_launch.h"

namespace hc {

constexpr int kTcRows = 128;               // output rows per CTA (MMA M)
constexpr int kTcChunk = 64;               // K per operand buffer
constexpr int kTcImg = 2176;               // Q8_0 tile-block image: 16 rows x 128 K
constexpr int kTcGps = 2;                  // 128-K groups per weight stage
constexpr int kTcWStage = 8 * kTcGps * kTcImg;  // the CTA's 8 row tiles x kTcGps groups
constexpr int kTcABytes = kTcRows * kTcChunk * 2;  // one f16 operand buffer (16 KB)
constexpr int kTcThreads = 320;            // 10 warps
constexpr int kTcMaxRing = 8;
constexpr float kTcWScale = 256.f;         // w' = q * d * 2^8

struct TcArgs {
    const uint8_t* w[2];  // tile-major Q8_0 matrices (blockIdx.z picks one)
    long long tstride;    // bytes per 16-row tile
    int M, K;
    const uint8_t* xc;    // activations, canonical: [K / 64 chunks][N rows][64] f16
    int N, B;             // MMA N = 2 Bp (hi rows, then lo rows); real rows
    int cps;              // 64-K chunks per K split (even)
    float* out;           // [z][split][B][M] partial outputs
    int* err;
    int SW, NX, NA;       // ring depths: weight groups, activation chunks, operand buffers
};

// Byte offset of (row r, k) in a 64-K operand buffer in the K-major 128-byte-swizzled layout:
// every row is 128 B (64 f16 of K), 8 rows form a 1024-B atom, and the 16-byte chunk k / 8 of
// row r sits at chunk (k / 8) ^ (r % 8), so the rows of an atom spread over all banks (the
// unswizzled interleaved layout put every 8-row group on the same banks and ran the MMA at a
// third of its rate).  Buffers start on 1024-byte boundaries (the swizzle keys on address bits).
__host__ __device__ __forceinline__ int tc_canon(int r, int k) {
    return r * 128 + ((((k >> 3) ^ r) & 7) << 4) + (k & 7) * 2;
}

// Shared-memory matrix descriptor (sm100 UMMA, K-major, SWIZZLE_128B): start address, leading
// byte offset 16 (unused by the swizzled K-major form, set to one unit), stride byte offset 1024
// (8-row atoms), version 1, layout type 2.  K steps of 16 advance the start by 32 bytes.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Four int8 codes (one word) times the block scale: exact hi/lo f16 pairs, k-adjacent codes
// packed low half first.
__device__ __forceinline__ void tc_dequant4(uint32_t word, __half2 d, uint2& hi, uint2& lo) {
    const uint32_t f = word ^ 0x80808080u;  // offset-binary codes q + 128
    const uint32_t kBias = 0x64806480u;     // f16 (1152, 1152) = 1024 magic + 128
    const __half2 q01 = u32_as_h2(hsub2_u32(prmt(f, 0x64646464u, 0x4140u), kBias));
    const __half2 q23 = u32_as_h2(hsub2_u32(prmt(f, 0x64646464u, 0x4342u), kBias));
    const __half2 h01 = __hmul2(q01, d), h23 = __hmul2(q23, d);
    hi = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
    lo = make_uint2(h2_as_u32(__hfma2(q01, d, __hneg2(h01))), h2_as_u32(__hfma2(q23, d, __hneg2(h23))));
}

__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint32_t s_tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // barriers: w_full, w_empty [SW], x_full, x_empty [NX], a_full, a_empty [NA], done
    // 1024-byte aligned base for the swizzled operand buffers (the launch adds 1 KB of slack)
    const uint32_t raw = smem_addr(smem), bars = (raw + 1023) & ~1023u;
    uint8_t* base = smem + (bars - raw);
    const uint32_t w_full = bars, w_empty = w_full + 8 * kTcMaxRing, x_full = w_empty + 8 * kTcMaxRing,
                   x_empty = x_full + 8 * kTcMaxRing, a_full = x_empty + 8 * kTcMaxRing,
                   a_empty = a_full + 8 * kTcMaxRing, done = a_empty + 8 * kTcMaxRing;
    uint8_t* wring = base + 1024;
    uint8_t* xring = wring + a.SW * kTcWStage;
    const int xbytes = a.N * kTcChunk * 2;
    uint8_t* aring = xring + ((a.NX * xbytes + 1023) & ~1023);
    const uint8_t* W = a.w[blockIdx.z];
    const int m0 = blockIdx.x * kTcRows, t0 = m0 / 16;
    const int nchunk = a.K / kTcChunk;
    const int c0 = blockIdx.y * a.cps, c1 = min(c0 + a.cps, nchunk), nj = c1 - c0;  // c0 even
    // two accumulators (the A_hi and the A_lo products: independent MMA chains), N columns each
    const uint32_t ncols = 2 * a.N <= 32 ? 32u : 2 * a.N <= 64 ? 64u : 2 * a.N <= 128 ? 128u : 2 * a.N <= 256 ? 256u : 512u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < a.SW; ++i) {
            mbar_init(w_full + 8 * i, 1);
            mbar_init(w_empty + 8 * i, 8);  // the 8 dequant warps
        }
        for (int i = 0; i < a.NX; ++i) {
            mbar_init(x_full + 8 * i, 1);
            mbar_init(x_empty + 8 * i, 1);  // tcgen05.commit
        }
        for (int i = 0; i < a.NA; ++i) {
            mbar_init(a_full + 8 * i, 8);
            mbar_init(a_empty + 8 * i, 1);
        }
        mbar_init(done, 1);
        mbar_fence_init();
    }
    if (warp == 1) {  // TMEM columns for the accumulator (warp-wide)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool bad = false, timeout = false;

    if (warp == 0) {
        // ---- producers: lane 0 streams the weight groups, lane 1 the activation chunks, each
        // as far ahead as its own ring allows (one thread for both let a full activation ring
        // hold back the weight stream to two groups in flight)
        if (lane == 0) {
            // a stage: kTcGps consecutive groups of each of the 8 row tiles, one contiguous
            // copy per tile (the groups of a tile are adjacent in the tile-major layout)
            const int ng = nj / 2, ns = (ng + kTcGps - 1) / kTcGps;
            for (int i = 0; i < ns; ++i) {
                const int sw = i % a.SW, g = (c0 >> 1) + kTcGps * i, n = min(kTcGps, ng - kTcGps * i);
                if (i >= a.SW && !mbar_wait(w_empty + 8 * sw, ((i / a.SW) - 1) & 1)) {
                    timeout = true;
                    break;
                }
                mbar_arrive_expect_tx(w_full + 8 * sw, (uint32_t)(8 * n * kTcImg));
                for (int rt = 0; rt < 8; ++rt)
                    bulk_g2s(smem_addr(wring + sw * kTcWStage + rt * kTcGps * kTcImg),
                             W + (size_t)(t0 + rt) * a.tstride + (size_t)g * kTcImg, (uint32_t)(n * kTcImg),
                             w_full + 8 * sw);
            }
            // wait (bounded) until the last copies landed, so none writes after the CTA ends
            for (int i = ns - a.SW < 0 ? 0 : ns - a.SW; i < ns && !timeout; ++i)
                if (!mbar_wait(w_full + 8 * (i % a.SW), (i / a.SW) & 1)) timeout = true;
        } else if (lane == 1) {
            for (int j = 0; j < nj; ++j) {
                const int sx = j % a.NX;
                if (j >= a.NX && !mbar_wait(x_empty + 8 * sx, ((j / a.NX) - 1) & 1)) {
                    timeout = true;
                    break;
                }
                mbar_arrive_expect_tx(x_full + 8 * sx, (uint32_t)xbytes);
                bulk_g2s(smem_addr(xring + sx * xbytes), a.xc + (size_t)(c0 + j) * xbytes, (uint32_t)xbytes,
                         x_full + 8 * sx);
            }
            for (int j = nj - a.NX < 0 ? 0 : nj - a.NX; j < nj && !timeout; ++j)
                if (!mbar_wait(x_full + 8 * (j % a.NX), (j / a.NX) & 1)) timeout = true;
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(a.N >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
            for (int j = 0; j < nj && !timeout; ++j) {
                const int sa = j % a.NA, sx = j % a.NX;
                if (!mbar_wait(a_full + 8 * sa, (j / a.NA) & 1) || !mbar_wait(x_full + 8 * sx, (j / a.NX) & 1)) {
                    timeout = true;
                    break;
                }
                tc_fence_after();
                const uint32_t ahi = smem_addr(aring + sa * 2 * kTcABytes), alo = ahi + kTcABytes;
                const uint32_t xs = smem_addr(xring + sx * xbytes);
#pragma unroll
                for (int s = 0; s < kTcChunk / 16; ++s) {
                    tc_mma(tmem, tc_desc(ahi + 32 * s), tc_desc(xs + 32 * s), idesc, (j | s) != 0);
                    tc_mma(tmem + (uint32_t)a.N, tc_desc(alo + 32 * s), tc_desc(xs + 32 * s), idesc, (j | s) != 0);
                }
                tc_commit(a_empty + 8 * sa);
                tc_commit(x_empty + 8 * sx);
            }
            tc_commit(done);
        }
    } else {
        // ---- dequantisation: 256 threads, items (row r, piece t) x 2 per half-group; the
        // shared-memory offsets of a thread's items are the same for every chunk
        const int dt = threadIdx.x - 64;
        int cw[2], dwo[2], ao[2][4];
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const int item = dt + 256 * it, r = item >> 2, t = item & 3, rt = r >> 4, rr = r & 15;
            cw[it] = rt * (kTcGps * kTcImg / 4) + (rr * 4 + t) * 4;  // code words (+ group image + 256 h)
            dwo[it] = rt * (kTcGps * kTcImg / 4) + 512 + 2 * rr;      // d words (+ group image + h)
#pragma unroll
            for (int q = 0; q < 4; ++q) ao[it][q] = tc_canon(r, 32 * (q >> 1) + 16 * (q & 1) + 4 * t);
        }
        uint32_t dbits = 0;  // OR of the scales' f16 bits: bit 14 = a |d| >= 2 (127 d 2^8 past f16)
        for (int j = 0; j < nj && !timeout; ++j) {
            const int gl = j >> 1, i = gl / kTcGps, h = j & 1, sw = i % a.SW, sa = j % a.NA;
            const int gw = (gl % kTcGps) * (kTcImg / 4);  // the group's image inside each tile's run
            const bool stage_first = (j % (2 * kTcGps)) == 0, stage_last = (j % (2 * kTcGps)) == 2 * kTcGps - 1;
            if (stage_first && !mbar_wait(w_full + 8 * sw, (i / a.SW) & 1)) {
                timeout = true;
                break;
            }
            if (j >= a.NA && !mbar_wait(a_empty + 8 * sa, ((j / a.NA) - 1) & 1)) {
                timeout = true;
                break;
            }
            const uint32_t* ws = reinterpret_cast<const uint32_t*>(wring + sw * kTcWStage);
            uint8_t* ahi = aring + sa * 2 * kTcABytes;
            uint8_t* alo = ahi + kTcABytes;
            uint4 c[2];
            uint32_t dw[2];
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                c[it] = *reinterpret_cast<const uint4*>(ws + cw[it] + gw + h * 256);
                dw[it] = ws[dwo[it] + gw + h];  // f16 d of blocks 2h (low) and 2h + 1 (high)
            }
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                dbits |= dw[it];
                const __half2 dd = __hmul2(u32_as_h2(dw[it]), __float2half2_rn(kTcWScale));
                const __half2 d0 = __low2half2(dd), d1 = __high2half2(dd);
                const uint32_t words[4] = {c[it].x, c[it].y, c[it].z, c[it].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // k = 32 (q >> 1) + 16 (q & 1) + 4 t
                    uint2 hi, lo;
                    tc_dequant4(words[q], q < 2 ? d0 : d1, hi, lo);
                    *reinterpret_cast<uint2*>(ahi + ao[it][q]) = hi;
                    *reinterpret_cast<uint2*>(alo + ao[it][q]) = lo;
                }
            }
            // the MMA reads the operands through the async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(a_full + 8 * sa);
                if (stage_last || j == nj - 1) mbar_arrive(w_empty + 8 * sw);
            }
        }
        if (dbits & 0x40004000u) bad = true;
        // ---- epilogue: warps 2-5 read one TMEM lane quarter each
        if (warp < 6 && !timeout) {
            if (!mbar_wait(done, 0)) {
                timeout = true;
            } else {
                tc_fence_after();
                const int quarter = warp & 3, row = m0 + 32 * quarter + lane;
                const int Bp = a.N >> 1;
                float* out = a.out + ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * (size_t)a.B * a.M;
                for (int cb = 0; cb < Bp; cb += 8) {
                    float vh[8], vl[8], wh[8], wl[8];
                    const uint32_t base = tmem + ((uint32_t)(32 * quarter) << 16);
                    tc_ld8(base + cb, vh);
                    tc_ld8(base + Bp + cb, vl);
                    tc_ld8(base + a.N + cb, wh);  // the A_lo products
                    tc_ld8(base + a.N + Bp + cb, wl);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        vh[e] += wh[e];
                        vl[e] += wl[e];
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int t = cb + e;
                        if (t < a.B && row < a.M)
                            out[(size_t)t * a.M + row] = (vh[e] + vl[e] * (1.0f / 2048.0f)) * (1.0f / kTcWScale);
                    }
                }
            }
        }
    }
    if (bad && a.err) atomicOr(a.err, 1);
    if (timeout && a.err) atomicOr(a.err, 2);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// Activation rows -> the canonical B operand: row t < B of x (optionally RMS-normalised: x * inv
// * w for k < norm_len, 0 beyond; rms_norm, crates/hayai-cpu/src/attention.rs:142-147), split
// x = hi + lo * 2^-11 into rows t and Bp + t; rows [B, Bp) are zero.  Block (t, slice): row t,
// K elements [1024 slice, +1024), 4 consecutive elements per thread (one float4 in, one 8-byte
// store per half out).  K is a multiple of 128.
__global__ void __launch_bounds__(256) tc_prep_kernel(const float* __restrict__ x, int ldx, int B, int Bp, int K,
                                                      const float* __restrict__ norm_w, int norm_len, float eps,
                                                      uint8_t* __restrict__ xc, int* err) {
    __shared__ float s_red[8];
    const int t = blockIdx.x;
    const int N = 2 * Bp;
    const bool live = t < B;
    float inv = 1.0f;
    if (live && norm_w) {  // the whole row's sum of squares (every slice block recomputes it)
        float s = 0.f;
        const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)t * ldx);
        for (int c = threadIdx.x; c < (norm_len >> 2); c += blockDim.x) {
            const float4 v = x4[c];
            s += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
        }
        for (int k = (norm_len & ~3) + threadIdx.x; k < norm_len; k += blockDim.x) {
            const float v = x[(size_t)t * ldx + k];
            s += v * v;
        }
        s = warp_sum(s);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = s;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) tot += s_red[i];
        inv = 1.0f / sqrtf(tot / (float)norm_len + eps);
    }
    const int k = blockIdx.y * 1024 + 4 * threadIdx.x;
    if (k >= K) return;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (live) {
        const float4 a = *reinterpret_cast<const float4*>(x + (size_t)t * ldx + k);
        v[0] = a.x;
        v[1] = a.y;
        v[2] = a.z;
        v[3] = a.w;
        if (norm_w) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = k + j < norm_len ? v[j] * inv * norm_w[k + j] : 0.f;
        }
    }
    bool bad = false;
    __half hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (fabsf(v[j]) >= 65504.0f && isfinite(v[j])) bad = true;
        split_f16(v[j], hi[j], lo[j]);
    }
    uint8_t* chunk = xc + (size_t)(k / kTcChunk) * N * kTcChunk * 2;
    const int kk = k % kTcChunk;
    *reinterpret_cast<uint2*>(chunk + tc_canon(t, kk)) =
        make_uint2(h2_as_u32(__halves2half2(hi[0], hi[1])), h2_as_u32(__halves2half2(hi[2], hi[3])));
    *reinterpret_cast<uint2*>(chunk + tc_canon(Bp + t, kk)) =
        make_uint2(h2_as_u32(__halves2half2(lo[0], lo[1])), h2_as_u32(__halves2half2(lo[2], lo[3])));
    if (bad && err) atomicOr(err, 1);
}

// Outputs, 4 per thread: y[t][m] = [resid[t][m] +] sum over splits (in order) of the partials
// of matrix 0; with `gu`, h[t][m] = silu(sum g) * (sum u) over matrices 0 and 1.  M is a
// multiple of 128.
__global__ void tc_finish_kernel(const float* __restrict__ part, int splits, int B, int M, float* y, int ldy,
                                 const float* resid, int ldr, bool gu) {
    const int m4 = M >> 2;
    const int n4 = B * m4;
    const size_t n = (size_t)B * M;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const int t = i / m4, m = (i - t * m4) * 4;
        float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
        for (int s = 0; s < splits; ++s) {
            const float4 p = reinterpret_cast<const float4*>(part + (size_t)s * n)[i];
            s0.x += p.x;
            s0.y += p.y;
            s0.z += p.z;
            s0.w += p.w;
        }
        float o[4];
        if (gu) {
            for (int s = 0; s < splits; ++s) {
                const float4 p = reinterpret_cast<const float4*>(part + ((size_t)splits + s) * n)[i];
                s1.x += p.x;
                s1.y += p.y;
                s1.z += p.z;
                s1.w += p.w;
            }
            o[0] = silu_mul(s0.x, s1.x);
            o[1] = silu_mul(s0.y, s1.y);
            o[2] = silu_mul(s0.z, s1.z);
            o[3] = silu_mul(s0.w, s1.w);
        } else {
            o[0] = s0.x;
            o[1] = s0.y;
            o[2] = s0.z;
            o[3] = s0.w;
            if (resid) {  // may alias y: read, then written, here
#pragma unroll
                for (int j = 0; j < 4; ++j) o[j] = resid[(size_t)t * ldr + m + j] + o[j];
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) y[(size_t)t * ldy + m + j] = o[j];
    }
}

// ------------------------------------------------------------------ host side
static int tc_bp(int B) { return (B + 7) / 8 * 8; }

bool tc_gemm_supported(int type, int M, int K, int nvec) {
    return type == T_Q8_0 && nvec >= 8 && nvec <= 128 && M % kTcRows == 0 && K % 128 == 0 && M > 0 && K > 0;
}

// K splits: the count whose CTAs fill their last wave best (ties -> fewer splits), at least 4
// groups of 128 K per split.
static int tc_splits(int M, int K, int num_sms, int mats) {
    const int blocks = M / kTcRows * mats, groups = K / 128;
    int best = 1;
    double best_eff = 0.0;
    for (int s = 1; s <= 16 && groups / s >= 4; ++s) {
        const int cps = ((2 * groups + s - 1) / s + 1) & ~1;  // chunks per split, even
        const int real = (2 * groups + cps - 1) / cps;           // splits after rounding
        if (real != s) continue;
        const double waves = (double)blocks * s / num_sms;
        const double eff = waves / std::ceil(waves);
        if (eff > best_eff + 0.02) {
            best_eff = eff;
            best = s;
        }
    }
    return best;
}

size_t tc_workspace_bytes(int M, int K, int nvec, int num_sms, int mats) {
    const size_t N = 2 * (size_t)tc_bp(nvec);
    const size_t xc = (size_t)K * N * 2, part = (size_t)mats * tc_splits(M, K, num_sms, mats) * nvec * M * 4;
    return (xc + 255) / 256 * 256 + part;
}

// y = W x (+ resid) for nvec rows of x (gate/up: w2 != nullptr, y = h = silu(G x) * (U x) with
// x optionally RMS-normalised).  ws: tc_workspace_bytes(M, K, nvec, num_sms, 1 or 2) bytes.
cudaError_t launch_tc_gemm(const uint8_t* w, const uint8_t* w2, long long tstride, int M, int K, const float* x,
                           int ldx, int nvec, float* y, int ldy, const float* resid, int ldr, const float* norm_w,
                           int norm_len, float eps, void* ws, int* err, int num_sms, int smem_limit,
                           cudaStream_t stream) {
    const int mats = w2 ? 2 : 1;
    const int Bp = tc_bp(nvec), N = 2 * Bp;
    const int splits = tc_splits(M, K, num_sms, mats);
    uint8_t* xc = static_cast<uint8_t*>(ws);
    float* part = reinterpret_cast<float*>(xc + ((size_t)K * N * 2 + 255) / 256 * 256);
    tc_prep_kernel<<<dim3(Bp, (K + 1023) / 1024), 256, 0, stream>>>(x, ldx, nvec, Bp, K, norm_w, norm_len, eps, xc,
                                                                   err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    TcArgs a{};
    a.w[0] = w;
    a.w[1] = w2 ? w2 : w;
    a.tstride = tstride;
    a.M = M;
    a.K = K;
    a.xc = xc;
    a.N = N;
    a.B = nvec;
    const int nchunk = K / kTcChunk;
    a.cps = ((nchunk + splits - 1) / splits + 1) & ~1;
    a.out = part;
    a.err = err;
    // rings: what fits, operand buffers first
    const int xbytes = N * kTcChunk * 2;
    // The operand buffers bound the throughput: each makes a round trip dequant -> MMA ->
    // commit -> dequant of about 2 us, so they get the shared memory first.
    a.NA = 4;
    a.SW = 2;
    a.NX = 4;
    auto smem_of = [&](const TcArgs& t) {
        return 1024 + t.SW * kTcWStage + ((t.NX * xbytes + 1023) & ~1023) + t.NA * 2 * kTcABytes;
    };
    while (smem_of(a) > smem_limit - 2048 && a.NX > 2) --a.NX;
    while (smem_of(a) > smem_limit - 2048 && a.NA > 2) --a.NA;
    while (smem_of(a) > smem_limit - 2048 && a.SW > 1) --a.SW;
    if (smem_of(a) > smem_limit - 2048) return cudaErrorInvalidConfiguration;
    const int smem = smem_of(a) + 1024;  // slack for the 1024-byte alignment of the buffers
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || configured[dev] < smem) {
        e = cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev] = smem;
    }
    const dim3 grid(M / kTcRows, (nchunk + a.cps - 1) / a.cps, mats);
    tc_gemm_kernel<<<grid, kTcThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t n = (size_t)nvec * M / 4;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    tc_finish_kernel<<<blocks, 256, 0, stream>>>(part, (int)grid.y, nvec, M, y, ldy, resid, ldr, mats == 2);
    return cudaGetLastError();
}

}  // namespace hc
