// gemm_tc.cu -- batched quantized GEMV (B >= 8 activation rows) on the 5th-generation tensor
// cores, for Q8_0, Q4_K and Q6_K weights in the tile-major layout.
//
// Reference semantics: gemv_q8_0 (crates/hayai-model/src/quant.rs:598-615), gemv_q4_k
// (q4k.rs:206-256 with gemv_q4k_sub32 :10-32 and get_scale_min_k4 :34-43) and gemv_q6_k
// (q6k.rs:26-90) applied to every row of a batch, the multi-row case of
// execute_quant_gemv_batched (crates/hayai-opencl/src/orchestrator.rs:240-267, which loops over
// rows on the CPU path).
//
// Y[t][m] = sum_k W[m][k] x[t][k].  The quantization scales change every 16-32 elements and
// every row, so they cannot ride on a TMEM accumulator; instead every weight is dequantised in
// shared memory to its f32 value exactly as the reference forms it, scaled by 2^8 (exact), and
// split into two f16 operands w' = A_hi + A_lo:
//   Q8_0  w' = q d 2^8: A_hi = f16(w') (HMUL2), A_lo = w' - A_hi (one HFMA2, exact: q has 8
//         significant bits and d 11, so the remainder has at most 8);
//   Q4_K  w' = (q d1 - m1) 2^8 (one FFMA, the reference's single rounding of f d1 - m1v with
//         d1 = d sc, m1 = dmin m): A_hi = w' truncated to 11 significant bits, A_lo = f16(w' - A_hi);
//   Q6_K  w' = q (d sc) 2^8 (one FMUL, the reference's rounding): split as for Q4_K.
// The activations enter as two f16 columns per row, x = x_hi + x_lo * 2^-11 (rows [0, Bp) and
// [Bp, 2 Bp) of the B operand), so one tcgen05.mma with N = 2 Bp multiplies both, and
// D = A_hi X + A_lo X accumulates in f32 in TMEM (both products into one accumulator); the
// epilogue forms y = (D[:, t] + D[:, Bp + t] * 2^-11) * 2^-8.
//
// Persistent, stream-K: one CTA per SM walks a contiguous range of the work units (one weight
// image = 128 or 256 K of one 128-row block of one matrix, in the order row block, matrix, K),
// so the weight stream never pauses between row blocks.  A maximal run of units of one (row
// block, matrix) in a CTA is a segment: it accumulates in chains of at most kTcChainK K, each
// in one of two TMEM accumulator sets in turn, which the epilogue adds in order into the
// segment's partial-output slot; the finishing kernel adds a row block's slots in CTA order
// (deterministic), then SiLU(g) * u or the residual.  15 warps:
//   warp 0     weight producer: per unit one bulk copy per 16-row tile of the tile-major
//              layout (8 copies of one image);
//   warp 1     owns the TMEM columns; one elected lane issues the MMAs (4 K-steps x {hi, lo}
//              per 64-K chunk), tcgen05.commit frees the operand buffers and, at a chain's
//              end, hands its accumulator set to the epilogue;
//   warps 2-9  dequantise each 64-K chunk into the A_hi / A_lo operand buffers (K-major,
//              128-byte swizzle: rows of 128 B, 16-byte chunks XOR-permuted by row);
//   warps 10-13 the epilogue: one TMEM lane quarter each (tcgen05.ld), partial outputs out,
//              then the accumulator set is free again;
//   warp 14    activation producer: the 64-K chunks (prepared in the MMA's operand layout by
//              tc_prep_kernel), one copy each.  Not a second lane of warp 0: the two producers'
//              suspended mbarrier waits then held each other up (one third of the run time).
// TMEM operand form (TA, batches up to 64, the default): warps 2-9 dequantise straight into
// TMEM with tcgen05.st, and every hand-over (dequant -> MMA -> release) covers two 64-K chunks
// (the activation copies too).  One tcgen05.mma (M 128, N <= 64, K 16) takes ~60 cycles
// whatever N is (measured), and each hand-over adds fences, commits and barrier round trips:
// halving the hand-overs gained 29-36 %; doubling the dequantising warps lost 5 %.
// Every wait is bounded (~1 s; error bit 1), and the TMEM columns are freed on every path.
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "gemv_launch.h"

namespace hc {

constexpr int kTcRows = 128;               // output rows per CTA (MMA M)
constexpr int kTcChunk = 64;               // K per operand buffer
constexpr int kTcABytes = kTcRows * kTcChunk * 2;  // one f16 operand buffer (16 KB)
constexpr int kTcThreads = 480;            // 15 warps
constexpr int kTcMaxRing = 12;
static_assert(6 * 8 * kTcMaxRing + 32 <= 1024, "the mbarriers fit the 1 KB head of shared memory");
constexpr float kTcWScale = 256.f;         // w' = w * 2^8
// K elements per accumulator chain: the tensor core adds each MMA's products into its f32
// accumulator with a truncating (biased) alignment, so a chain over a whole row (up to 28672
// K here) drifts by up to ~1e-3 absolute at the 70B shapes.  A segment is therefore cut into
// chains of at most kTcChainK; the epilogue adds the chains of a segment in f32 (round to
// nearest), in order, into the segment's partial slot.
constexpr int kTcChainK = 1024;
// TMEM operand form: one hand-over (dequant -> MMA -> release) covers kTaKH 64-K chunks; a
// buffer is kTaBuf columns: A_hi of chunk k at [32k, 32k + 32), A_lo at kTaLo + 32k.
constexpr int kTaKH = 2, kTaLo = 32 * kTaKH, kTaBuf = 2 * kTaLo;
constexpr int kTaEsum = 64 * kTcRows * 4;  // the epilogue's segment sums (batches up to 64)

// Tile-block image of each format (repack.cu): bytes, K elements, images per weight stage
// (one: a stage is one work unit).
struct TcQ80 {
    static constexpr int kType = T_Q8_0, kImg = 2176, kImgK = 128, kGps = 1;
};
struct TcQ4K {
    static constexpr int kType = T_Q4_K, kImg = 2304, kImgK = 256, kGps = 1;
};
struct TcQ6K {
    static constexpr int kType = T_Q6_K, kImg = 3360, kImgK = 256, kGps = 1;
};
template <class F>
__host__ __device__ constexpr int tc_wstage() {  // the CTA's 8 row tiles x kGps images
    return 8 * F::kGps * F::kImg;
}

struct TcArgs {
    const uint8_t* w[2];  // tile-major matrices (the unit's matrix index picks one)
    long long tstride;    // bytes per 16-row tile
    int M, K;
    const uint8_t* xc;    // activations, canonical: [K / 64 chunks][N rows][64] f16
    int N, B;             // MMA N = 2 Bp (hi rows, then lo rows); real rows
    int mats, nimg;       // matrices (1, or 2 for gate/up); images per row block and matrix
    long long U;          // work units: (M / 128) * mats * nimg
    int slots;            // partial-output slots per (row block, matrix)
    int nsets;            // TMEM accumulator sets (2: the epilogue drains one while the other fills)
    float* out;           // partials [(row block, matrix)][slot][B][128]
    int* err;
    int SW, NX, NA;       // ring depths: weight units, activation chunks, operand buffers
};

// The CTA (of G) whose unit range [c U / G, (c + 1) U / G) holds unit u.
__host__ __device__ __forceinline__ int tc_owner(long long u, long long U, int G) {
    return (int)(((u + 1) * G - 1) / U);
}

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

// Registers of this thread -> consecutive 32-bit columns of its TMEM lane (lane = the warp's
// quarter base + thread; taddr carries the quarter's base lane in bits 31:16).
__device__ __forceinline__ void tc_st4(uint32_t taddr, const uint32_t (&r)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (+)= A B with A read from TMEM (128 lanes = rows, K packed two f16 per column), B from
// shared memory.
__device__ __forceinline__ void tc_mma_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
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

// Two f32 weights (already x 2^8) as (hi, lo) f16x2 words: hi = the value truncated to 11
// significant bits (exact in f16 for |w| in [2^-14, 65504)), lo = f16 of the exact remainder.
__device__ __forceinline__ void tc_split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const float ha = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
    const float hb = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
    hi = pack_h2(ha, hb);
    lo = pack_h2(a - ha, b - hb);
}

// Per-thread dequantisation of one 64-K chunk of the CTA's 128 rows (256 threads, dt = 0..255).
// init() fixes the thread's offsets (words inside a weight stage, bytes inside an operand
// buffer); chunk() reads the image at word offset `gw` of every tile run, chunk `sub` of it.
template <class F>
struct TcDq;

// Q8_0 image (2176 B, 128 K): [q0: (r,t) at 16(4r+t)][q1: at 1024 + 16(4r+t)][d: row r at
// 2048 + 8r]; word wi of piece (r,t) (q0: wi < 4, q1: wi - 4) = codes 16(wi & 1) + 4t..+3 of
// block wi / 2.  Items (row r, piece t) x 2 per thread; chunk h = blocks 2h, 2h + 1.
template <>
struct TcDq<TcQ80> {
    int cw[2], dwo[2], ao[2][4];
    uint32_t dbits = 0;  // OR of the scales' f16 bits: bit 14 = a |d| >= 2 (127 d 2^8 past f16)
    __device__ __forceinline__ void init(int dt) {
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const int item = dt + 256 * it, r = item >> 2, t = item & 3, rt = r >> 4, rr = r & 15;
            cw[it] = rt * (TcQ80::kGps * TcQ80::kImg / 4) + (rr * 4 + t) * 4;
            dwo[it] = rt * (TcQ80::kGps * TcQ80::kImg / 4) + 512 + 2 * rr;
#pragma unroll
            for (int q = 0; q < 4; ++q) ao[it][q] = tc_canon(r, 32 * (q >> 1) + 16 * (q & 1) + 4 * t);
        }
    }
    __device__ __forceinline__ void chunk(const uint32_t* ws, int h, uint8_t* ahi, uint8_t* alo) {
        uint4 c[2];
        uint32_t dw[2];
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            c[it] = *reinterpret_cast<const uint4*>(ws + cw[it] + h * 256);
            dw[it] = ws[dwo[it] + h];  // f16 d of blocks 2h (low) and 2h + 1 (high)
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
    }
    __device__ __forceinline__ bool bad() const { return (dbits & 0x40004000u) != 0; }
};

// Q4_K image (2304 B, 256 K): [hdr: row r at 16r = d, dmin, then 24 bits per chunk c at byte
// 4 + 3c: sc(2c) | sc(2c+1) << 6 | m(2c) << 12 | m(2c+1) << 18][q0: (r,t) at
// 256 + 16(4r+t) = qs bytes 32t..32t+15][q1: at 1280 + 16(4r+t) = qs bytes 32t+16..32t+31].
// qs byte 32c + l holds element 64c + l (low nibble, sub-block 2c) and 64c + 32 + l (high
// nibble, sub-block 2c + 1), so chunk c is piece t = c of every row.  Item = (row r, piece p):
// chunk elements 16p + 0..15 (low nibbles) and 32 + 16p + 0..15 (high nibbles).
template <>
struct TcDq<TcQ4K> {
    int hw, qw, ao[4];
    float big = 0.f;  // max over sub-blocks of 2^8 (|d1| 15 + |m1|): w' must stay below 65504
    __device__ __forceinline__ void init(int dt) {
        const int r = dt >> 1, p = dt & 1, rt = r >> 4, rr = r & 15;
        const int base = rt * (TcQ4K::kGps * TcQ4K::kImg / 4);
        hw = base + 4 * rr;
        qw = base + 64 + 16 * rr + 256 * p;
        ao[0] = tc_canon(r, 16 * p);
        ao[1] = tc_canon(r, 16 * p + 8);
        ao[2] = tc_canon(r, 32 + 16 * p);
        ao[3] = tc_canon(r, 40 + 16 * p);
    }
    __device__ __forceinline__ void chunk(const uint32_t* ws, int c, uint8_t* ahi, uint8_t* alo) {
        const uint4 hd = *reinterpret_cast<const uint4*>(ws + hw);
        const uint4 q = *reinterpret_cast<const uint4*>(ws + qw + 4 * c);
        // get_scale_min_k4 of sub-blocks 2c and 2c + 1 (regrouped by the repack)
        const uint32_t V = __funnelshift_r(c < 2 ? hd.y : (c == 2 ? hd.z : hd.w), c < 2 ? hd.z : hd.w, (24 * c) & 31);
        const float2 dd = __half22float2(u32_as_h2(hd.x));
        float d1[2], m1[2];
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const float sc = (float)((V >> (6 * s)) & 63u), mn = (float)((V >> (12 + 6 * s)) & 63u);
            d1[s] = (dd.x * sc) * kTcWScale;  // d1 = d sc, m1v = dmin m (exact)
            m1[s] = (dd.y * mn) * kTcWScale;
            big = fmaxf(big, fmaf(fabsf(d1[s]), 15.f, fabsf(m1[s])));
        }
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int s = 0; s < 2; ++s) {  // s = 0: low nibbles (k 16p + 4wi + b), 1: high (+32)
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                const uint32_t n = (s ? words[wi] >> 4 : words[wi]) & 0x0F0F0F0Fu;
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) v[b] = fmaf(u8_to_f32(n, b), d1[s], -m1[s]);
                tc_split2(v[0], v[1], hi[wi & 1 ? 2 : 0], lo[wi & 1 ? 2 : 0]);
                tc_split2(v[2], v[3], hi[wi & 1 ? 3 : 1], lo[wi & 1 ? 3 : 1]);
                if (wi & 1) {
                    const int o = ao[2 * s + (wi >> 1)];
                    *reinterpret_cast<uint4*>(ahi + o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4*>(alo + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                }
            }
        }
    }
    __device__ __forceinline__ bool bad() const { return !(big < 65504.f); }
};

// Q6_K image (3360 B, 256 K), lane-distributed (repack.cu): piece (r, t) of l0 / l1 / qh at
// 16(4r + t) in its 1024-B region holds ql bytes 64h + 16s + i / ql bytes 64h + 32 + 16s + i /
// qh bytes 32h + 16s + i (h = t >> 1, s = t & 1, i < 16); word t of row r's scales (3072 +
// 16r) holds sc[8h + s + 2q] in byte q; d of row r at 3328 + 2r.  Chunk c = 2h + nib of the
// super-block: elements 32qq + l of half h (q = 2 nib + qq, l = 16s + i), code
// nibble_nib(ql) | ((qh >> 2q) & 3) << 4, minus 32, scale byte q of word 2h + s
// (q6k.rs:35-55).  One item (row r, s) per thread: its 32 elements of every chunk.
template <>
struct TcDq<TcQ6K> {
    int lw, sw, dw, dsh, ao[2][4];
    float big = 0.f;  // max 2^8 |d sc| (|q| <= 32): w' must stay below 65504
    __device__ __forceinline__ void init(int dt) {
        const int r = dt >> 1, s = dt & 1, rt = r >> 4, rr = r & 15;
        const int base = rt * (TcQ6K::kGps * TcQ6K::kImg / 4);
        lw = base + 4 * (4 * rr + s);  // piece t = 2h + s: + 8h words
        sw = base + 768 + 4 * rr + s;  // word t: + 2h
        dw = base + 832 + (rr >> 1);
        dsh = 16 * (rr & 1);
#pragma unroll
        for (int qq = 0; qq < 2; ++qq)
#pragma unroll
            for (int k = 0; k < 4; ++k) ao[qq][k] = tc_canon(r, 32 * qq + 16 * s + 4 * k);
    }
    __device__ __forceinline__ void chunk(const uint32_t* ws, int c, uint8_t* ahi, uint8_t* alo) {
        const int h = c >> 1, nib = c & 1;
        const uint4 l0 = *reinterpret_cast<const uint4*>(ws + lw + 8 * h);
        const uint4 l1 = *reinterpret_cast<const uint4*>(ws + lw + 8 * h + 256);
        const uint4 qh = *reinterpret_cast<const uint4*>(ws + lw + 8 * h + 512);
        const uint32_t scw = ws[sw + 2 * h] ^ 0x80808080u;
        const float d = h2f((uint16_t)(ws[dw] >> dsh));
        const uint32_t Q[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
            const int q = 2 * nib + qq;
            const float ds = (d * s8_to_f32_flipped(scw, q)) * kTcWScale;  // (d sc) 2^8, exact
            big = fmaxf(big, fabsf(ds) * 32.f);
            const uint32_t L[4] = {qq ? l1.x : l0.x, qq ? l1.y : l0.y, qq ? l1.z : l0.z, qq ? l1.w : l0.w};
            const int hs = 2 * q;  // the 2 qh bits move to bits 4-5 of each byte
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t lo4 = (nib ? L[k] >> 4 : L[k]) & 0x0F0F0F0Fu;
                const uint32_t up = (hs <= 4 ? Q[k] << (4 - hs) : Q[k] >> (hs - 4)) & 0x30303030u;
                const uint32_t code = lo4 | up;
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    uint32_t u;  // code byte b as f32 (2^23 + code) by PRMT, minus 2^23 + 32
                    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(u) : "r"(code), "r"(0x4B000000u), "r"(0x7440u | b));
                    v[b] = (__uint_as_float(u) - 8388640.0f) * ds;
                }
                uint2 hi, lo;
                tc_split2(v[0], v[1], hi.x, lo.x);
                tc_split2(v[2], v[3], hi.y, lo.y);
                *reinterpret_cast<uint2*>(ahi + ao[qq][k]) = hi;
                *reinterpret_cast<uint2*>(alo + ao[qq][k]) = lo;
            }
        }
    }
    __device__ __forceinline__ bool bad() const { return !(big < 65504.f); }
};

// ---- dequantisers into TMEM operands (the TA form of the kernel).  Thread (row r, half jj)
// of the 8 dequantising warps: warp w covers TMEM lanes (= rows) 32 (w % 4) + lane, and the
// two warps of a lane quarter split each 64-K chunk's work in halves.  A chunk's operands are
// 32 columns of A_hi at tA and 32 of A_lo at tA + kTaLo; column n holds chunk elements 2n (low
// half) and 2n + 1.  chunk() writes the thread's columns with tcgen05.st (tA carries the
// quarter's base lane).
template <class F>
struct TcDqT;

// Q8_0: chunk h of an image = blocks 2h, 2h + 1 = region h (q0 / q1): row rr's 64 bytes at
// 1024 h + 64 rr, piece t = 16 bytes: word 2bb + hw = codes 16 hw + 4t..+3 of block 2h + bb.
// Thread jj reads pieces t = 2jj, 2jj + 1: chunk elements 32 bb + 16 hw + 4t + i, i.e. columns
// 16 bb + 8 hw + 4 jj + [0, 4).
template <>
struct TcDqT<TcQ80> {
    int pw, dwo, jj;
    uint32_t dbits = 0;
    __device__ __forceinline__ void init(int r, int j) {
        const int rt = r >> 4, rr = r & 15, base = rt * (TcQ80::kGps * TcQ80::kImg / 4);
        jj = j;
        pw = base + 16 * rr + 8 * j;  // piece 2jj of region 0
        dwo = base + 512 + 2 * rr;
    }
    __device__ __forceinline__ void chunk(const uint32_t* ws, int h, uint32_t tA) {
        const uint4 p0 = *reinterpret_cast<const uint4*>(ws + pw + 256 * h);
        const uint4 p1 = *reinterpret_cast<const uint4*>(ws + pw + 256 * h + 4);
        const uint32_t dw = ws[dwo + h];
        dbits |= dw;
        const __half2 dd = __hmul2(u32_as_h2(dw), __float2half2_rn(kTcWScale));
        const __half2 d0 = __low2half2(dd), d1 = __high2half2(dd);
        const uint32_t w0[4] = {p0.x, p0.y, p0.z, p0.w}, w1[4] = {p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // g = 2 bb + hw
            uint2 h0, l0, h1, l1;
            tc_dequant4(w0[g], g < 2 ? d0 : d1, h0, l0);
            tc_dequant4(w1[g], g < 2 ? d0 : d1, h1, l1);
            const uint32_t hv[4] = {h0.x, h0.y, h1.x, h1.y}, lv[4] = {l0.x, l0.y, l1.x, l1.y};
            const uint32_t col = 16 * (g >> 1) + 8 * (g & 1) + 4 * jj;
            tc_st4(tA + col, hv);
            tc_st4(tA + kTaLo + col, lv);
        }
    }
    __device__ __forceinline__ bool bad() const { return (dbits & 0x40004000u) != 0; }
};

// Q4_K: chunk c = qs bytes 32c..32c+31 of the super-block; thread jj reads piece q_jj of
// (rr, c) = bytes 32c + 16jj + [0, 16): low nibbles are chunk elements 16jj + i (sub-block 2c,
// columns 8jj + i/2), high nibbles 32 + 16jj + i (sub-block 2c + 1, columns 16 + 8jj + i/2).
template <>
struct TcDqT<TcQ4K> {
    int hw, qw, jj;
    float big = 0.f;
    __device__ __forceinline__ void init(int r, int j) {
        const int rt = r >> 4, rr = r & 15, base = rt * (TcQ4K::kGps * TcQ4K::kImg / 4);
        jj = j;
        hw = base + 4 * rr;
        qw = base + 64 + 16 * rr + 256 * j;
    }
    __device__ __forceinline__ void chunk(const uint32_t* ws, int c, uint32_t tA) {
        const uint4 hd = *reinterpret_cast<const uint4*>(ws + hw);
        const uint4 q = *reinterpret_cast<const uint4*>(ws + qw + 4 * c);
        const uint32_t V = __funnelshift_r(c < 2 ? hd.y : (c == 2 ? hd.z : hd.w), c < 2 ? hd.z : hd.w, (24 * c) & 31);
        const float2 dd = __half22float2(u32_as_h2(hd.x));
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const float sc = (float)((V >> (6 * s)) & 63u), mn = (float)((V >> (12 + 6 * s)) & 63u);
            const float d1 = (dd.x * sc) * kTcWScale, m1 = (dd.y * mn) * kTcWScale;
            big = fmaxf(big, fmaf(fabsf(d1), 15.f, fabsf(m1)));
            uint32_t hv[8], lv[8];
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                const uint32_t n = (s ? words[wi] >> 4 : words[wi]) & 0x0F0F0F0Fu;
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) v[b] = fmaf(u8_to_f32(n, b), d1, -m1);
                tc_split2(v[0], v[1], hv[2 * wi], lv[2 * wi]);
                tc_split2(v[2], v[3], hv[2 * wi + 1], lv[2 * wi + 1]);
            }
            const uint32_t col = 16 * s + 8 * jj;
            tc_st8(tA + col, hv);
            tc_st8(tA + kTaLo + col, lv);
        }
    }
    __device__ __forceinline__ bool bad() const { return !(big < 65504.f); }
};

// Q6_K (lane-distributed image): thread jj = s takes the pieces of lane t = 2h + s (ql l0 / l1,
// qh, its scale word); chunk c = 2h + nib covers groups q = 2 nib + qq, elements 32 qq + 16 s + i
// (columns 16 qq + 8 s + i/2).  The pieces serve both chunks of a half: loaded at nib = 0.
template <>
struct TcDqT<TcQ6K> {
    int lw, sw, dw, dsh, jj;
    uint4 l0, l1, qh;
    uint32_t scw = 0;
    float d = 0.f, big = 0.f;
    __device__ __forceinline__ void init(int r, int j) {
        const int rt = r >> 4, rr = r & 15, base = rt * (TcQ6K::kGps * TcQ6K::kImg / 4);
        jj = j;
        lw = base + 4 * (4 * rr + j);  // piece t = 2h + s: + 8h words
        sw = base + 768 + 4 * rr + j;  // word t: + 2h
        dw = base + 832 + (rr >> 1);
        dsh = 16 * (rr & 1);
    }
    __device__ __forceinline__ void chunk(const uint32_t* ws, int c, uint32_t tA) {
        const int h = c >> 1, nib = c & 1;
        if (nib == 0) {
            l0 = *reinterpret_cast<const uint4*>(ws + lw + 8 * h);
            l1 = *reinterpret_cast<const uint4*>(ws + lw + 8 * h + 256);
            qh = *reinterpret_cast<const uint4*>(ws + lw + 8 * h + 512);
            scw = ws[sw + 2 * h] ^ 0x80808080u;
            d = h2f((uint16_t)(ws[dw] >> dsh));
        }
        const uint32_t Q[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
            const int q = 2 * nib + qq;
            const float ds = (d * s8_to_f32_flipped(scw, q)) * kTcWScale;
            big = fmaxf(big, fabsf(ds) * 32.f);
            const uint32_t L[4] = {qq ? l1.x : l0.x, qq ? l1.y : l0.y, qq ? l1.z : l0.z, qq ? l1.w : l0.w};
            const int hs = 2 * q;
            uint32_t hv[8], lv[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t lo4 = (nib ? L[k] >> 4 : L[k]) & 0x0F0F0F0Fu;
                const uint32_t up = (hs <= 4 ? Q[k] << (4 - hs) : Q[k] >> (hs - 4)) & 0x30303030u;
                const uint32_t code = lo4 | up;
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    uint32_t u;
                    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(u) : "r"(code), "r"(0x4B000000u), "r"(0x7440u | b));
                    v[b] = (__uint_as_float(u) - 8388640.0f) * ds;
                }
                tc_split2(v[0], v[1], hv[2 * k], lv[2 * k]);
                tc_split2(v[2], v[3], hv[2 * k + 1], lv[2 * k + 1]);
            }
            const uint32_t col = 16 * qq + 8 * jj;
            tc_st8(tA + col, hv);
            tc_st8(tA + kTaLo + col, lv);
        }
    }
    __device__ __forceinline__ bool bad() const { return !(big < 65504.f); }
};

template <class F, bool TA>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(TcArgs a) {
    constexpr int CPI = F::kImgK / kTcChunk;  // chunks per image (= per unit)
    constexpr int KH = TA ? kTaKH : 1;         // chunks per hand-over
    constexpr int CHU = kTcChainK / F::kImgK;  // units per accumulator chain
    static_assert(CPI % KH == 0, "a hand-over stays inside one unit");
    static_assert(kTcChainK % F::kImgK == 0, "chains are whole units");
    constexpr int WST = tc_wstage<F>();
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint32_t s_tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const long long u0 = (long long)c * a.U / G, u1 = (long long)(c + 1) * a.U / G;
    if (u0 >= u1) return;  // (no TMEM, no barriers used yet)
    const int nu = (int)(u1 - u0), nj = nu * CPI, nh = nj / KH;
    // barriers: w_full, w_empty [SW], x_full, x_empty [NX], a_full, a_empty [NA],
    // acc_full, acc_empty [2]; 1024-byte aligned base for the swizzled operand buffers (the
    // launch adds 1 KB of slack)
    const uint32_t raw = smem_addr(smem), bars = (raw + 1023) & ~1023u;
    uint8_t* base = smem + (bars - raw);
    const uint32_t w_full = bars, w_empty = w_full + 8 * kTcMaxRing, x_full = w_empty + 8 * kTcMaxRing,
                   x_empty = x_full + 8 * kTcMaxRing, a_full = x_empty + 8 * kTcMaxRing,
                   a_empty = a_full + 8 * kTcMaxRing, acc_full = a_empty + 8 * kTcMaxRing, acc_empty = acc_full + 16;
    uint8_t* wring = base + 1024;
    uint8_t* xring = wring + ((a.SW * WST + 1023) & ~1023);
    const int xbytes = a.N * kTcChunk * 2, xslot = KH * xbytes;  // one chunk; one hand-over
    // the smem operand form's operand buffers; the TA form's epilogue sums
    uint8_t* aring = xring + ((a.NX * xslot + 1023) & ~1023);
    // accumulator set s: columns [s N, (s + 1) N), the A_hi and the A_lo products added into
    // one accumulator (a chain is short, see kTcChainK); in the TA form the NA operand buffers
    // follow (kTaBuf columns each)
    const int accW = a.N;
    const uint32_t accC = (uint32_t)(a.nsets * accW);
    const uint32_t need = accC + (TA ? (uint32_t)kTaBuf * (uint32_t)a.NA : 0u);
    const uint32_t ncols = need <= 32 ? 32u : need <= 64 ? 64u : need <= 128 ? 128u : need <= 256 ? 256u : 512u;

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
        for (int i = 0; i < 2; ++i) {
            mbar_init(acc_full + 8 * i, 1);   // tcgen05.commit at an accumulator chain's end
            mbar_init(acc_empty + 8 * i, 4);  // the 4 epilogue warps
        }
        mbar_fence_init();
    }
    if (warp == 1) {  // TMEM columns for the accumulators (warp-wide)
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

    if (warp == 0 || warp == 14) {
        // ---- producers, each as far ahead as its own ring allows: warp 0 the weight units,
        // warp 14 the activation chunks
        if (warp == 0 && lane == 0) {
            for (int i = 0; i < nu; ++i) {
                const long long u = u0 + i;
                const int run = (int)(u / a.nimg), img = (int)(u % a.nimg), rb = run / a.mats, z = run % a.mats;
                const int sw = i % a.SW;
                if (i >= a.SW && !mbar_wait(w_empty + 8 * sw, ((i / a.SW) - 1) & 1)) {
                    timeout = true;
                    break;
                }
                mbar_arrive_expect_tx(w_full + 8 * sw, (uint32_t)(8 * F::kImg));
                // (a select, not a.w[z]: a runtime index into the parameter struct makes the
                // compiler copy the whole struct to local memory)
                const uint8_t* W = (z ? a.w[1] : a.w[0]) + (size_t)rb * 8 * a.tstride + (size_t)img * F::kImg;
                for (int rt = 0; rt < 8; ++rt)
                    bulk_g2s(smem_addr(wring + sw * WST + rt * F::kImg), W + (size_t)rt * a.tstride,
                             (uint32_t)F::kImg, w_full + 8 * sw);
            }
            // wait (bounded) until the last copies landed, so none writes after the CTA ends
            for (int i = nu - a.SW < 0 ? 0 : nu - a.SW; i < nu && !timeout; ++i)
                if (!mbar_wait(w_full + 8 * (i % a.SW), (i / a.SW) & 1)) timeout = true;
        } else if (warp == 14 && lane == 0) {
            for (int h = 0; h < nh; ++h) {  // the hand-over's KH chunks are adjacent in K
                const int j = h * KH, sx = h % a.NX;
                const int kc = (int)((u0 + j / CPI) % a.nimg) * CPI + j % CPI;  // the first chunk's K index
                if (h >= a.NX && !mbar_wait(x_empty + 8 * sx, ((h / a.NX) - 1) & 1)) {
                    timeout = true;
                    break;
                }
                mbar_arrive_expect_tx(x_full + 8 * sx, (uint32_t)xslot);
                bulk_g2s(smem_addr(xring + sx * xslot), a.xc + (size_t)kc * xbytes, (uint32_t)xslot,
                         x_full + 8 * sx);
            }
            for (int h = nh - a.NX < 0 ? 0 : nh - a.NX; h < nh && !timeout; ++h)
                if (!mbar_wait(x_full + 8 * (h % a.NX), (h / a.NX) & 1)) timeout = true;
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(a.N >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
            int seg = -1;
            uint32_t acc = 0;
            for (int h = 0; h < nh && !timeout; ++h) {
                const int j = h * KH;
                const long long u = u0 + j / CPI;
                const int sub = j % CPI, img = (int)(u % a.nimg);
                const bool first = sub == 0 && (img % CHU == 0 || u == u0);
                const bool last = sub + KH - 1 == CPI - 1 && (img % CHU == CHU - 1 || img == a.nimg - 1 || u == u1 - 1);
                if (first) {
                    ++seg;
                    const int s = seg % a.nsets;
                    acc = tmem + (uint32_t)(s * accW);
                    // the set's previous chain must have been read out
                    if (seg >= a.nsets && !mbar_wait(acc_empty + 8 * s, ((seg / a.nsets) - 1) & 1)) {
                        timeout = true;
                        break;
                    }
                }
                const int sa = h % a.NA, sx = h % a.NX;
                if (!mbar_wait(a_full + 8 * sa, (h / a.NA) & 1) || !mbar_wait(x_full + 8 * sx, (h / a.NX) & 1)) {
                    timeout = true;
                    break;
                }
                tc_fence_after();
                const uint32_t xs = smem_addr(xring + sx * xslot);
                if constexpr (TA) {
                    const uint32_t at = tmem + accC + (uint32_t)kTaBuf * (uint32_t)sa;  // lane 0, the buffer
#pragma unroll
                    for (int k = 0; k < KH; ++k)
#pragma unroll
                        for (int ks = 0; ks < kTcChunk / 16; ++ks) {
                            const uint32_t on = (first && k == 0 && ks == 0) ? 0u : 1u;
                            const uint64_t bd = tc_desc(xs + (uint32_t)(k * xbytes) + 32 * ks);
                            tc_mma_ta(acc, at + 32 * k + 8 * ks, bd, idesc, on);
                            tc_mma_ta(acc, at + kTaLo + 32 * k + 8 * ks, bd, idesc, 1u);
                        }
                } else {
                    const uint32_t ahi = smem_addr(aring + sa * 2 * kTcABytes), alo = ahi + kTcABytes;
#pragma unroll
                    for (int ks = 0; ks < kTcChunk / 16; ++ks) {
                        const uint32_t on = (first && ks == 0) ? 0u : 1u;
                        tc_mma(acc, tc_desc(ahi + 32 * ks), tc_desc(xs + 32 * ks), idesc, on);
                        tc_mma(acc, tc_desc(alo + 32 * ks), tc_desc(xs + 32 * ks), idesc, 1u);
                    }
                }
                tc_commit(a_empty + 8 * sa);
                tc_commit(x_empty + 8 * sx);
                if (last) tc_commit(acc_full + 8 * (seg % a.nsets));
            }
        }
    } else if (warp < 10 && TA) {
        // ---- dequantisation into TMEM operand buffers: warp w writes lanes 32 (w % 4) + lane
        const int quarter = warp & 3;
        TcDqT<F> dq;
        dq.init(32 * quarter + lane, (warp - 2) >> 2);
        const uint32_t tq = tmem + ((uint32_t)(32 * quarter) << 16) + accC;
        for (int h = 0; h < nh && !timeout; ++h) {
            const int j = h * KH, i = j / CPI, sub = j % CPI, sw = i % a.SW, sa = h % a.NA;
            if (sub == 0 && !mbar_wait(w_full + 8 * sw, (i / a.SW) & 1)) {
                timeout = true;
                break;
            }
            if (h >= a.NA && !mbar_wait(a_empty + 8 * sa, ((h / a.NA) - 1) & 1)) {
                timeout = true;
                break;
            }
            tc_fence_after();  // the MMAs that read this buffer have completed
#pragma unroll
            for (int k = 0; k < KH; ++k)
                dq.chunk(reinterpret_cast<const uint32_t*>(wring + sw * WST), sub + k,
                         tq + (uint32_t)kTaBuf * (uint32_t)sa + 32u * (uint32_t)k);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(a_full + 8 * sa);
                if (sub + KH - 1 == CPI - 1) mbar_arrive(w_empty + 8 * sw);
            }
        }
        bad = dq.bad();
    } else if (warp < 10) {
        // ---- dequantisation: 256 threads; a thread's shared-memory offsets are the same for
        // every chunk
        TcDq<F> dq;
        dq.init(threadIdx.x - 64);
        for (int j = 0; j < nj && !timeout; ++j) {
            const int i = j / CPI, sub = j % CPI, sw = i % a.SW, sa = j % a.NA;
            if (sub == 0 && !mbar_wait(w_full + 8 * sw, (i / a.SW) & 1)) {
                timeout = true;
                break;
            }
            if (j >= a.NA && !mbar_wait(a_empty + 8 * sa, ((j / a.NA) - 1) & 1)) {
                timeout = true;
                break;
            }
            uint8_t* ahi = aring + sa * 2 * kTcABytes;
            dq.chunk(reinterpret_cast<const uint32_t*>(wring + sw * WST), sub, ahi, ahi + kTcABytes);
            // the MMA reads the operands through the async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(a_full + 8 * sa);
                if (sub == CPI - 1) mbar_arrive(w_empty + 8 * sw);
            }
        }
        bad = dq.bad();
    } else {
        // ---- epilogue: warps 10-13 read TMEM lane quarters 2, 3, 0, 1 (warp % 4)
        const int quarter = warp & 3, row = 32 * quarter + lane, Bp = a.N >> 1;
        float* esum = reinterpret_cast<float*>(aring);  // TA form: the segment sums [64][128]
        int seg = 0;  // accumulator chains so far
        for (long long u = u0; u < u1 && !timeout; ++seg) {
            const int run = (int)(u / a.nimg), img = (int)(u % a.nimg);
            long long ue = u - img % CHU + CHU;  // the chain ends at the next CHU boundary,
            if (ue > (long long)(run + 1) * a.nimg) ue = (long long)(run + 1) * a.nimg;  // the run's end
            if (ue > u1) ue = u1;                                                          // or the CTA's
            const bool chain0 = img == 0 || u == u0;  // the segment's first chain stores, the others add
            const int s = seg % a.nsets;
            if (!mbar_wait(acc_full + 8 * s, (seg / a.nsets) & 1)) {
                timeout = true;
                break;
            }
            tc_fence_after();
            const int slot = c - tc_owner((long long)run * a.nimg, a.U, G);
            float* out = a.out + ((size_t)run * a.slots + slot) * (size_t)a.B * kTcRows;
            const uint32_t tb = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(s * accW);
            if constexpr (TA) {
                // Bp <= 64: the row's sums over the segment's chains collect in shared memory
                // ([t][row]: a warp's lanes hit consecutive words), and the set is released as
                // soon as it has been read (with one accumulator set the next chain's MMAs wait
                // only for these TMEM loads)
                for (int cb = 0; cb < Bp; cb += 8) {
                    float vh[8], vl[8];
                    tc_ld8(tb + cb, vh);       // A x_hi
                    tc_ld8(tb + Bp + cb, vl);  // A x_lo
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float v = (vh[e] + vl[e] * (1.0f / 2048.0f)) * (1.0f / kTcWScale);
                        float* o = esum + (cb + e) * kTcRows + row;
                        *o = chain0 ? v : *o + v;
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty + 8 * s);
                if (ue == u1 || ue == (long long)(run + 1) * a.nimg) {  // the segment's last chain
                    for (int t = 0; t < a.B; ++t) out[(size_t)t * kTcRows + row] = esum[t * kTcRows + row];
                }
            } else {
                for (int cb = 0; cb < Bp; cb += 8) {
                    float vh[8], vl[8];
                    tc_ld8(tb + cb, vh);       // A x_hi
                    tc_ld8(tb + Bp + cb, vl);  // A x_lo
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int t = cb + e;
                        if (t < a.B) {
                            const float v = (vh[e] + vl[e] * (1.0f / 2048.0f)) * (1.0f / kTcWScale);
                            float* o = out + (size_t)t * kTcRows + row;  // (this thread's own earlier store)
                            *o = chain0 ? v : *o + v;
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty + 8 * s);
            }
            u = ue;
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

// Outputs, 4 per thread: y[t][m] = [resid[t][m] +] the sum over a row block's partial slots
// (CTA order) of matrix 0; with `gu`, h[t][m] = silu(sum g) * (sum u) over matrices 0 and 1.
// M is a multiple of 128; the slots of (row block, matrix) run r are those of the CTAs that
// own its first through last unit.
__global__ void tc_finish_kernel(const float* __restrict__ part, long long U, int G, int nimg, int slots, int B, int M,
                                 float* y, int ldy, const float* resid, int ldr, bool gu) {
    const int m4 = M >> 2;
    const int n4 = B * m4;
    const int mats = gu ? 2 : 1;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const int t = i / m4, m = (i - t * m4) * 4, rb = m / kTcRows, row = m % kTcRows;
        float4 sum[2];
        for (int z = 0; z < mats; ++z) {
            const int run = rb * mats + z;
            const int cf = tc_owner((long long)run * nimg, U, G), cl = tc_owner((long long)(run + 1) * nimg - 1, U, G);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j <= cl - cf; ++j) {
                const float4 p =
                    *reinterpret_cast<const float4*>(part + (((size_t)run * slots + j) * B + t) * kTcRows + row);
                acc.x += p.x;
                acc.y += p.y;
                acc.z += p.z;
                acc.w += p.w;
            }
            sum[z] = acc;
        }
        float o[4];
        if (gu) {
            o[0] = silu_mul(sum[0].x, sum[1].x);
            o[1] = silu_mul(sum[0].y, sum[1].y);
            o[2] = silu_mul(sum[0].z, sum[1].z);
            o[3] = silu_mul(sum[0].w, sum[1].w);
        } else {
            o[0] = sum[0].x;
            o[1] = sum[0].y;
            o[2] = sum[0].z;
            o[3] = sum[0].w;
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
static int tc_cpi(int type) { return type == T_Q8_0 ? TcQ80::kImgK / kTcChunk : TcQ4K::kImgK / kTcChunk; }

// From 8 rows for Q4_K / Q6_K and 9 for Q8_0: below that the mma.sync GEMV (one weight pass per
// 4 rows, cheaper per pass for Q8_0) is as fast or faster (measured on the Llama-3-8B FFN shapes).
bool tc_gemm_supported(int type, int M, int K, int nvec) {
    if (type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K) return false;
    const int min_rows = type == T_Q8_0 ? 9 : 8;
    return nvec >= min_rows && nvec <= 128 && M > 0 && K > 0 && M % kTcRows == 0 &&
           K % (kTcChunk * tc_cpi(type)) == 0;
}

// The stream-K partition of an M x K launch over min(num_sms, U) CTAs.
struct TcPlan {
    int nimg, mats, G, slots;
    long long U;
};

static TcPlan tc_plan(int type, int M, int K, int num_sms, int mats) {
    TcPlan p{};
    p.nimg = K / (kTcChunk * tc_cpi(type));
    p.mats = mats;
    p.U = (long long)(M / kTcRows) * mats * p.nimg;
    p.G = (int)(p.U < num_sms ? p.U : num_sms);
    p.slots = 1;
    for (long long r = 0; r < p.U / p.nimg; ++r) {
        const int n = tc_owner((r + 1) * p.nimg - 1, p.U, p.G) - tc_owner(r * p.nimg, p.U, p.G) + 1;
        p.slots = n > p.slots ? n : p.slots;
    }
    return p;
}

size_t tc_workspace_bytes(int type, int M, int K, int nvec, int num_sms, int mats) {
    const TcPlan p = tc_plan(type, M, K, num_sms, mats);
    const size_t N = 2 * (size_t)tc_bp(nvec);
    const size_t xc = (size_t)K * N * 2;
    const size_t part = (size_t)(M / kTcRows) * mats * p.slots * nvec * kTcRows * 4;
    return (xc + 255) / 256 * 256 + part;
}

// The TA form (operands dequantised into TMEM; shared memory holds only the weight and
// activation rings) when the accumulators leave room for four 64-column operand buffers:
// N <= 128 (batches up to 64).  HAYAI_TC_TMEM_A=0 keeps the shared-memory operand form.
static bool tc_use_ta(int N) {
    static const bool on = [] {
        const char* v = std::getenv("HAYAI_TC_TMEM_A");
        return !(v && v[0] == '0');
    }();
    return on && N <= 128;
}

template <class F>
static cudaError_t tc_launch_ta(TcArgs a, int G, int smem_limit, cudaStream_t stream) {
    constexpr int WST = tc_wstage<F>();
    const int xbytes = a.N * kTcChunk * 2;
    // three operand buffers, and two accumulator sets (N columns each: the epilogue drains
    // one while the other fills) where TMEM holds them beside (N <= 64), else one (the
    // epilogue then releases it right after its TMEM loads)
    a.NA = 3;
    a.nsets = 2 * a.N + kTaBuf * 3 <= 512 ? 2 : 1;
    a.NX = 4;
    auto smem_of = [&](const TcArgs& t) {
        return 1024 + ((t.SW * WST + 1023) & ~1023) + ((t.NX * kTaKH * xbytes + 1023) & ~1023) + kTaEsum;
    };
    a.SW = kTcMaxRing;
    while (smem_of(a) > smem_limit - 2048 && a.SW > 2) --a.SW;
    if (smem_of(a) > smem_limit - 2048) return cudaErrorInvalidConfiguration;
    const int smem = smem_of(a) + 1024;
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || configured[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<F, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev] = smem;
    }
    tc_gemm_kernel<F, true><<<G, kTcThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

// Ring depths that fit, operand buffers first, and the kernel's dynamic shared memory.
template <class F>
static cudaError_t tc_launch_kernel(TcArgs a, int G, int smem_limit, cudaStream_t stream) {
    if (tc_use_ta(a.N)) return tc_launch_ta<F>(a, G, smem_limit, stream);
    constexpr int WST = tc_wstage<F>();
    const int xbytes = a.N * kTcChunk * 2;
    // The operand buffers take the shared memory first (each makes a round trip dequant ->
    // MMA -> commit -> dequant); the weight ring keeps about 64 KB in flight.
    a.NA = 4;
    a.SW = 70000 / WST > 2 ? (70000 / WST < kTcMaxRing ? 70000 / WST : kTcMaxRing) : 2;
    a.NX = 4;
    auto smem_of = [&](const TcArgs& t) {
        return 1024 + ((t.SW * WST + 1023) & ~1023) + ((t.NX * xbytes + 1023) & ~1023) + t.NA * 2 * kTcABytes;
    };
    while (smem_of(a) > smem_limit - 2048 && a.NX > 2) --a.NX;
    while (smem_of(a) > smem_limit - 2048 && a.NA > 2) --a.NA;
    while (smem_of(a) > smem_limit - 2048 && a.SW > 2) --a.SW;
    if (smem_of(a) > smem_limit - 2048) return cudaErrorInvalidConfiguration;
    const int smem = smem_of(a) + 1024;  // slack for the 1024-byte alignment of the buffers
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || configured[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<F, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev] = smem;
    }
    tc_gemm_kernel<F, false><<<G, kTcThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

// y = W x (+ resid) for nvec rows of x (gate/up: w2 != nullptr, y = h = silu(G x) * (U x) with
// x optionally RMS-normalised).  ws: tc_workspace_bytes(type, M, K, nvec, num_sms, 1 or 2) bytes.
cudaError_t launch_tc_gemm(int type, const uint8_t* w, const uint8_t* w2, long long tstride, int M, int K,
                           const float* x, int ldx, int nvec, float* y, int ldy, const float* resid, int ldr,
                           const float* norm_w, int norm_len, float eps, void* ws, int* err, int num_sms,
                           int smem_limit, cudaStream_t stream) {
    if (!tc_gemm_supported(type, M, K, nvec)) return cudaErrorInvalidValue;
    const int mats = w2 ? 2 : 1;
    const int Bp = tc_bp(nvec), N = 2 * Bp;
    const TcPlan p = tc_plan(type, M, K, num_sms, mats);
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
    a.mats = mats;
    a.nimg = p.nimg;
    a.U = p.U;
    a.slots = p.slots;
    a.nsets = 2;  // 2 N <= 512 TMEM columns: N <= 256
    a.out = part;
    a.err = err;
    switch (type) {
        case T_Q8_0: e = tc_launch_kernel<TcQ80>(a, p.G, smem_limit, stream); break;
        case T_Q4_K: e = tc_launch_kernel<TcQ4K>(a, p.G, smem_limit, stream); break;
        default: e = tc_launch_kernel<TcQ6K>(a, p.G, smem_limit, stream); break;
    }
    if (e != cudaSuccess) return e;
    const size_t n = (size_t)nvec * M / 4;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    tc_finish_kernel<<<blocks, 256, 0, stream>>>(part, p.U, p.G, p.nimg, p.slots, nvec, M, y, ldy, resid, ldr,
                                                 mats == 2);
    return cudaGetLastError();
}

}  // namespace hc
