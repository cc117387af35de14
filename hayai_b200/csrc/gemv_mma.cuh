// gemv_mma.cuh -- batch-1..4 quantized GEMV on tensor-core tiles (sm_100a).
//
// y[v][r] = resid[v][r] + sum_k W[r][k] * x[v][k]   for the packed formats Q4_K, Q6_K, Q8_0.
//
// Design (one warp = one 16-row tile over a range of super-blocks):
//  * Weights are dequantized in registers straight into the A fragment of
//    mma.m16n8k16 (f16 in, f32 accumulate).  Integer codes are exact in f16.
//    Q4_K and Q6_K are lane-distributed (each lane's k-slots belong to its own
//    sub-blocks / scale groups, so an accumulator column holds one group) and
//    apply their scales once per group in f32; Q8_0 applies its scale per MMA.
//  * Activations are split as x = hi + lo * 2^-11 (both f16), occupying two
//    columns of the B operand, so the tensor-core product carries ~22 bits of
//    x -- enough for the reference's f32 contract (rel-L2 <= 1e-4).  Columns
//    2v / 2v+1 hold vector v, so up to 4 vectors share one MMA for free.
//  * The B fragments of the whole K range are built once per CTA into shared
//    memory in exactly the order the lanes consume them (one LDS.64 per MMA).
//  * CTAs are persistent; the warps of a CTA split K of the same row tile and
//    reduce through shared memory, so each output is written once (no atomics).
#pragma once

#include "common.cuh"

namespace hc {

// Layout of the per-CTA shared memory: [xt table][zero block][Sx (Q4_K)][reduction]
struct GemvSmem {
    int table_bytes;
    int zero_bytes;  // one zeroed block of table entries (B fragments of empty columns)
    int sx_bytes;
    int red_bytes;
    __host__ __device__ int total() const { return table_bytes + zero_bytes + sx_bytes + red_bytes; }
};

struct GemvArgs {
    const uint8_t* w;    // weights in the tile-major GPU layout of the format
    long long row_stride;  // bytes per 16-row tile in that layout
    int M, K;            // rows, columns
    const float* x;      // [nvec][ldx]
    int ldx;
    float* y;            // [nvec][ldy]
    int ldy;
    const float* resid;  // optional [nvec][ldr], added to y
    int ldr;
    int wk;              // warps splitting K for one row tile (1, 2, 4, 8)
    // fused SwiGLU: second matrix (up) with the same layout; y receives silu(W x) * (W2 x)
    const uint8_t* w2;
    int* err;            // device error flag (activation outside the f16 range)
    const float* norm_w; // optional RMSNorm weight applied to x first (nullptr = none)
    int norm_len;        // normalized length (<= K)
    float norm_eps;
    // stream-K split: partial sums of tiles shared by several warps + per-tile arrival
    // counters (zero between launches); filled by the launcher
    float* sk_ws;
    int* sk_cnt;
    int sk_slots;
    int stages;          // depth of each warp's cp.async ring
};

// ------------------------------------------------------------------ formats
// Tile-block images (16 rows x one kernel block) of the GPU layout: byte offsets of the
// regions; a lane's 16-byte piece of row r sits at region + 16 * (4r + t).
struct FmtQ4K {
    static constexpr int kType = T_Q4_K;
    static constexpr int kTile = 2304, kHdr = 0, kQ0 = 256, kQ1 = 1280;
    static constexpr int kBlockElems = 256;
    static constexpr int kMmaPerBlock = 16;
    // element index (within the block) of lane t's k-slot j of MMA `mi`:
    // byte p = 32t + 4wi + j of qs; low nibble -> 64t + 4wi + j, high -> +32
    __device__ static int base(int mi, int t) { return 64 * t + 4 * (mi >> 1) + 32 * (mi & 1); }
    static constexpr bool kNeedSx = true;
    // accumulators come back per lane (lane-distributed columns): lane shares summed over t
    static constexpr bool kLaneShares = true;
    // table slot (within a block) of the hi part of MMA mi = 2 wi + nib, vector v, lane t:
    // the lo- and hi-nibble fragments of one word sit side by side (one 128-bit load)
    template <int NV>
    __device__ static int tab(int mi, int v, int t) {
        return (((mi >> 1) * 2 * NV + 2 * v) * 4 + t) * 2 + (mi & 1);
    }
    static constexpr int kLoOff = 8;  // lo part of the same slot
};

struct FmtQ6K {
    static constexpr int kType = T_Q6_K;
    static constexpr int kTile = 3360, kL0 = 0, kL1 = 1024, kQh = 2048, kSc = 3072, kD = 3328;
    static constexpr int kBlockElems = 256;
    static constexpr int kMmaPerBlock = 16;
    // lane-distributed: lane t owns half h = t >> 1, l in [16s, 16s + 16), s = t & 1; MMA
    // mi = 4q + j takes elements 4j..4j+3 of its scale group q (128h + 32q + 16s + 4j)
    __device__ static int base(int mi, int t) {
        return 128 * (t >> 1) + 32 * (mi >> 2) + 16 * (t & 1) + 4 * (mi & 3);
    }
    static constexpr bool kNeedSx = false;
    static constexpr bool kLaneShares = true;
    // the B table of Q4_K: MMA pairs side by side, hi and lo parts 8 entries apart
    template <int NV>
    __device__ static int tab(int mi, int v, int t) {
        return (((mi >> 1) * 2 * NV + 2 * v) * 4 + t) * 2 + (mi & 1);
    }
    static constexpr int kLoOff = 8;
};

// Q8_0 kernels work on groups of 4 Q8_0 blocks (128 elements, 8 MMAs); mi = 2*blk + half.
struct FmtQ80 {
    static constexpr int kType = T_Q8_0;
    static constexpr int kTile = 2176, kQ0 = 0, kQ1 = 1024, kD = 2048;
    static constexpr int kBlockElems = 128;
    static constexpr int kMmaPerBlock = 8;
    __device__ static int base(int mi, int t) { return 16 * mi + 4 * t; }
    static constexpr bool kNeedSx = false;
    static constexpr bool kLaneShares = false;
    template <int NV>
    __device__ static int tab(int mi, int v, int t) {
        return (mi * 2 * NV + 2 * v) * 4 + t;
    }
    static constexpr int kLoOff = 4;
};

template <class F>
__host__ __device__ constexpr int table_entries_per_block(int nv) {
    return F::kMmaPerBlock * 2 * nv * 4;
}

// ------------------------------------------------------------------ host-side sizing
template <class F>
__host__ __device__ inline GemvSmem gemv_smem_layout(int K, int nv, bool fused) {
    GemvSmem s;
    int nb = (K + F::kBlockElems - 1) / F::kBlockElems;
    s.table_bytes = nb * table_entries_per_block<F>(nv) * 8;
    s.zero_bytes = table_entries_per_block<F>(nv) * 8;
    s.sx_bytes = F::kNeedSx ? ((nv * (K / 32) * 4 + 15) / 16) * 16 : 0;
    s.red_bytes = 8 * 16 * nv * 4 * (fused ? 2 : 1);
    return s;
}

}  // namespace hc
