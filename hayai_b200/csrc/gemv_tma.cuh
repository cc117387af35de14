// gemv_tma.cuh -- the warp-specialised TMA pipeline of the dense GEMV, as device building
// blocks shared by the single-GEMV kernel (gemv_tma.cu) and the persistent FFN-stack kernel
// (ffn_stack.cu).
//
// Work.  A unit is one kernel block (256 elements; 128 for Q8_0) of one 16-row tile; unit
// u is tile u / nbk, block u % nbk.  CTA c owns units [c*T/C, (c+1)*T/C) of a GEMV (stream-K:
// every SM streams the same number of bytes, +-1 unit, whatever the shape).  The range is
// cut into stages: runs of at most SB blocks inside one tile and one SB-aligned block chunk,
// SB = 8 for the fused gate/up pair (8 blocks x 2 matrices) and 16 for one matrix, so a
// stage holds exactly one unit per consumer warp.
//
// Memory.  The weights are tile-major (repack.cu): the blocks of a stage are one contiguous
// run of tile-block images per matrix, so the producer moves a stage (18-54 KB) with one
// cp.async.bulk per matrix completing on the stage's full mbarrier.  (A TMA bulk copy costs
// about the same per instruction whatever its size up to several KB, so per-row copies of
// ~1 KB cap the stream near 3 TB/s; whole stages reach the copy peak.)  Lanes read their
// 16-byte pieces at consecutive addresses: no bank conflicts.  Every byte crosses L2 -> SM
// once.  The weights never depend on the activations, so the producer runs ahead of the
// consumers by up to S stages, across prologues and phase boundaries.
//
// Compute.  Consumer warp w takes unit (matrix w / 8, block w % 8) of every stage of the
// fused pair, or block w of every single-matrix stage; every warp waits for and releases
// every stage in order (so no mbarrier phase can be mistaken for another).  (Two units per
// warp, both matrices of a block sharing their B fragments, needs more registers than 17
// warps can have and a shallower ring: it measured slower.)  Sixteen warps
// (four per scheduler) keep enough independent MMA chains in flight.  Each warp accumulates
// its share of the current tile in registers; at the tile's last stage it drops the partial
// into the tile's shared-memory slot and counts itself in, without waiting: the last warp
// to arrive adds the 16 partials in warp order and finishes the tile (or, for a tile shared
// with the next CTA, stores its partial and lets the last CTA to arrive finish it, adding
// CTA partials in CTA order).  A barrier at every tile end would line all warps up behind
// the slowest unit.  All mbarrier waits are bounded: on expiry the kernel raises bit 1 of
// the error flag and skips the remaining work.
#pragma once

#include "gemv_mma.cuh"
#include "gemv_mma_impl.cuh"

namespace hc {

constexpr int kCW = 16;     // consumer warps
constexpr int kUnits = 16;  // units per stage (one per consumer warp)
constexpr int kTThreads = (kCW + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kMaxTileSlots = kMaxStages + 2;
constexpr int kBarPro = 2;   // named barrier: prologue (consumers only)
constexpr int kBarGrid = 3;  // named barrier: around the grid barrier (consumers only)

// blocks per stage and matrix
__host__ __device__ constexpr int stage_blocks(bool fused) { return fused ? kUnits / 2 : kUnits; }

template <class F>
__host__ __device__ constexpr int tma_stage_bytes(bool /*fused*/) {
    return kUnits * F::kTile;
}

// bytes of one tile slot of per-warp partials
__host__ __device__ constexpr int tile_slot_bytes(int nv) { return kCW * nv * 16 * 4; }

// matrix of consumer warp w
__host__ __device__ constexpr int warp_matrix(int w, bool fused) { return fused ? w / (kUnits / 2) : 0; }

// The IQ formats' unit (gemv_iq.cuh; instantiated by the dense GEMV only).
template <class F, int NV>
__device__ __forceinline__ void iq_stage_unit(const uint8_t* tb, int kbj, const LaneCtx<NV>& ctx,
                                              float (&pA)[1][NV], float (&pB)[1][NV]);

// One consumer warp's unit of a stage: rows g, g+8 of the tile-block image at tb.  Q4_K, Q6_K
// and the IQ formats accumulate lane shares in pA/pB, Q8_0 row sums in yA/yB.
template <class F, int NV>
__device__ __forceinline__ void stage_unit(const uint8_t* tb, int kbj, const LaneCtx<NV>& ctx, float& yA, float& yB,
                                           float (&pA)[1][NV], float (&pB)[1][NV]) {
    if constexpr (F::kType == T_Q4_K) {
        Q4KBlk A[1], B[1];
        tile_load<F, true>(A[0], B[0], tb, ctx.g, ctx.t);
        const int kbs[1] = {kbj};
        q4k_unit<NV, 1>(A, B, kbs, ctx, pA, pB);
    } else if constexpr (F::kType == T_Q6_K) {
        Q6KBlk A, B;
        tile_load<F, true>(A, B, tb, ctx.g, ctx.t);
        q6k_unit<NV>(A, B, kbj, ctx, pA, pB);
    } else if constexpr (is_iq_type(F::kType)) {
        iq_stage_unit<F, NV>(tb, kbj, ctx, pA, pB);
    } else {
        typename BlkOf<F>::T A, B;
        tile_load<F, true>(A, B, tb, ctx.g, ctx.t);
        float dA, dB;
        blk_compute<F, NV>(A, B, kbj, ctx, dA, dB);
        yA += dA;
        yB += dB;
    }
}

// End of a tile (or chunk) for one warp: its partials (lane shares reduced over t first)
// go to red_w[v][16 rows]; the accumulators restart at zero.
template <class F, int NV>
__device__ __forceinline__ void warp_partials(float* red_w, int g, int t, float& yA, float& yB, float (&pA)[1][NV],
                                              float (&pB)[1][NV]) {
    if constexpr (F::kLaneShares) {
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            float sa = pA[0][v], sb = pB[0][v];
            sa += __shfl_xor_sync(kFull, sa, 1);
            sb += __shfl_xor_sync(kFull, sb, 1);
            sa += __shfl_xor_sync(kFull, sa, 2);
            sb += __shfl_xor_sync(kFull, sb, 2);
            if (t == v) {
                yA = sa;
                yB = sb;
            }
            pA[0][v] = pB[0][v] = 0.f;
        }
    }
    if (t < NV) {
        red_w[t * 16 + g] = yA;
        red_w[t * 16 + g + 8] = yB;
    }
    yA = yB = 0.f;
}

// CTA that owns unit u when T units are split over C CTAs (C <= T).
__host__ __device__ __forceinline__ int cta_owner(int u, int C, int T) {
    return (int)(((long long)(u + 1) * C - 1) / T);
}

// Stage ring shared by the producer and the consumers; the position carries across GEMVs.
struct Ring {
    uint32_t full0, empty0;  // mbarrier arrays (8 bytes each)
    uint8_t* base;           // slot 0
    uint32_t base_s;         // its shared-window address
    int S;                   // slots
    int slot_bytes;          // bytes per slot
    int slot, round;         // position of the next stage
    __device__ void advance() {
        if (++slot == S) {
            slot = 0;
            ++round;
        }
    }
};

// One GEMV as the pipeline sees it.
struct GemvPhase {
    const uint8_t* w;   // tile-major weights
    const uint8_t* w2;  // second matrix of the fused pair
    long long tstride;  // bytes per 16-row tile
    int M, K;
    int nbk;            // kernel blocks per row
    int u0, u1;         // this CTA's units
    int T, C, cta;      // all units, CTAs, this CTA
};

template <class F>
__device__ __forceinline__ GemvPhase make_phase(const uint8_t* w, const uint8_t* w2, long long tstride, int M, int K) {
    GemvPhase p;
    p.w = w;
    p.w2 = w2;
    p.tstride = tstride;
    p.M = M;
    p.K = K;
    p.nbk = (K + F::kBlockElems - 1) / F::kBlockElems;
    p.T = ((M + 15) / 16) * p.nbk;
    p.C = gridDim.x;
    p.cta = blockIdx.x;
    p.u0 = (int)((long long)p.cta * p.T / p.C);
    p.u1 = (int)((long long)(p.cta + 1) * p.T / p.C);
    return p;
}

// Producer warp: stream every stage of the phase into the ring.  Returns false when a wait
// for a free slot expired (the consumers stopped).
template <class F, bool FUSED>
__device__ bool produce_phase(Ring& r, const GemvPhase& p, int lane) {
    constexpr int kMats = FUSED ? 2 : 1;
    constexpr int SB = stage_blocks(FUSED);
    int tile = p.u0 / p.nbk, kb = p.u0 - tile * p.nbk;
    for (int u = p.u0; u < p.u1;) {
        const int n = min(min(SB - kb % SB, p.nbk - kb), p.u1 - u);
        if (r.round > 0 && !mbar_wait(r.empty0 + 8 * r.slot, (r.round - 1) & 1)) return false;
        // blocks [kb, kb+n) of the tile are one contiguous run of tile-block images
        const uint32_t bytes = (uint32_t)n * F::kTile;
        const uint32_t full = r.full0 + 8 * r.slot;
        if (lane == 0) mbar_arrive_expect_tx(full, (uint32_t)kMats * bytes);
        __syncwarp();
        if (lane < kMats) {
            const uint8_t* src = (lane ? p.w2 : p.w) + (size_t)tile * p.tstride + (size_t)kb * F::kTile;
            const uint32_t dst = r.base_s + r.slot * r.slot_bytes + (lane * SB + kb % SB) * F::kTile;
            bulk_g2s(dst, src, bytes, full);
        }
        u += n;
        kb += n;
        if (kb == p.nbk) {
            kb = 0;
            ++tile;
        }
        r.advance();
    }
    return true;
}

// Producer warp, after its last stage: wait (bounded) until every copy it issued has landed,
// so the CTA never exits with a bulk copy still writing its shared memory.
__device__ __forceinline__ void drain_ring(const Ring& r, int issued) {
    for (int i = 0; i < r.S && i < issued; ++i) {
        const int last = issued - 1 - i, sl = last % r.S;
        mbar_wait(r.full0 + 8 * sl, (last / r.S) & 1);
    }
}

// Where a finished tile goes.
struct TileOut {
    float* y;            // [nvec][ldy]
    int ldy;
    const float* resid;  // optional [nvec][ldr] (may alias y: each element is read, then written, by one lane)
    int ldr;
    int nvec;
    float* sk_ws;        // cross-CTA partials
    int* sk_cnt;         // per-tile arrival counters (zero between GEMVs)
    int sk_slots;
};

// Consumer warps: consume every stage of the phase (tables already built), finish tiles.
// red/tcnt: tile slots in shared memory; tslot carries across phases.
template <class F, int NV, bool FUSED>
__device__ void consume_phase(Ring& r, const GemvPhase& p, const LaneCtx<NV>& ctx, const TileOut& o, float* red,
                              int* tcnt, int& tslot, bool& aborted, int* err) {
    constexpr int kMats = FUSED ? 2 : 1;
    constexpr int SB = stage_blocks(FUSED);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int NT = r.S + 2;  // tile slots: a warp runs at most S stages (so S tile ends) ahead
    const int mt = warp_matrix(warp, FUSED), jj = warp % SB;  // this warp's matrix and block
    float yA = 0.f, yB = 0.f;
    float pA[1][NV], pB[1][NV];  // Q4_K: this lane's shares (see q4k_unit)
#pragma unroll
    for (int v = 0; v < NV; ++v) pA[0][v] = pB[0][v] = 0.f;
    int tile = p.u0 / p.nbk, kb = p.u0 - tile * p.nbk;
    for (int u = p.u0; u < p.u1;) {
        const int j0 = kb % SB;
        const int n = min(min(SB - j0, p.nbk - kb), p.u1 - u);
        if (!aborted && !mbar_wait(r.full0 + 8 * r.slot, r.round & 1)) {
            aborted = true;
            if (lane == 0 && err) atomicOr(err, 2);
        }
        if (!aborted && jj >= j0 && jj < j0 + n)
            stage_unit<F, NV>(r.base + r.slot * r.slot_bytes + (mt * SB + jj) * F::kTile, kb - j0 + jj, ctx, yA, yB,
                              pA, pB);
        __syncwarp();
        if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
        r.advance();
        u += n;
        kb += n;
        const int ftile = tile;
        if (kb == p.nbk) {
            kb = 0;
            ++tile;
        }
        if (kb != 0 && u != p.u1) continue;

        // ------------------------------------------------------------ tile flush
        // Partials go to red[tslot][warp][v][16 rows] (warp w holds matrix w / SB).  No warp
        // waits: the last warp to arrive (shared-memory counter) adds the 16 partials in warp
        // order and finishes the tile, the others move on.
        warp_partials<F, NV>(red + (size_t)(tslot * kCW + warp) * NV * 16, g, t, yA, yB, pA, pB);
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&tcnt[tslot], 1);
        }
        old = __shfl_sync(kFull, old, 0);
        if (old == kCW - 1) {
            __syncwarp();
            __threadfence_block();
            const int tu0 = ftile * p.nbk, tu1 = tu0 + p.nbk;
            const bool whole = tu0 >= p.u0 && tu1 <= p.u1;
            const int row = lane & 15;
            const int grow = ftile * 16 + row;
            const float* rr = red + (size_t)tslot * kCW * NV * 16;
            int cf = 0, ncon = 1;
            if (!whole) {
                cf = cta_owner(tu0, p.C, p.T);
                ncon = cta_owner(tu1 - 1, p.C, p.T) - cf + 1;
            }
            float* ws = o.sk_ws + (size_t)ftile * o.sk_slots * kMats * 4 * 16;
            float f[2][kMats];  // vectors lane>>4 and (lane>>4)+2
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int v = (lane >> 4) + 2 * q;
#pragma unroll
                for (int m = 0; m < kMats; ++m) {
                    float acc = 0.f;
                    if (v < NV) {
#pragma unroll
                        for (int w = m * SB; w < (m + 1) * SB; ++w) acc += rr[(w * NV + v) * 16 + row];
                    }
                    f[q][m] = acc;
                    if (!whole && v < NV) ws[(((size_t)(p.cta - cf) * kMats + m) * 4 + v) * 16 + row] = acc;
                }
            }
            bool last = whole;
            if (!whole) {
                __threadfence();
                __syncwarp();
                int prev = 0;
                if (lane == 0) prev = atomicAdd(o.sk_cnt + ftile, 1);
                prev = __shfl_sync(kFull, prev, 0);
                last = prev == ncon - 1;
                if (last) {
                    __threadfence();
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int v = (lane >> 4) + 2 * q;
#pragma unroll
                        for (int m = 0; m < kMats; ++m) {
                            float acc = 0.f;
                            if (v < NV)
                                for (int sl = 0; sl < ncon; ++sl)
                                    acc += __ldcg(ws + (((size_t)sl * kMats + m) * 4 + v) * 16 + row);
                            f[q][m] = acc;
                        }
                    }
                    if (lane == 0) o.sk_cnt[ftile] = 0;  // re-arm for the next GEMV
                }
            }
            if (last && grow < p.M) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int v = (lane >> 4) + 2 * q;
                    if (v < NV && v < o.nvec) {
                        float val = f[q][0];
                        if constexpr (FUSED) val = silu_mul(f[q][0], f[q][kMats - 1]);
                        if (o.resid) val += o.resid[(size_t)v * o.ldr + grow];
                        o.y[(size_t)v * o.ldy + grow] = val;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) tcnt[tslot] = 0;  // slot free for tile + NT
        }
        if (++tslot == NT) tslot = 0;
    }
}

}  // namespace hc
