// gemv_tma.cu -- dense Q4_K / Q6_K / Q8_0 GEMV and fused SwiGLU gate/up, warp-specialised:
// one producer warp streams the weights with TMA bulk copies into a ring of shared-memory
// stages, sixteen consumer warps dequantise them into mma.m16n8k16 tiles.
//
// Reference semantics: gemv_q4_k (crates/hayai-model/src/q4k.rs:206-256), gemv_q6_k
// (crates/hayai-model/src/q6k.rs:59-90), gemv_q8_0 (crates/hayai-model/src/quant.rs:598-615)
// and the host SwiGLU combine (crates/hayai-core/src/stream_infer.rs:3836-3840).  Summation
// order differs from the reference's sequential sums (tensor-core tiles, then a fixed-order
// reduction over warps and CTAs); results agree within the f32 parity tolerance and are
// deterministic.
//
// Work.  A unit is one kernel block (256 elements; 128 for Q8_0) of one 16-row tile; unit
// u is tile u / nbk, block u % nbk.  CTA c owns units [c*T/C, (c+1)*T/C) (stream-K: every
// SM streams the same number of bytes, +-1 unit, whatever the shape).  The range is cut
// into stages: runs of at most SB blocks inside one tile and one SB-aligned block chunk,
// SB = 8 for the fused gate/up pair (8 blocks x 2 matrices) and 16 for one matrix, so a
// stage holds exactly one unit per consumer warp.
//
// Memory.  The weights are tile-major (repack.cu): the blocks of a stage are one contiguous
// run of tile-block images per matrix, so the producer moves a stage (18-54 KB) with one
// cp.async.bulk per matrix completing on the stage's full mbarrier.  (A TMA bulk copy costs
// about the same per instruction whatever its size up to several KB, so per-row copies of
// ~1 KB cap the stream near 3 TB/s; whole stages reach the copy peak.)  Lanes read their
// 16-byte pieces at consecutive addresses: no bank conflicts.  Every byte crosses L2 -> SM
// once.  The producer starts before the activation table exists, so weight streaming
// overlaps the prologue, and it runs up to S stages ahead of the consumers (S = what fits
// in 227 KB).
//
// Compute.  Consumer warp w takes unit (matrix w / 8, block w % 8) of every stage of the
// fused pair, or block w of every single-matrix stage; every warp waits for and releases
// every stage in order (so no mbarrier phase can be mistaken for another).  Sixteen warps
// (four per scheduler) keep enough independent MMA chains in flight.  Each warp
// accumulates its share of the current tile in registers; at the tile's last stage it
// drops the partial into the tile's shared-memory slot and counts itself in, without
// waiting: the last warp to arrive adds the 16 partials in warp order and finishes the tile
// (or, for a tile shared with the next CTA, stores its partial and lets the last CTA to
// arrive finish it, adding CTA partials in CTA order).  A barrier at every tile end would
// line all warps up behind the slowest unit and cost a third of the run time.  All mbarrier
// waits are bounded: on expiry the kernel raises bit 1 of the error flag and skips the
// remaining work.
#include "gemv_launch.h"
#include "gemv_mma.cuh"
#include "gemv_mma_impl.cuh"

namespace hc {

constexpr int kCW = 16;      // consumer warps
constexpr int kUnits = 16;   // units per stage (one per consumer warp)
constexpr int kTThreads = (kCW + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kBarPro = 2;   // named barrier: prologue (consumers only)
constexpr int kMaxTileSlots = kMaxStages + 2;

// blocks per stage and matrix
__host__ __device__ constexpr int stage_blocks(bool fused) { return fused ? kUnits / 2 : kUnits; }

template <class F>
__host__ __device__ constexpr int tma_stage_bytes(bool fused) {
    return kUnits * F::kTile;
}

// Shared memory: [2S mbarriers, 128 B][table][zero block][Sx][tile partials: S+2 slots][ring]
struct TmaSmem {
    int table, zero, sx, red, ring;  // byte offsets
};

// bytes of one tile slot of per-warp partials
__host__ __device__ constexpr int tile_slot_bytes(int nv) { return kCW * nv * 16 * 4; }

template <class F>
__host__ __device__ inline TmaSmem tma_smem_layout(int K, int nv, int stages) {
    const GemvSmem g = gemv_smem_layout<F>(K, nv, false);
    TmaSmem s;
    s.table = 128;
    s.zero = s.table + g.table_bytes;
    s.sx = s.zero + g.zero_bytes;
    s.red = s.sx + g.sx_bytes;
    s.ring = s.red + (stages + 2) * tile_slot_bytes(nv);
    s.ring = (s.ring + 127) & ~127;
    return s;
}

// CTA that owns unit u when T units are split over C CTAs (C <= T).
__host__ __device__ __forceinline__ int cta_owner(int u, int C, int T) {
    return (int)(((long long)(u + 1) * C - 1) / T);
}

template <class F, int NV, bool FUSED>
__global__ void __launch_bounds__(kTThreads, 1) gemv_tma_kernel(GemvArgs a, int nvec) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int kMats = FUSED ? 2 : 1;
    constexpr int SB = stage_blocks(FUSED);
    constexpr int kStage = tma_stage_bytes<F>(FUSED);
    const int S = a.stages;
    const TmaSmem L = tma_smem_layout<F>(a.K, NV, S);
    uint8_t* ring = smem + L.ring;
    const uint32_t full0 = smem_addr(smem), empty0 = full0 + 8 * kMaxStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    const int ntiles = (a.M + 15) / 16;
    const int T = ntiles * nbk;
    const int C = gridDim.x, cta = blockIdx.x;
    const int u0 = (int)((long long)cta * T / C), u1 = (int)((long long)(cta + 1) * T / C);

    __shared__ int s_tcnt[kMaxTileSlots];  // arrivals per tile slot (see the tile flush)
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kCW);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < kMaxTileSlots) s_tcnt[threadIdx.x] = 0;
    __syncthreads();

    if (warp == kCW) {
        // ---------------------------------------------------------------- producer
        const uint32_t ring_s = smem_addr(ring);
        int s = 0, slot = 0, round = 0;
        int tile = u0 / nbk, kb = u0 - tile * nbk;
        bool ok = true;
        for (int u = u0; u < u1 && ok;) {
            const int n = min(min(SB - kb % SB, nbk - kb), u1 - u);
            if (round > 0 && !mbar_wait(empty0 + 8 * slot, (round - 1) & 1)) ok = false;
            if (ok) {
                // blocks [kb, kb+n) of the tile are one contiguous run of tile-block images
                const uint32_t bytes = (uint32_t)n * F::kTile;
                const uint32_t full = full0 + 8 * slot;
                if (lane == 0) mbar_arrive_expect_tx(full, (uint32_t)kMats * bytes);
                __syncwarp();
                if (lane < kMats) {
                    const uint8_t* src = (lane ? a.w2 : a.w) + (size_t)tile * a.row_stride + (size_t)kb * F::kTile;
                    const uint32_t dst = ring_s + slot * kStage + (lane * SB + kb % SB) * F::kTile;
                    bulk_g2s(dst, src, bytes, full);
                }
            }
            u += n;
            kb += n;
            if (kb == nbk) {
                kb = 0;
                ++tile;
            }
            ++s;
            if (++slot == S) {
                slot = 0;
                ++round;
            }
        }
        // do not leave while copies may still land: wait for the last fill of every slot
        const int nst = s;
        for (int i = 0; i < S && i < nst; ++i) {
            const int last = nst - 1 - i, sl = last % S;
            mbar_wait(full0 + 8 * sl, (last / S) & 1);
        }
        if (!ok && lane == 0 && a.err) atomicOr(a.err, 2);
        return;
    }

    // -------------------------------------------------------------------- consumers
    uint2* xt = reinterpret_cast<uint2*>(smem + L.table);
    uint2* zero = reinterpret_cast<uint2*>(smem + L.zero);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    float* red = reinterpret_cast<float*>(smem + L.red);
    __shared__ float s_red[32];
    for (int i = threadIdx.x; i < table_entries_per_block<F>(NV); i += kCW * 32) zero[i] = make_uint2(0u, 0u);
    const NormArgs nrm{a.norm_w, a.norm_len, a.norm_eps};
    build_prologue<F, NV>(xt, sx, a.x, a.ldx, a.K, nvec, nrm, s_red, a.err, kCW * 32, kBarPro);
    named_bar_sync(kBarPro, kCW * 32);

    const int g = lane >> 2, t = lane & 3;
    const LaneCtx<NV> ctx = make_ctx<F, NV>(xt, zero, sx, a.K, lane);

    // Warp w takes block w % SB of matrix w / SB of every stage.
    const int mt = FUSED ? warp / SB : 0;
    const int jj = warp % SB;
    using Blk = typename BlkOf<F>::T;
    float yA = 0.f, yB = 0.f;
    float pA[1][NV], pB[1][NV];  // Q4_K: this lane's shares (see q4k_unit)
#pragma unroll
    for (int v = 0; v < NV; ++v) pA[0][v] = pB[0][v] = 0.f;
    bool aborted = false;
    int slot = 0, round = 0, tslot = 0;
    const int NT = S + 2;  // tile slots: a warp runs at most S stages (so S tile ends) ahead
    int tile = u0 / nbk, kb = u0 - tile * nbk;
    for (int u = u0; u < u1;) {
        const int j0 = kb % SB;
        const int n = min(min(SB - j0, nbk - kb), u1 - u);
        if (!aborted && !mbar_wait(full0 + 8 * slot, round & 1)) {
            aborted = true;
            if (lane == 0 && a.err) atomicOr(a.err, 2);
        }
        if (!aborted && jj >= j0 && jj < j0 + n) {
            const int kbj = kb - j0 + jj;
            const uint8_t* tb = ring + slot * kStage + (mt * SB + jj) * F::kTile;
            if constexpr (F::kType == T_Q4_K) {
                Q4KBlk A[1], B[1];
                tile_load<F, true>(A[0], B[0], tb, g, t);
                const int kbs[1] = {kbj};
                q4k_unit<NV, 1>(A, B, kbs, ctx, pA, pB);
            } else {
                Blk A, B;
                tile_load<F, true>(A, B, tb, g, t);
                float dA, dB;
                blk_compute<F, NV>(A, B, kbj, ctx, dA, dB);
                yA += dA;
                yB += dB;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * slot);
        if (++slot == S) {
            slot = 0;
            ++round;
        }
        u += n;
        kb += n;
        const int ftile = tile;
        if (kb == nbk) {
            kb = 0;
            ++tile;
        }
        if (kb != 0 && u != u1) continue;

        // ------------------------------------------------------------ tile flush
        if constexpr (F::kType == T_Q4_K) {
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
        // Partials go to red[tslot][warp][v][16 rows] (warp w holds matrix w / SB).  No warp
        // waits: the last warp to arrive (shared-memory counter) adds the 16 partials in warp
        // order and finishes the tile, the others move on.
        float* rw = red + (size_t)(tslot * kCW + warp) * NV * 16;
        if (t < NV) {
            rw[t * 16 + g] = yA;
            rw[t * 16 + g + 8] = yB;
        }
        yA = yB = 0.f;
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&s_tcnt[tslot], 1);
        }
        old = __shfl_sync(kFull, old, 0);
        if (old == kCW - 1) {
            __syncwarp();
            __threadfence_block();
            const int tu0 = ftile * nbk, tu1 = tu0 + nbk;
            const bool whole = tu0 >= u0 && tu1 <= u1;
            const int row = lane & 15;
            const int grow = ftile * 16 + row;
            const float* rr = red + (size_t)tslot * kCW * NV * 16;
            int cf = 0, ncon = 1;
            if (!whole) {
                cf = cta_owner(tu0, C, T);
                ncon = cta_owner(tu1 - 1, C, T) - cf + 1;
            }
            float* ws = a.sk_ws + (size_t)ftile * a.sk_slots * kMats * 4 * 16;
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
                    if (!whole && v < NV) ws[(((size_t)(cta - cf) * kMats + m) * 4 + v) * 16 + row] = acc;
                }
            }
            bool last = whole;
            if (!whole) {
                __threadfence();
                __syncwarp();
                int old = 0;
                if (lane == 0) old = atomicAdd(a.sk_cnt + ftile, 1);
                old = __shfl_sync(kFull, old, 0);
                last = old == ncon - 1;
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
                    if (lane == 0) a.sk_cnt[ftile] = 0;  // re-arm for the next launch
                }
            }
            if (last && grow < a.M) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int v = (lane >> 4) + 2 * q;
                    if (v < NV && v < nvec) {
                        float val = f[q][0];
                        if constexpr (FUSED) val = silu_mul(f[q][0], f[q][kMats - 1]);
                        if (a.resid) val += a.resid[(size_t)v * a.ldr + grow];
                        a.y[(size_t)v * a.ldy + grow] = val;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) s_tcnt[tslot] = 0;  // slot free for tile + NT
        }
        if (++tslot == NT) tslot = 0;
    }
}

// ------------------------------------------------------------------ host launch
template <class F>
static int tma_stages(int K, int nv, bool fused, int smem_limit) {
    const int fixed = tma_smem_layout<F>(K, nv, 0).ring + 512;  // + static shared
    int s = (smem_limit - fixed) / (tma_stage_bytes<F>(fused) + tile_slot_bytes(nv));
    return s > kMaxStages ? kMaxStages : s;
}

static int tma_grid(int M, int nbk, int num_sms) {
    const long long T = (long long)((M + 15) / 16) * nbk;
    return (int)(T < num_sms ? (T < 1 ? 1 : T) : num_sms);
}

// Most CTAs any tile is split over (the stream-K slots a tile needs).
static int tma_slots(int M, int nbk, int grid) {
    const int T = ((M + 15) / 16) * nbk;
    int best = 1;
    for (int tile = 0; tile * nbk < T; ++tile) {
        const int c = cta_owner(tile * nbk + nbk - 1, grid, T) - cta_owner(tile * nbk, grid, T) + 1;
        best = c > best ? c : best;
    }
    return best;
}

template <class F, int NV, bool FUSED>
static cudaError_t tma_launch_one(GemvArgs a, int nvec, int num_sms, int smem_limit, cudaStream_t stream) {
    const int S = tma_stages<F>(a.K, NV, FUSED, smem_limit);
    if (S < 2) return cudaErrorInvalidConfiguration;
    a.stages = S;
    const int smem = tma_smem_layout<F>(a.K, NV, S).ring + S * tma_stage_bytes<F>(FUSED);
    auto kern = gemv_tma_kernel<F, NV, FUSED>;
    static int configured_smem[64];  // per template instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && configured_smem[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured_smem[dev] = smem;
    }
    const int nbk = (a.K + F::kBlockElems - 1) / F::kBlockElems;
    kern<<<tma_grid(a.M, nbk, num_sms), kTThreads, smem, stream>>>(a, nvec);
    return cudaGetLastError();
}

template <class F>
static int tma_max_nv(int K, bool fused, int smem_limit) {
    for (int nv = 4; nv >= 1; nv >>= 1)
        if (tma_stages<F>(K, nv, fused, smem_limit) >= 2) return nv;
    return 0;
}

template <class F>
static cudaError_t tma_launch_fmt(GemvArgs a, int nvec, bool fused, int num_sms, int smem_limit,
                                  cudaStream_t stream) {
    const int cap = tma_max_nv<F>(a.K, fused, smem_limit);
    if (cap == 0) return cudaErrorInvalidConfiguration;
    for (int v0 = 0; v0 < nvec;) {
        const int left = nvec - v0;
        int nv = left >= 4 && cap >= 4 ? 4 : (left >= 2 && cap >= 2 ? 2 : 1);
        if (left == 3 && cap >= 4) nv = 4;
        const int cnt = left < nv ? left : nv;
        GemvArgs b = a;
        b.x = a.x + (size_t)v0 * a.ldx;
        b.y = a.y + (size_t)v0 * a.ldy;
        b.resid = a.resid ? a.resid + (size_t)v0 * a.ldr : nullptr;
        cudaError_t e;
        if (nv == 4)
            e = fused ? tma_launch_one<F, 4, true>(b, cnt, num_sms, smem_limit, stream)
                      : tma_launch_one<F, 4, false>(b, cnt, num_sms, smem_limit, stream);
        else if (nv == 2)
            e = fused ? tma_launch_one<F, 2, true>(b, cnt, num_sms, smem_limit, stream)
                      : tma_launch_one<F, 2, false>(b, cnt, num_sms, smem_limit, stream);
        else
            e = fused ? tma_launch_one<F, 1, true>(b, cnt, num_sms, smem_limit, stream)
                      : tma_launch_one<F, 1, false>(b, cnt, num_sms, smem_limit, stream);
        if (e != cudaSuccess) return e;
        v0 += cnt;
    }
    return cudaSuccess;
}

// Workspace the stream-K split needs for an M x K launch of `type`: partial-sum floats and
// per-tile counters (which must be zero before the first launch; kernels leave them zero).
void gemv_sk_workspace(int type, int M, int K, bool fused, int num_sms, size_t* ws_floats, size_t* counters) {
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nbk = (K + be - 1) / be;
    const int slots = tma_slots(M, nbk, tma_grid(M, nbk, num_sms));
    *ws_floats = (size_t)((M + 15) / 16) * slots * (fused ? 2 : 1) * 4 * 16;
    *counters = (size_t)((M + 15) / 16);
}

cudaError_t launch_gemv_mma(int type, const GemvArgs& a0, int nvec, bool fused, int num_sms, int smem_limit,
                            cudaStream_t stream) {
    GemvArgs a = a0;
    const int be = type == T_Q8_0 ? 128 : 256;
    const int nbk = (a.K + be - 1) / be;
    a.sk_slots = tma_slots(a.M, nbk, tma_grid(a.M, nbk, num_sms));
    switch (type) {
        case T_Q4_K: return tma_launch_fmt<FmtQ4K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q6_K: return tma_launch_fmt<FmtQ6K>(a, nvec, fused, num_sms, smem_limit, stream);
        case T_Q8_0: return tma_launch_fmt<FmtQ80>(a, nvec, fused, num_sms, smem_limit, stream);
        default: return cudaErrorInvalidValue;
    }
}

bool gemv_mma_supported(int type) { return type == T_Q4_K || type == T_Q6_K || type == T_Q8_0; }

}  // namespace hc
