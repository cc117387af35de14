// ffn_stack.cu -- a whole residual SwiGLU FFN stack, batch 1, as ONE persistent kernel.
//
// Reference semantics: the per-layer FFN of a decode step (crates/hayai-core/src/
// stream_infer.rs:2166, :3752-3864: rms_norm -> gate/up GEMV -> silu(g)*u -> down GEMV ->
// residual add), layer after layer, on the GEMV pipeline of gemv_tma.cuh.
//
// Why one kernel: a launch of ~60 MB of weights streams at ~5 TB/s once it is running, but
// the first stage of a launch only becomes usable ~4.5 us after the start (every SM's first
// copies reach DRAM together), and the launch itself costs more.  In a stack the weights
// never depend on the activations, so here the producer warp of every CTA streams the
// weights of phase after phase (gate/up of layer 0, down of layer 0, gate/up of layer 1, ...)
// through one ring without a pause, while the consumer warps cross a grid-wide barrier
// between phases (the down GEMV needs all of h, the next gate/up all of x).  The first-data
// latency is paid once per stack instead of twice per layer.
//
// Grid barrier: a counter in global memory (zeroed by the host before the launch); each CTA
// adds one per phase and spins, bounded by a one-second timeout, until all CTAs have.  The
// launch is cooperative, so all CTAs are resident.  On a timeout the kernel raises bit 1 of
// the error flag and skips the remaining work; the producer's own waits are bounded too.
// Activations written inside the kernel are read with coherent (L2) loads.
//
// Phase boundaries are kept short: the warp that completes a 16-row tile of h writes it
// straight into the down GEMV's fragment table in global memory (the down prologue is then a
// copy), and the gate/up prologue completes x, sums its squares and normalises in two passes
// over registers.
#include <cuda_runtime.h>

#include <cstdlib>

#include "gemv_launch.h"
#include "gemv_tma.cuh"

namespace hc {

struct StackLayerPtrs {
    const uint8_t* g;
    const uint8_t* u;
    const uint8_t* d;
    const float* norm;  // RMSNorm weight [dm] or nullptr
};

struct StackKArgs {
    const StackLayerPtrs* layers;  // device array [L]
    int L;
    int dm, ff;
    long long ts_a, ts_b;  // tile strides of gate/up and of down
    float* x;              // [dm] the caller's vector: x_0 on entry, x_L on exit
    float* xbuf;           // [2][dm] residual stream: x_l (0 < l < L) lives in xbuf[l & 1]
    float* parts;          // [dm / 16][chunks per tile][16] down partial sums
    uint2* htab;           // the down GEMV's fragment table of h, in global memory
    float* hsx;            // [ff / 16] 16-element sums of h (Q4_K down)
    float eps;
    int* err;
    unsigned* bar;  // [1 + 2L]: grid-barrier counter, then one chunk counter per phase (zero at launch)
    int stages;
    int slot_bytes;
    // tensor parallelism (tp_size > 1): the layers are this rank's d_ff shard; down chunk
    // partials are stored into every rank's exchange region, [2][dm / 16][tp_size * cpt][16]
    // (buffer = cross-GPU phase & 1, rank-major within a tile), and every rank adds them up in
    // the same order, so the replicated residual stream stays identical on all ranks.
    int tp_rank, tp_size;
    char* const* tp_regions;  // [tp_size] the ranks' exchange regions as mapped on this GPU
    unsigned tp_base;         // cross-GPU phases completed before this launch
};

// Shared memory: [mbarriers, 256 B][table][zero block][Sx][tile slots][ring], each table-side
// region sized for the larger of the two GEMVs (they are used one after the other).
struct StackSmem {
    int table, zero, sx, red, ring;
};


template <class FA, class FD>
__host__ __device__ inline StackSmem stack_smem_layout(int dm, int ff, int stages) {
    const GemvSmem a = gemv_smem_layout<FA>(dm, 1, false), b = gemv_smem_layout<FD>(ff, 1, false);
    StackSmem s;
    s.table = 256;
    s.zero = s.table + (a.table_bytes > b.table_bytes ? a.table_bytes : b.table_bytes);
    s.sx = s.zero + (a.zero_bytes > b.zero_bytes ? a.zero_bytes : b.zero_bytes);
    s.red = s.sx + (a.sx_bytes > b.sx_bytes ? a.sx_bytes : b.sx_bytes);
    s.ring = s.red + (stages + 2) * tile_slot_bytes(1);
    s.ring = (s.ring + 127) & ~127;
    return s;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Consumer warps of every CTA meet here; `target` = CTAs x phases completed.  The arrival is a
// release (it publishes every write the CTA's consumers made before the first bar.sync), the
// poll an acquire; the second bar.sync passes the acquire on to the other consumer threads.
__device__ void grid_sync(unsigned* bar, unsigned target, int* err, int* s_abort) {
    named_bar_sync(kBarGrid, kCW * 32);  // this CTA's consumers are done with the phase
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        if (!*s_abort) {
            const unsigned long long t0 = global_ns();
            while (ld_acquire(bar) < target) {
                if (global_ns() - t0 > 1000000000ull) {
                    if (err) atomicOr(err, 2);
                    *s_abort = 1;
                    break;
                }
            }
        }
    }
    named_bar_sync(kBarGrid, kCW * 32);
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Cross-GPU phase end under tensor parallelism.  After the CTA barrier (which orders every
// consumer thread's stores to the peers' regions before thread 0's next operations), thread 0
// alone makes them visible system-wide with one fence (cumulative over what the barrier
// ordered) before the CTA's local arrival; CTA 0 waits for all local CTAs, then adds one
// (release, system scope) to every rank's cross counter; all CTAs wait (acquire, system scope)
// until their own rank's counter shows all ranks' signals for this phase.  Both waits are
// bounded by one second (error bit 1, abort).
__device__ void tp_sync(unsigned* bar, unsigned target, char* const* regions, int tp_rank, int tp_size,
                        unsigned xtarget, int* err, int* s_abort) {
    named_bar_sync(kBarGrid, kCW * 32);
    if (threadIdx.x == 0) {
        __threadfence_system();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const unsigned* xbar = reinterpret_cast<const unsigned*>(regions[tp_rank] + kPeerTpBar);
        const unsigned long long t0 = global_ns();
        if (!*s_abort && blockIdx.x == 0) {
            while (ld_acquire(bar) < target) {
                if (global_ns() - t0 > 1000000000ull) {
                    if (err) atomicOr(err, 2);
                    *s_abort = 1;
                    break;
                }
            }
            if (!*s_abort)
                for (int q = 0; q < tp_size; ++q)
                    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(regions[q] + kPeerTpBar)
                                 : "memory");
        }
        if (!*s_abort) {
            while ((int)(ld_acquire_sys(xbar) - xtarget) < 0) {
                if (global_ns() - t0 > 1000000000ull) {
                    if (err) atomicOr(err, 2);
                    *s_abort = 1;
                    break;
                }
            }
        }
    }
    named_bar_sync(kBarGrid, kCW * 32);
}

// ------------------------------------------------------------------ dynamic chunks
// A phase (one GEMV) is cut into fixed chunks: gate/up into whole 16-row tiles, down into
// runs of 16 kernel blocks of a tile.  CTAs take chunks from a per-phase counter as their
// producer gets to them, so SMs that happen to stream faster take more (across a phase the
// SMs' rates differ by up to ~25%, and which SMs are slow changes from phase to phase: an
// equal static split would leave every phase waiting for the slowest SM).  Every value is
// reduced in an order fixed by the chunk boundaries, never by which CTA ran a chunk, so the
// result is deterministic.
//   gate/up: the warp that completes a tile writes h = silu(g) * u for its 16 rows straight
//            into the down GEMV's fragment table in global memory (f16 hi/lo pairs at their
//            table slots) plus the rows' sum (the Q4_K down needs 32-element sums of h), so
//            the down prologue is a plain copy;
//   down:    chunks leave their 16-row partial sums in a buffer; the next gate/up prologue
//            adds them to the residual stream in chunk order.
// (Completing the down tiles in the phase instead, the last chunk to arrive adding up the
// others, costs a release/acquire round trip per chunk on the warp that is already the
// furthest behind: it measured ~25% slower.)
struct StageDesc {
    int tile, kb, n;  // blocks [kb, kb + n) of the tile
    int part;         // chunk of the tile
    int flags;
};
constexpr int kLastOfChunk = 1, kPhaseEnd = 2;

struct PhaseGeo {
    int nbk;      // kernel blocks per row
    int cb;       // blocks per chunk
    int cpt;      // chunks per tile
    int nchunks;  // all chunks of the phase
};

template <class F>
__host__ __device__ __forceinline__ PhaseGeo phase_geo(int M, int K, int cb) {
    PhaseGeo g;
    g.nbk = (K + F::kBlockElems - 1) / F::kBlockElems;
    g.cb = cb < g.nbk ? cb : g.nbk;
    g.cpt = (g.nbk + g.cb - 1) / g.cb;
    g.nchunks = ((M + 15) / 16) * g.cpt;
    return g;
}

// Producer warp: take chunks until the phase is exhausted, then post the phase-end marker.
template <class F, bool FUSED>
__device__ bool produce_chunks(Ring& r, StageDesc* desc, const uint8_t* w, const uint8_t* w2, long long tstride,
                               const PhaseGeo& pg, unsigned* counter, int lane) {
    constexpr int kMats = FUSED ? 2 : 1;
    constexpr int SB = stage_blocks(FUSED);
    while (true) {
        // take a chunk only once a slot is free for it (late binding balances the SMs)
        if (r.round > 0 && !mbar_wait(r.empty0 + 8 * r.slot, (r.round - 1) & 1)) return false;
        int c = 0;
        if (lane == 0) c = (int)atomicAdd(counter, 1u);
        c = __shfl_sync(kFull, c, 0);
        if (c >= pg.nchunks) {
            if (lane == 0) {
                desc[r.slot] = StageDesc{0, 0, 0, 0, kPhaseEnd};
                mbar_arrive(r.full0 + 8 * r.slot);  // no bytes: completes at once
            }
            __syncwarp();
            r.advance();
            return true;
        }
        const int tile = c / pg.cpt, part = c - tile * pg.cpt;
        const int kb1 = min((part + 1) * pg.cb, pg.nbk);
        int kb = part * pg.cb;
        while (true) {
            const int n = min(SB - kb % SB, kb1 - kb);
            const bool last = kb + n >= kb1;
            const uint32_t full = r.full0 + 8 * r.slot;
            if (lane == 0) {
                desc[r.slot] = StageDesc{tile, kb, n, part, last ? kLastOfChunk : 0};
                mbar_arrive_expect_tx(full, (uint32_t)(kMats * n * F::kTile));
            }
            __syncwarp();
            if (lane < kMats) {
                const uint8_t* src = (lane ? w2 : w) + (size_t)tile * tstride + (size_t)kb * F::kTile;
                bulk_g2s(r.base_s + r.slot * r.slot_bytes + (lane * SB + kb % SB) * F::kTile, src,
                         (uint32_t)(n * F::kTile), full);
            }
            r.advance();
            kb += n;
            if (last) break;
            if (r.round > 0 && !mbar_wait(r.empty0 + 8 * r.slot, (r.round - 1) & 1)) return false;
        }
    }
}

// Where the chunks of a phase go.
struct ChunkOut {
    int M;         // rows of the GEMV
    float* parts;  // down: chunk partials [tiles][chunks per tile][16]
    uint2* htab;   // gate/up: the down GEMV's fragment table
    float* hsx;    // gate/up: 16-row sums of h
    // down under tensor parallelism: partials go to parts_off (floats) in every rank's region,
    // tile stride tp_size * cpt, this rank's chunks at tp_rank * cpt
    char* const* regions;
    int tp_rank, tp_size;
    size_t parts_off;
};

// Gate/up tile: h for rows tile*16 + (lane & 15) (lanes 16-31 repeat lanes 0-15), written into
// FT's fragment table; 4-row chunks are gathered on lanes 0, 4, 8, 12.
template <class FT>
__device__ __forceinline__ void finish_gateup(const ChunkOut& o, int tile, int lane, float g, float u, bool& bad) {
    const int grow = tile * 16 + (lane & 15);
    const float h = grow < o.M ? silu_mul(g, u) : 0.f;
    const float h1 = __shfl_down_sync(kFull, h, 1), h2 = __shfl_down_sync(kFull, h, 2),
                h3 = __shfl_down_sync(kFull, h, 3);
    if (lane < 16 && (lane & 3) == 0) {
        const float xs[4] = {h, h1, h2, h3};
        const int slot = chunk_slot<FT>(tile * 4 + (lane >> 2));
        pack_chunk(xs, o.htab[slot], o.htab[slot + FT::kLoOff], bad);
    }
    if constexpr (FT::kNeedSx) {
        float s = h;
        s += __shfl_xor_sync(kFull, s, 1);
        s += __shfl_xor_sync(kFull, s, 2);
        s += __shfl_xor_sync(kFull, s, 4);
        s += __shfl_xor_sync(kFull, s, 8);
        if (lane == 0) o.hsx[tile] = s;
    }
}

// Consumer warps: every stage of the phase until the end marker.  F = weight format, FT = the
// format whose fragment table the gate/up finishers write (the down GEMV's).
template <class F, class FT, bool FUSED>
__device__ void consume_chunks(Ring& r, const StageDesc* desc, const LaneCtx<1>& ctx, const PhaseGeo& pg,
                               const ChunkOut& o, float* red, int* tcnt, int& tslot, bool& aborted, int* err) {
    constexpr int kMats = FUSED ? 2 : 1;
    constexpr int SB = stage_blocks(FUSED);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int NT = r.S + 2;
    const int mt = warp_matrix(warp, FUSED), jj = warp % SB;  // this warp's matrix and block
    float yA = 0.f, yB = 0.f;
    float pA[1][1] = {{0.f}}, pB[1][1] = {{0.f}};
    bool bad = false;
    while (!aborted) {
        if (!mbar_wait(r.full0 + 8 * r.slot, r.round & 1)) {
            aborted = true;
            if (lane == 0 && err) atomicOr(err, 2);
            break;
        }
        const StageDesc d = desc[r.slot];
        if (d.flags & kPhaseEnd) {
            __syncwarp();
            if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
            r.advance();
            break;
        }
        const int j0 = d.kb % SB;
        if (jj >= j0 && jj < j0 + d.n)
            stage_unit<F, 1>(r.base + r.slot * r.slot_bytes + (mt * SB + jj) * F::kTile, d.kb - j0 + jj, ctx, yA, yB,
                             pA, pB);
        __syncwarp();
        if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
        r.advance();
        if (!(d.flags & kLastOfChunk)) continue;

        // chunk flush: per-warp partials into a tile slot, the last warp to arrive reduces
        warp_partials<F, 1>(red + (size_t)(tslot * kCW + warp) * 16, g, t, yA, yB, pA, pB);
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
            const float* rr = red + (size_t)tslot * kCW * 16;
            const int row = lane & 15;
            float f[kMats];
#pragma unroll
            for (int m = 0; m < kMats; ++m) {
                float acc = 0.f;
#pragma unroll
                for (int w = m * SB; w < (m + 1) * SB; ++w) acc += rr[w * 16 + row];
                f[m] = acc;
            }
            __syncwarp();
            if (lane == 0) tcnt[tslot] = 0;  // slot free for chunk + NT
            if constexpr (FUSED) {
                finish_gateup<FT>(o, d.tile, lane, f[0], f[kMats - 1], bad);
            } else if (o.tp_size == 1) {
                if (lane < 16) o.parts[((size_t)d.tile * pg.cpt + d.part) * 16 + row] = f[0];
            } else if (lane < 16) {
                // the fused all-reduce: this chunk's 16 sums into every rank's region (NVLink
                // stores; made visible system-wide before the phase's cross-GPU signal)
                const size_t off = ((size_t)d.tile * (o.tp_size * pg.cpt) + o.tp_rank * pg.cpt + d.part) * 16 + row;
                for (int q = 0; q < o.tp_size; ++q)
                    reinterpret_cast<float*>(o.regions[q])[o.parts_off + off] = f[0];
            }
        }
        if (++tslot == NT) tslot = 0;
    }
    if (bad && err) atomicOr(err, 1);
}

// Down prologue: the fragment table the gate/up finishers left in global memory is copied
// into shared memory by one bulk copy (issued by consumer thread 0 after the phase barrier's
// acquire, completing on tab_bar), while the threads build the Q4_K 32-element sums from
// pairs of 16-row sums.  Returns false when the copy did not land in time.
template <class F>
__device__ __forceinline__ bool load_down_table(uint2* xt, float* sx, const StackKArgs& a, int tiles_a, uint32_t tab_bar,
                                                uint32_t parity) {
    const int bytes = gemv_smem_layout<F>(a.ff, 1, false).table_bytes;
    if (threadIdx.x == 0) {
        // the table was written through the generic proxy (by other SMs) and the shared
        // region was last read through it; the copy goes through the async proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_expect_tx(tab_bar, (uint32_t)bytes);
        bulk_g2s(smem_addr(xt), a.htab, (uint32_t)bytes, tab_bar);
    }
    if constexpr (F::kNeedSx) {
        for (int j = threadIdx.x; j < bytes / 128; j += kCW * 32) {  // 32 elements = 8 chunks of 16 bytes
            const float s0 = 2 * j < tiles_a ? __ldcg(a.hsx + 2 * j) : 0.f;
            const float s1 = 2 * j + 1 < tiles_a ? __ldcg(a.hsx + 2 * j + 1) : 0.f;
            sx[j] = s0 + s1;
        }
    }
    return mbar_wait(tab_bar, parity);
}

// Gate/up prologue of a layer l > 0.  Pass 1: x_l = x_{l-1} + the down partials of layer l-1
// (added in chunk order), this CTA's share [c0, c1) written back, sum of squares accumulated,
// x_l * w kept in registers (the norm weight loads ride in the same round trip as the
// activation's).  Pass 2: xn = (x_l * w) * inv (rms_norm, crates/hayai-cpu/src/attention.rs:
// 142-147) into the fragment table, with F's 32-element sums for Q4_K.  A thread owns chunks
// tid + k * 512, k < kXRegs: d_model up to 4 * 4 * 512 = 8192 (checked at launch).
constexpr int kXRegs = 4;

template <class F>
__device__ void stack_prologue_a(uint2* xt, float* sx, const float* xin, const XAccum& acc, float* xnext, int c0,
                                 int c1, const float* nw, int dm, float eps, float* scratch, int* err) {
    constexpr int kStep = kCW * 32;
    const int nchunk = dm >> 2;
    const int ntab = (((dm + F::kBlockElems - 1) / F::kBlockElems) * F::kBlockElems) >> 2;  // a multiple of 32
    const float4* nw4 = reinterpret_cast<const float4*>(nw);
    float4 xw[kXRegs];
    float ssq = 0.f;
#pragma unroll
    for (int k = 0; k < kXRegs; ++k) {
        const int c = threadIdx.x + k * kStep;
        xw[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < nchunk) {
            const float4 w = nw ? __ldg(nw4 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 v = load_x4<kLdcg>(xin, c, acc);
            if (c >= c0 && c < c1) reinterpret_cast<float4*>(xnext)[c] = v;
            ssq += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
            xw[k] = make_float4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
        }
    }
    const float tot = block_sum(ssq, scratch, kStep, kBarPro);
    const float inv = nw ? 1.0f / sqrtf(tot / (float)dm + eps) : 1.0f;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < kXRegs; ++k) {
        const int c = threadIdx.x + k * kStep;
        if (c < ntab) {  // whole warps: ntab is a multiple of 32
            const float v4[4] = {xw[k].x * inv, xw[k].y * inv, xw[k].z * inv, xw[k].w * inv};
            const int slot = chunk_slot<F>(c);
            pack_chunk(v4, xt[slot], xt[slot + F::kLoOff], bad);
            if constexpr (F::kNeedSx) {
                // 8 consecutive chunks (= consecutive lanes) form one 32-element sub-block
                float s = (v4[0] + v4[1]) + (v4[2] + v4[3]);
                s += __shfl_xor_sync(kFull, s, 1);
                s += __shfl_xor_sync(kFull, s, 2);
                s += __shfl_xor_sync(kFull, s, 4);
                if ((threadIdx.x & 7) == 0) sx[c >> 3] = s;
            }
        }
    }
    if (bad && err) atomicOr(err, 1);
}

template <class FA, class FD>
__global__ void __launch_bounds__(kTThreads, 1) ffn_stack_kernel(StackKArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_tcnt[kMaxTileSlots];
    __shared__ float s_red[32];
    __shared__ int s_abort;
    __shared__ StageDesc s_desc[kMaxStages];
    const int S = a.stages;
    const StackSmem L = stack_smem_layout<FA, FD>(a.dm, a.ff, S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring r;
    r.full0 = smem_addr(smem);
    r.empty0 = r.full0 + 8 * kMaxStages;
    const uint32_t tab_bar = r.empty0 + 8 * kMaxStages;  // the down table copy
    r.base = smem + L.ring;
    r.base_s = smem_addr(r.base);
    r.S = S;
    r.slot_bytes = a.slot_bytes;
    r.slot = r.round = 0;
    const PhaseGeo ga = phase_geo<FA>(a.ff, a.dm, 1 << 20);  // gate/up: whole tiles
    const PhaseGeo gd = phase_geo<FD>(a.dm, a.ff, kUnits);   // down: 16-block runs
    const int tiles_a = (a.ff + 15) / 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(r.full0 + 8 * s, 1);
            mbar_init(r.empty0 + 8 * s, kCW);
        }
        mbar_init(tab_bar, 1);
        mbar_fence_init();
        s_abort = 0;
    }
    if (threadIdx.x < kMaxTileSlots) s_tcnt[threadIdx.x] = 0;
    __syncthreads();

    if (warp == kCW) {  // producer: every phase's weights, back to back
        bool ok = true;
        for (int l = 0; l < a.L && ok; ++l) {
            const StackLayerPtrs ly = a.layers[l];
            ok = produce_chunks<FA, true>(r, s_desc, ly.g, ly.u, a.ts_a, ga, a.bar + 1 + 2 * l, lane);
            if (ok) ok = produce_chunks<FD, false>(r, s_desc, ly.d, nullptr, a.ts_b, gd, a.bar + 2 + 2 * l, lane);
        }
        drain_ring(r, r.round * S + r.slot);
        if (!ok && lane == 0 && a.err) atomicOr(a.err, 2);
        return;
    }

    uint2* xt = reinterpret_cast<uint2*>(smem + L.table);
    uint2* zero = reinterpret_cast<uint2*>(smem + L.zero);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    float* red = reinterpret_cast<float*>(smem + L.red);
    for (int i = threadIdx.x; i < (L.sx - L.zero) / 8; i += kCW * 32) zero[i] = make_uint2(0u, 0u);
    // table chunks past the last tile of h are padding no finisher writes: zero them once
    if (blockIdx.x == 0) {
        const int nchunk = gemv_smem_layout<FD>(a.ff, 1, false).table_bytes / 16;
        for (int c = tiles_a * 4 + (int)threadIdx.x; c < nchunk; c += kCW * 32) {
            const int sl = chunk_slot<FD>(c);
            a.htab[sl] = a.htab[sl + FD::kLoOff] = make_uint2(0u, 0u);
        }
    }
    int tslot = 0;
    bool aborted = false;
    unsigned phases = 0;
    const unsigned C = gridDim.x;
    const int nc4 = a.dm / 4;  // float4 chunks of x; this CTA writes back [c0, c1)
    const int c0 = (int)((long long)blockIdx.x * nc4 / C), c1 = (int)((long long)(blockIdx.x + 1) * nc4 / C);
    const bool tp = a.tp_size > 1;
    const size_t tp_buf = (size_t)((a.dm + 15) / 16) * a.tp_size * gd.cpt * 16;  // floats per buffer
    // down partials of cross phase q (TP) or of the previous layer
    auto parts_acc = [&](unsigned q) {
        if (!tp) return XAccum{a.parts, gd.cpt, nullptr, 0, 0};
        float* base = reinterpret_cast<float*>(a.tp_regions[a.tp_rank] + kPeerTpParts);
        return XAccum{base + (q & 1) * tp_buf, a.tp_size * gd.cpt, nullptr, 0, 0};
    };
    // x_l: x_0 = the caller's x, then xbuf[l & 1]
    auto xres = [&](int l) { return l == 0 ? a.x : a.xbuf + (size_t)(l & 1) * a.dm; };
    for (int l = 0; l < a.L; ++l) {
        const StackLayerPtrs ly = a.layers[l];
        // gate/up: h = silu(G xn) * (U xn), xn = rms_norm(x_l), x_l = x_{l-1} + D_{l-1} h_{l-1}
        {
            if (l == 0) {
                const NormArgs nrm{ly.norm, a.dm, a.eps};
                build_prologue<FA, 1, kLdcg>(xt, sx, a.x, a.dm, a.dm, 1, nrm, s_red, a.err, kCW * 32, kBarPro);
            } else {
                stack_prologue_a<FA>(xt, sx, xres(l - 1), parts_acc(a.tp_base + l - 1), xres(l), c0, c1, ly.norm, a.dm,
                                     a.eps, s_red, a.err);
            }
            named_bar_sync(kBarPro, kCW * 32);
            const LaneCtx<1> ctx = make_ctx<FA, 1>(xt, zero, sx, a.dm, lane);
            const ChunkOut o{a.ff, nullptr, a.htab, a.hsx, nullptr, 0, 1, 0};
            consume_chunks<FA, FD, true>(r, s_desc, ctx, ga, o, red, s_tcnt, tslot, aborted, a.err);
            grid_sync(a.bar, ++phases * C, a.err, &s_abort);
            if (s_abort) aborted = true;
        }
        // down: chunk partials of D h
        {
            if (!aborted && !load_down_table<FD>(xt, sx, a, tiles_a, tab_bar, l & 1)) {
                aborted = true;
                if (threadIdx.x == 0 && a.err) atomicOr(a.err, 2);
            }
            named_bar_sync(kBarPro, kCW * 32);
            const LaneCtx<1> ctx = make_ctx<FD, 1>(xt, zero, sx, a.ff, lane);
            const unsigned q = a.tp_base + l;  // cross-GPU phase
            const ChunkOut o{a.dm,       a.parts,   nullptr,   nullptr,
                             a.tp_regions, a.tp_rank, a.tp_size, (kPeerTpParts / 4) + (q & 1) * tp_buf};
            consume_chunks<FD, FD, false>(r, s_desc, ctx, gd, o, red, s_tcnt, tslot, aborted, a.err);
            if (tp)
                tp_sync(a.bar, ++phases * C, a.tp_regions, a.tp_rank, a.tp_size, (q + 1) * (unsigned)a.tp_size, a.err,
                        &s_abort);
            else
                grid_sync(a.bar, ++phases * C, a.err, &s_abort);
            if (s_abort) aborted = true;
        }
    }
    // x_L = x_{L-1} + the last down partials, into the caller's x (for L = 1 each element is
    // read and then written by the same thread)
    if (!aborted) {
        const float* xin = xres(a.L - 1);
        const XAccum acc = parts_acc(a.tp_base + a.L - 1);
        for (int c = c0 + (int)threadIdx.x; c < c1; c += kCW * 32)
            reinterpret_cast<float4*>(a.x)[c] = load_x4<kLdcg>(xin, c, acc);
    }
}

// ------------------------------------------------------------------ host side
// Scratch layout (byte offsets, 256-aligned).
struct StackScratch {
    size_t bar, xbuf, parts, htab, hsx, total;
};

template <class FA, class FD>
static StackScratch stack_scratch(int L, int dm, int ff) {
    const PhaseGeo gd = phase_geo<FD>(dm, ff, kUnits);
    const size_t ta = (size_t)(ff + 15) / 16, td = (size_t)(dm + 15) / 16;
    StackScratch s;
    size_t off = 0;
    auto take = [&off](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 255) & ~(size_t)255;
        return o;
    };
    s.bar = take((1 + 2 * (size_t)L) * 4);
    s.xbuf = take(2 * (size_t)dm * 4);
    s.parts = take(td * gd.cpt * 16 * 4);
    s.htab = take((size_t)gemv_smem_layout<FD>(ff, 1, false).table_bytes);
    s.hsx = take(ta * 4);
    s.total = off;
    return s;
}

template <class FA, class FD>
static int stack_stages(int dm, int ff, int smem_limit, int* slot_bytes) {
    const int sa = tma_stage_bytes<FA>(true), sb = tma_stage_bytes<FD>(false);
    *slot_bytes = sa > sb ? sa : sb;
    const int fixed = stack_smem_layout<FA, FD>(dm, ff, 0).ring + 512;  // + static shared
    int s = (smem_limit - fixed) / (*slot_bytes + tile_slot_bytes(1));
    return s > kMaxStages ? kMaxStages : s;
}

template <class FA, class FD>
static cudaError_t launch_stack_t(const StackLaunch& s, int num_sms, int smem_limit, cudaStream_t stream, bool dry,
                                  size_t* scratch_bytes) {
    const PhaseGeo ga = phase_geo<FA>(s.ff, s.dm, 1 << 20), gd = phase_geo<FD>(s.dm, s.ff, kUnits);
    if ((long long)((s.ff + 15) / 16) * ga.nbk < num_sms || (long long)((s.dm + 15) / 16) * gd.nbk < num_sms)
        return cudaErrorInvalidConfiguration;  // fewer units than SMs: the per-layer kernels shrink their grid
    if ((((s.dm + FA::kBlockElems - 1) / FA::kBlockElems) * FA::kBlockElems) / 4 > kXRegs * kCW * 32)
        return cudaErrorInvalidConfiguration;  // the gate/up prologue holds at most kXRegs chunks per thread
    const int tp = s.tp_size < 1 ? 1 : s.tp_size;
    if (gd.cpt * tp > kMaxParts || s.dm % 4 || s.ff % 4)
        return cudaErrorInvalidConfiguration;  // more down partials per tile than the prologue adds up
    if (tp > 1 && (size_t)2 * ((s.dm + 15) / 16) * tp * gd.cpt * 16 * 4 > kPeerTpPartsBytes)
        return cudaErrorInvalidConfiguration;
    int slot_bytes = 0;
    const int S = stack_stages<FA, FD>(s.dm, s.ff, smem_limit, &slot_bytes);
    if (S < 3) return cudaErrorInvalidConfiguration;  // too shallow to pay off: use the per-layer kernels
    const int smem = stack_smem_layout<FA, FD>(s.dm, s.ff, S).ring + S * slot_bytes;
    auto kern = ffn_stack_kernel<FA, FD>;
    // the shared-memory opt-in and the one-CTA-per-SM check, once per device and size
    static int checked[64];  // per device: the largest size configured and found to fit
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || checked[dev] < smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTThreads, smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
        if (dev < 64) checked[dev] = smem;
    }
    const StackScratch sc = stack_scratch<FA, FD>(s.L, s.dm, s.ff);
    if (dry) {
        if (scratch_bytes) *scratch_bytes = sc.total;
        return cudaSuccess;
    }
    uint8_t* base = static_cast<uint8_t*>(s.scratch);
    StackKArgs a{};
    a.layers = (const StackLayerPtrs*)s.layers;
    a.L = s.L;
    a.dm = s.dm;
    a.ff = s.ff;
    a.ts_a = s.ts_a;
    a.ts_b = s.ts_b;
    a.x = s.x;
    a.xbuf = reinterpret_cast<float*>(base + sc.xbuf);
    a.parts = reinterpret_cast<float*>(base + sc.parts);
    a.htab = reinterpret_cast<uint2*>(base + sc.htab);
    a.hsx = reinterpret_cast<float*>(base + sc.hsx);
    a.eps = s.eps;
    a.err = s.err;
    a.bar = reinterpret_cast<unsigned*>(base + sc.bar);
    a.stages = S;
    a.slot_bytes = slot_bytes;
    a.tp_rank = tp > 1 ? s.tp_rank : 0;
    a.tp_size = tp;
    a.tp_regions = reinterpret_cast<char* const*>(s.tp_regions);
    a.tp_base = s.tp_base;
    e = cudaMemsetAsync(a.bar, 0, sc.xbuf - sc.bar, stream);
    if (e != cudaSuccess) return e;
    void* args[] = {&a};
    return cudaLaunchCooperativeKernel((const void*)kern, dim3(num_sms), dim3(kTThreads), args, smem, stream);
}

static bool flow_enabled() {
    static const bool on = [] {
        const char* v = getenv("HAYAI_FLOW_KERNEL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// The CTA count the kernel runs with: one per SM.
cudaError_t launch_ffn_stack(int type_a, int type_d, const StackLaunch& s, int num_sms, int smem_limit,
                             cudaStream_t stream, bool dry, size_t* scratch_bytes) {
    if (flow_enabled()) {
        const cudaError_t e = launch_ffn_flow(type_a, type_d, s, num_sms, smem_limit, stream, dry, scratch_bytes);
        if (e != cudaErrorInvalidConfiguration) return e;
        cudaGetLastError();
    }
#define HC_STACK_CASE(TA, FAT, TD, FDT) \
    if (type_a == TA && type_d == TD)   \
        return launch_stack_t<FAT, FDT>(s, num_sms, smem_limit, stream, dry, scratch_bytes);
    HC_STACK_CASE(T_Q4_K, FmtQ4K, T_Q6_K, FmtQ6K)
    HC_STACK_CASE(T_Q4_K, FmtQ4K, T_Q4_K, FmtQ4K)
    HC_STACK_CASE(T_Q6_K, FmtQ6K, T_Q6_K, FmtQ6K)
    HC_STACK_CASE(T_Q8_0, FmtQ80, T_Q8_0, FmtQ80)
#undef HC_STACK_CASE
    return cudaErrorInvalidConfiguration;
}

}  // namespace hc
