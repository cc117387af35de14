// ffn_flow.cu -- the batch-1 residual SwiGLU FFN stack as ONE persistent dataflow kernel.
//
// Reference semantics: the per-layer FFN of a decode step (crates/hayai-core/src/
// stream_infer.rs:2166, :3752-3864: rms_norm (crates/hayai-cpu/src/attention.rs:142-147) ->
// gate/up GEMV -> silu(g) * u -> down GEMV -> residual add), layer after layer.
//
// Why a dataflow kernel.  The weights never depend on the activations, so one producer warp
// per SM streams every layer's gate/up and down weights through a ring of shared-memory
// stages without pausing (gemv_tma.cuh), and sixteen consumer warps decode them on the
// tensor cores.  What remains is the two dependencies of a layer, and neither is a grid-wide
// barrier here:
//   gate/up -> down: the down GEMV is cut into K-parts of 16 blocks (4096 elements of h) and
//     its chunks are taken part-major, so part p only waits until the gate/up tiles that
//     produce h[4096p, 4096p + 4096) are done.  Those tiles were taken first, so a CTA that
//     runs out of gate/up work moves straight on to down work.  The producer waits for the
//     part (a per-part counter, acquire) and copies its slice of h's fragment table into one
//     of two shared-memory table slots, ahead of the consumers.
//   down -> next gate/up: every gate/up row needs the whole normalised x.  The chunk that
//     adds the last K-part of a down tile finishes it: it adds the earlier parts' partial
//     sums in part order to the residual, stores x, and writes x * w_norm (next layer) straight
//     into the next gate/up's fragment table in global memory, with the tile's 16-row sums of
//     x * w and of x^2.  A CTA starts the next layer once all 256 tiles are final: one bulk
//     copy of the table, and 1/rms from the 256 squared sums (the norm's scalar is applied to
//     the gate and up outputs: silu(inv * G(x w)) * (inv * U(x w))).
// Every sum has a fixed order (chunk boundaries, warp order, part order), so the result is
// deterministic and independent of which CTA ran what.
//
// Tensor parallelism (up to 8 GPUs, each holding a d_ff shard of every layer): the chunk of a
// tile's last local K-part sums the local parts and stores the tile's 16 partial outputs into
// slot [rank] of every rank's exchange region over NVLink (plain stores, one system fence, one
// system-scope counter add per rank and tile).  An extra warp per CTA, the x-tile completer,
// owns tiles c, c + C, ... : it waits (acquire, system scope, bounded) until the tile's counter
// shows every rank's partial, adds them in rank order to the replicated residual (the same sum
// on every rank) and finishes the tile as above.  The finishers never wait on another GPU, so
// no hand-over slot can be held while a peer waits for it.  Slots alternate with the phase
// parity; the counters only grow (their targets carry the phases of earlier launches).
//
// Counters (global, per layer, zeroed by the host before the launch): chunk counters of the
// two phases, h-part readiness, per-tile down arrivals, finished x tiles, and the CTAs that
// copied a layer's x table (a guard: the double-buffered table is only rewritten after every
// CTA copied the previous one).  Every wait is bounded (about a second, error bit 1) and also
// gives up when another CTA has raised the error flag, so a failure ends the kernel quickly.
#include <cuda_runtime.h>

#include "gemv_launch.h"
#include "gemv_tma.cuh"

namespace hc {
namespace flow {

constexpr int kPartBlocks = 16;  // down K-parts: at most 16 super-blocks (4096 elements of h) each
constexpr int kMaxS = 6;
constexpr int kFW = 3;                            // finisher warps
constexpr int kThreads = (kCW + 1 + kFW) * 32;    // consumers, producer, finishers
constexpr int kThreadsTP = kThreads + 32;          // + the x-tile completer of tensor parallelism
constexpr int kNT = 8;                            // hand-over slots (chunk partials) to the finishers
// mbarriers at the head of shared memory: ring full / empty, x table, two down-table slots,
// hand-over full / free
constexpr int kBarBytes = 16 * kMaxS + 8 + 16 + 16 * kNT;
static_assert(kBarBytes <= 256, "the mbarriers fit the 256-byte head of shared memory");

struct Layer {  // same layout as the host's per-layer pointer table
    const uint8_t* g;
    const uint8_t* u;
    const uint8_t* d;
    const float* norm;  // RMSNorm weight [dm] or nullptr
};

// per-layer counters: [0] gate/up chunks, [1] down chunks, [2] finished x tiles, [3] CTAs that
// copied this layer's x table, [4, 4 + np) finished gate/up tiles per h part,
// [4 + np, 4 + np + td) arrived down parts per tile
constexpr int kCtrGu = 0, kCtrDn = 1, kXcnt = 2, kCopied = 3, kHcnt = 4;

struct Args {
    const Layer* layers;
    int L, dm, ff;
    long long ts_a, ts_b;  // tile strides of gate/up and of down
    float* x;              // caller's x: x_0 on entry, x_L on exit
    float* xbuf;           // [2][dm] residual stream (x_l in xbuf[l & 1] for l >= 1)
    float* parts;          // [td][np][16] down partial sums
    uint2* htab;           // down fragment table (all of K) in global memory
    uint2* xtab;           // [2][tab_a] gate/up fragment tables
    float* xs;             // [2][2 td]: 16-row sums of x * w, then 16-row sums of x^2
    unsigned* cnt;         // [L][cstride]
    int cstride;
    float eps;
    int* err;
    int S, slot_bytes, dsb;  // ring slots, bytes per slot, down blocks per stage
    // tensor parallelism (tp_size > 1): this rank holds a d_ff shard of every layer; each
    // tile's partial of the down output goes to every rank's region, x is completed per tile
    // once all ranks' partials are in (identically on every rank: rank order)
    char* const* regions;  // every rank's exchange region as mapped here
    int tp_rank, tp_size;
    unsigned tp_base;      // cross-GPU phases before this launch (slot parity)
    unsigned flow_base;    // this kernel's phases before this launch (per-tile counter targets)
};

struct Desc {
    int tile, kb, n;  // blocks [kb, kb + n) of the tile
    int part;         // down K-part (-1: gate/up)
    int flags;
};
constexpr int kLastOfChunk = 1, kPhaseEnd = 2;

// What a finisher needs to know about a chunk handed over in a slot.
struct Meta {
    int tile, part, layer, end;  // part -1: gate/up; end: no more chunks
};

template <class FA, class FD>
struct Geo {
    int nbk_a, nbk_d;  // kernel blocks per row
    int ta, td;        // 16-row tiles of gate/up and of down
    int np;            // down K-parts
    int pb;            // blocks per part (the last part may hold fewer)
    int tab_a;         // gate/up table bytes
    int tab_p;         // bytes of one down table part (16 blocks)
    __host__ __device__ Geo(int dm, int ff) {
        nbk_a = dm / FA::kBlockElems;
        nbk_d = ff / FD::kBlockElems;
        ta = ff / 16;
        td = dm / 16;
        // 16-block parts (parts of equal size measured slower: their stages are smaller); a short
        // d_ff (a tensor-parallel shard) gets parts of a quarter of it, at least 4 blocks, so the
        // down GEMV can still start before the last gate/up tiles are done
        pb = nbk_d >= 3 * kPartBlocks ? kPartBlocks : ((nbk_d + 3) / 4 > 4 ? (nbk_d + 3) / 4 : 4);
        np = (nbk_d + pb - 1) / pb;
        tab_a = nbk_a * table_entries_per_block<FA>(1) * 8;
        tab_p = pb * table_entries_per_block<FD>(1) * 8;
    }
    __host__ __device__ int part_blocks(int p) const {
        return nbk_d - p * pb < pb ? nbk_d - p * pb : pb;
    }
    __host__ __device__ int part_tiles(int p) const {  // gate/up tiles producing h of part p
        const int t0 = p * pb * FD::kBlockElems / 16;
        const int t1 = t0 + part_blocks(p) * FD::kBlockElems / 16;
        return (t1 < ta ? t1 : ta) - t0;
    }
};

// Shared memory: [barriers 256 B][gate/up table][sx][down table slots x 2][zero block]
// [x sums staging 2 td floats][hand-over slots: partials kNT x 1 KB, then kNT Meta][ring]
struct Smem {
    int tab_a, sx, tab_d, zero, stage, red, meta, ring, total;
};

template <class FA, class FD>
__host__ __device__ inline Smem smem_layout(int dm, int ff, int S, int slot_bytes) {
    const Geo<FA, FD> g(dm, ff);
    Smem s;
    s.tab_a = 256;  // after the mbarriers (kBarBytes)
    s.sx = s.tab_a + g.tab_a;
    s.tab_d = s.sx + (FA::kNeedSx ? ((dm / 32) * 4 + 15) / 16 * 16 : 0);
    s.zero = s.tab_d + 2 * g.tab_p;
    s.stage = s.zero + table_entries_per_block<FD>(1) * 8;
    s.red = s.stage + 2 * g.td * 4;
    s.meta = s.red + kNT * tile_slot_bytes(1);
    s.ring = (s.meta + kNT * (int)sizeof(Meta) + 127) & ~127;
    s.total = s.ring + S * slot_bytes;
    return s;
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_rel(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ bool err_raised(const int* err) {
    return (*reinterpret_cast<const volatile int*>(err) & 2) != 0;
}

__device__ __forceinline__ unsigned ld_acq_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_sys(unsigned* p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded acquire-wait (system scope: counters other GPUs raise) until *p >= target.
__device__ bool wait_ge_sys(const unsigned* p, unsigned target, int* err) {
    const unsigned long long t0 = now_ns();
    for (int i = 0;; ++i) {
        if ((int)(ld_acq_sys(p) - target) >= 0) return true;
        if ((i & 63) == 63) {
            if (err_raised(err) || now_ns() - t0 > 1000000000ull) {
                atomicOr(err, 2);
                return false;
            }
        }
    }
}

// Bounded acquire-wait until *p >= target: about a second, or until another CTA raised the
// error flag.  On failure raises bit 1 of the flag and returns false.
__device__ bool wait_ge(const unsigned* p, unsigned target, int* err) {
    if (ld_acq(p) >= target) return true;
    const unsigned long long t0 = now_ns();
    for (int i = 0;; ++i) {
        if (ld_acq(p) >= target) return true;
        if ((i & 63) == 63) {
            if (err_raised(err) || now_ns() - t0 > 1000000000ull) {
                atomicOr(err, 2);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- producer
struct Prod {
    Ring r;
    uint32_t dbar0;     // two down-table barriers
    uint8_t* tab_d;     // down table slots (shared)
    int loads0, loads1;  // copies issued per table slot
    int last0, last1;    // last stage index that used each table slot (-1: none)
    __device__ int stage_index() const { return r.round * r.S + r.slot; }
};

// Take the next chunk index of a phase (lane 0's atomic, broadcast to the warp).
__device__ __forceinline__ int take(unsigned* ctr, int lane) {
    int c = 0;
    if (lane == 0) c = (int)atomicAdd(ctr, 1u);
    return __shfl_sync(kFull, c, 0);
}

// Wait for the ring slot of the next stage; false on timeout.
__device__ __forceinline__ bool slot_free(Ring& r) {
    return r.round == 0 || mbar_wait(r.empty0 + 8 * r.slot, (r.round - 1) & 1);
}

template <class FA, class FD>
__device__ bool produce_layer(Prod& P, Desc* desc, const Args& a, const Geo<FA, FD>& G, int l, int lane) {
    const Layer ly = a.layers[l];
    unsigned* cnt = a.cnt + (size_t)l * a.cstride;
    constexpr int SBA = stage_blocks(true);  // 8 blocks x 2 matrices
    Ring& r = P.r;
    // ---- gate/up: whole 16-row tiles, two stages each; the next index is taken while this
    // chunk's copies are issued (its latency hides behind them)
    int c = take(cnt + kCtrGu, lane);
    while (c < G.ta) {
        const int nc = take(cnt + kCtrGu, lane);
        for (int kb = 0; kb < G.nbk_a; kb += SBA) {
            const int n = min(SBA, G.nbk_a - kb);
            if (!slot_free(r)) return false;
            const uint32_t full = r.full0 + 8 * r.slot;
            if (lane == 0) {
                desc[r.slot] = Desc{c, kb, n, -1, kb + n >= G.nbk_a ? kLastOfChunk : 0};
                mbar_arrive_expect_tx(full, (uint32_t)(2 * n * FA::kTile));
            }
            __syncwarp();
            if (lane < 2) {
                const uint8_t* src = (lane ? ly.u : ly.g) + (size_t)c * a.ts_a + (size_t)kb * FA::kTile;
                bulk_g2s(r.base_s + r.slot * r.slot_bytes + lane * SBA * FA::kTile, src, (uint32_t)(n * FA::kTile),
                         full);
            }
            r.advance();
        }
        c = nc;
    }
    if (!slot_free(r)) return false;
    if (lane == 0) {
        desc[r.slot] = Desc{0, 0, 0, -1, kPhaseEnd};
        mbar_arrive(r.full0 + 8 * r.slot);  // no bytes: completes at once
    }
    __syncwarp();
    r.advance();

    // ---- down: (part, tile) chunks part-major; a part's table slice is copied into table slot
    // part & 1 once the gate/up tiles of that part are done and the slot's previous part is
    // consumed
    int cur = -1;
    unsigned next_ready = 0;  // the next part's counter, read ahead (its latency overlaps the copies)
    c = take(cnt + kCtrDn, lane);
    while (c < G.np * G.td) {
        const int p = c / G.td, tile = c - p * G.td;
        const int kb0 = p * G.pb, kb1 = kb0 + G.part_blocks(p);
        bool first = true;
        for (int kb = kb0; kb < kb1; kb += a.dsb) {
            const int n = min(a.dsb, kb1 - kb);
            if (!slot_free(r)) return false;
            if (first && p != cur) {
                const int ts = p & 1, X = P.stage_index();
                // the slot's previous part: every stage of it released
                const int lastq = ts ? P.last1 : P.last0;  // -1: the slot was never used
                if (lastq >= 0 && lastq > X - r.S) {
                    const int q = lastq;
                    if (!mbar_wait(r.empty0 + 8 * (q % r.S), (q / r.S) & 1)) return false;
                }
                bool ok = true;
                if (lane == 0) {
                    const unsigned want = (unsigned)G.part_tiles(p);
                    ok = (p == cur + 1 && next_ready >= want) || wait_ge(cnt + kHcnt + p, want, a.err);
                    if (ok) {
                        // h was written through the generic proxy by other SMs; the copy reads it
                        // through the async proxy
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        const uint32_t bar = P.dbar0 + 8 * ts;
                        const uint32_t bytes = (uint32_t)(G.part_blocks(p) * table_entries_per_block<FD>(1) * 8);
                        mbar_arrive_expect_tx(bar, bytes);
                        bulk_g2s(smem_addr(P.tab_d + ts * G.tab_p),
                                 reinterpret_cast<const uint8_t*>(a.htab) + (size_t)p * G.tab_p, bytes, bar);
                    }
                }
                ok = __shfl_sync(kFull, ok ? 1 : 0, 0) != 0;
                if (!ok) return false;
                if (ts) ++P.loads1;
                else ++P.loads0;
                cur = p;
                if (lane == 0 && p + 1 < G.np) next_ready = ld_acq(cnt + kHcnt + p + 1);
            }
            first = false;
            const uint32_t full = r.full0 + 8 * r.slot;
            if (lane == 0) {
                desc[r.slot] = Desc{tile, kb, n, p, kb + n >= kb1 ? kLastOfChunk : 0};
                mbar_arrive_expect_tx(full, (uint32_t)(n * FD::kTile));
            }
            __syncwarp();
            if (lane == 0)
                bulk_g2s(r.base_s + r.slot * r.slot_bytes, ly.d + (size_t)tile * a.ts_b + (size_t)kb * FD::kTile,
                         (uint32_t)(n * FD::kTile), full);
            if (p & 1) P.last1 = P.stage_index();
            else P.last0 = P.stage_index();
            r.advance();
        }
        if (!slot_free(r)) return false;  // claim the next chunk only once a slot is free for it
        c = take(cnt + kCtrDn, lane);
    }
    if (!slot_free(r)) return false;
    if (lane == 0) {
        desc[r.slot] = Desc{0, 0, 0, -1, kPhaseEnd};
        mbar_arrive(r.full0 + 8 * r.slot);
    }
    __syncwarp();
    r.advance();
    return true;
}

// ---------------------------------------------------------------- consumers
// 4-row groups of a 16-row column (value v on lanes 0..15, repeated on 16..31) packed into
// the fragment table of format FT: tile `tile`, chunks tile*4 .. tile*4+3.
template <class FT>
__device__ __forceinline__ void pack_rows(uint2* tab, int tile, int lane, float v, bool& bad) {
    const float v1 = __shfl_down_sync(kFull, v, 1), v2 = __shfl_down_sync(kFull, v, 2),
                v3 = __shfl_down_sync(kFull, v, 3);
    if (lane < 16 && (lane & 3) == 0) {
        const float xs[4] = {v, v1, v2, v3};
        const int slot = chunk_slot<FT>(tile * 4 + (lane >> 2));
        pack_chunk(xs, tab[slot], tab[slot + FT::kLoOff], bad);
    }
}

// Sum of v over lanes 0..15 (fixed tree), valid on lane 0.
__device__ __forceinline__ float sum16(float v) {
    v += __shfl_down_sync(kFull, v, 8);
    v += __shfl_down_sync(kFull, v, 4);
    v += __shfl_down_sync(kFull, v, 2);
    v += __shfl_down_sync(kFull, v, 1);
    return v;
}

// Finisher warp: completes chunks handed over in slot k % kNT, taking the next chunk index k
// from a shared counter whenever it is free (a finisher held up by an x tile's wait does not
// hold up the chunks after it).
//   gate/up chunk: g, u = the warp sums (8 + 8 warps), h = silu(inv g) * (inv u) into h's table
//                  in global memory, then the h part's counter (release);
//   down chunk, not the last K-part: the 16-row partial into `parts`, then the tile's counter;
//   down chunk of the last K-part: waits (acquire) for the tile's other parts, adds them in part
//                  order to the residual, stores x, and writes x * w_norm(next layer) into the next
//                  gate/up table with the tile's 16-row sums of x * w and x^2, then the layer's
//                  finished-tile counter.
// Global memory latency (stores, release fences, acquire waits) lands here, not on the warps
// that consume the weight stream.
template <class FA, class FD, bool TP>
__device__ void finisher(const Args& a, const Geo<FA, FD>& G, int* next, uint32_t tfull0, uint32_t tfree0,
                         const float* red, const Meta* meta, const float* s_inv, const float* stage, int lane) {
    bool bad = false;
    const int row = lane & 15;
    int copied_layer = -1;  // (lane 0) the layer whose table-copied count was seen complete
    int inv_layer = -1;     // the layer whose 1 / rms is in inv
    float inv = 1.0f;
    while (true) {
        int k = 0;
        if (lane == 0) k = atomicAdd(next, 1);
        k = __shfl_sync(kFull, k, 0);
        const int ts = k % kNT, use = k / kNT;
        if (!mbar_wait(tfull0 + 8 * ts, use & 1)) {
            if (lane == 0) atomicOr(a.err, 2);
            break;
        }
        const Meta m = meta[ts];
        if (m.end) break;
        const float* rr = red + (size_t)ts * kCW * 16;
        float f0 = 0.f, f1 = 0.f;
        if (m.part < 0) {
#pragma unroll
            for (int w = 0; w < kCW / 2; ++w) f0 += rr[w * 16 + row];
#pragma unroll
            for (int w = kCW / 2; w < kCW; ++w) f1 += rr[w * 16 + row];
        } else {
#pragma unroll
            for (int w = 0; w < kCW; ++w) f0 += rr[w * 16 + row];
        }
        if (m.layer != inv_layer) {  // 1 / rms(x) of this layer's input
            inv_layer = m.layer;
            if (m.layer == 0) {
                inv = *s_inv;  // (the consumers' first prologue)
            } else {  // from the copied sums of squares of x's 16-element tiles (fixed order)
                float q = 0.f;
                for (int i = lane; i < G.td; i += 32) q += stage[G.td + i];
                q = warp_sum(q);
                inv = a.layers[m.layer].norm ? 1.0f / sqrtf(q / (float)a.dm + a.eps) : 1.0f;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(tfree0 + 8 * ts);  // the slot may be refilled
        unsigned* cnt = a.cnt + (size_t)m.layer * a.cstride;
        const int tile = m.tile;
        if (m.part < 0) {
            const int grow = tile * 16 + row;
            const float h = grow < a.ff ? silu_mul(inv * f0, inv * f1) : 0.f;
            pack_rows<FD>(a.htab, tile, lane, h, bad);
            __syncwarp();
            if (lane == 0) red_rel(cnt + kHcnt + tile * 16 / (G.pb * FD::kBlockElems), 1u);
            continue;
        }
        unsigned* tc = cnt + kHcnt + G.np + tile;
        if (m.part < G.np - 1) {
            if (lane < 16) a.parts[((size_t)tile * G.np + m.part) * 16 + row] = f0;
            __syncwarp();
            if (lane == 0) red_rel(tc, 1u);
            continue;
        }
        const int l = m.layer;
        const bool last_layer = l == a.L - 1;
        if constexpr (TP) {
            // this rank's partial of the tile (its parts in part order) into slot [rank] of every
            // rank's region, then one counter add per rank; the completer warps finish x
            int okp = 1;
            if (lane == 0) okp = wait_ge(tc, (unsigned)(G.np - 1), a.err) ? 1 : 0;
            okp = __shfl_sync(kFull, okp, 0);
            __syncwarp();
            if (!okp) break;
            float loc = 0.f;
            for (int q = 0; q < G.np - 1; ++q) loc += __ldcg(a.parts + ((size_t)tile * G.np + q) * 16 + row);
            loc += f0;
            const size_t slot =
                (((size_t)((a.tp_base + l) & 1) * G.td + tile) * a.tp_size + a.tp_rank) * 16 + row;
            if (lane < 16)
                for (int q = 0; q < a.tp_size; ++q) reinterpret_cast<float*>(a.regions[q] + kPeerTpParts)[slot] = loc;
            __syncwarp();
            if (lane == 0) {
                __threadfence_system();  // the lanes' stores (ordered by the warp barrier) first
                for (int q = 0; q < a.tp_size; ++q)
                    red_sys(reinterpret_cast<unsigned*>(a.regions[q] + kPeerFlowTile) + tile, 1u);
            }
            continue;
        }
        // the tile's earlier parts have arrived (acquire), and every CTA copied the table about to
        // be overwritten (layer l - 1's, same buffer)
        int ok = 1;
        if (lane == 0) {
            ok = wait_ge(tc, (unsigned)(G.np - 1), a.err) ? 1 : 0;
            if (ok && l >= 2 && !last_layer && copied_layer != l) {
                ok = wait_ge(a.cnt + (size_t)(l - 1) * a.cstride + kCopied, gridDim.x, a.err) ? 1 : 0;
                copied_layer = l;
            }
        }
        ok = __shfl_sync(kFull, ok, 0);
        __syncwarp();  // lane 0's acquire orders the other lanes' loads below
        if (!ok) break;
        const float* xprev = l == 0 ? a.x : a.xbuf + (size_t)(l & 1) * a.dm;
        float xn = __ldcg(xprev + tile * 16 + row);
        for (int q = 0; q < G.np - 1; ++q) xn += __ldcg(a.parts + ((size_t)tile * G.np + q) * 16 + row);
        xn += f0;
        if (lane < 16) a.xbuf[(size_t)((l + 1) & 1) * a.dm + tile * 16 + row] = xn;
        if (!last_layer) {
            const float* wnext = a.layers[l + 1].norm;
            const float xw = wnext ? xn * __ldg(wnext + tile * 16 + row) : xn;
            pack_rows<FA>(a.xtab + (size_t)((l + 1) & 1) * (G.tab_a / 8), tile, lane, xw, bad);
            const float s1 = sum16(xw), s2 = sum16(xn * xn);
            float* snext = a.xs + (size_t)((l + 1) & 1) * 2 * G.td;
            if (lane == 0) {
                snext[tile] = s1;
                snext[G.td + tile] = s2;
            }
        }
        __syncwarp();
        if (lane == 0) red_rel(cnt + kXcnt, 1u);
    }
    if (bad) atomicOr(a.err, 1);
}

// Tensor parallelism: the x-tile completer warp of CTA c finishes tiles c, c + C, ... of every
// layer once every rank's partial of the tile is in this rank's region (system-scope counter),
// adding them in rank order to the residual (the same sum on every rank), then stores x, the
// next layer's gate/up table entries and the tile's sums, and raises the layer's finished-tile
// counter.  It consumes no hand-over slot, so a finisher never waits on another GPU.
template <class FA, class FD>
__device__ void completer(const Args& a, const Geo<FA, FD>& G, int lane) {
    bool bad = false;
    const int row = lane & 15;
    const unsigned* ctr = reinterpret_cast<const unsigned*>(a.regions[a.tp_rank] + kPeerFlowTile);
    for (int l = 0; l < a.L; ++l) {
        unsigned* cnt = a.cnt + (size_t)l * a.cstride;
        const bool last_layer = l == a.L - 1;
        const unsigned target = (a.flow_base + (unsigned)l + 1u) * (unsigned)a.tp_size;
        const float* slots = reinterpret_cast<const float*>(a.regions[a.tp_rank] + kPeerTpParts) +
                             (size_t)((a.tp_base + l) & 1) * G.td * a.tp_size * 16;
        for (int tile = blockIdx.x; tile < G.td; tile += gridDim.x) {
            int ok = 1;
            if (lane == 0) {
                ok = wait_ge_sys(ctr + tile, target, a.err) ? 1 : 0;
                if (ok && l >= 2 && !last_layer)
                    ok = wait_ge(a.cnt + (size_t)(l - 1) * a.cstride + kCopied, gridDim.x, a.err) ? 1 : 0;
            }
            ok = __shfl_sync(kFull, ok, 0);
            __syncwarp();  // lane 0's acquire orders the other lanes' loads below
            if (!ok) {
                if (bad) atomicOr(a.err, 1);
                return;
            }
            const float* xprev = l == 0 ? a.x : a.xbuf + (size_t)(l & 1) * a.dm;
            float xn = __ldcg(xprev + tile * 16 + row);
            for (int q = 0; q < a.tp_size; ++q) xn += __ldcg(slots + ((size_t)tile * a.tp_size + q) * 16 + row);
            if (lane < 16) a.xbuf[(size_t)((l + 1) & 1) * a.dm + tile * 16 + row] = xn;
            if (!last_layer) {
                const float* wnext = a.layers[l + 1].norm;
                const float xw = wnext ? xn * __ldg(wnext + tile * 16 + row) : xn;
                pack_rows<FA>(a.xtab + (size_t)((l + 1) & 1) * (G.tab_a / 8), tile, lane, xw, bad);
                const float s1 = sum16(xw), s2 = sum16(xn * xn);
                float* snext = a.xs + (size_t)((l + 1) & 1) * 2 * G.td;
                if (lane == 0) {
                    snext[tile] = s1;
                    snext[G.td + tile] = s2;
                }
            }
            __syncwarp();
            if (lane == 0) red_rel(cnt + kXcnt, 1u);
        }
    }
    if (bad) atomicOr(a.err, 1);
}

template <class FA, class FD, bool TP>
__global__ void __launch_bounds__(TP ? kThreadsTP : kThreads, 1) ffn_flow_kernel(Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[32];
    __shared__ float s_inv;
    __shared__ int s_abort;
    __shared__ int s_fnext;  // next chunk index a finisher takes
    __shared__ Desc s_desc[kMaxS];
    const Geo<FA, FD> G(a.dm, a.ff);
    const Smem L = smem_layout<FA, FD>(a.dm, a.ff, a.S, a.slot_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_addr(smem);
    Ring r;
    r.full0 = bar0;
    r.empty0 = bar0 + 8 * kMaxS;
    const uint32_t xbar = bar0 + 16 * kMaxS, dbar0 = xbar + 8;
    const uint32_t tfull0 = dbar0 + 16, tfree0 = tfull0 + 8 * kNT;
    r.base = smem + L.ring;
    r.base_s = smem_addr(r.base);
    r.S = a.S;
    r.slot_bytes = a.slot_bytes;
    r.slot = r.round = 0;
    uint2* xt = reinterpret_cast<uint2*>(smem + L.tab_a);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    uint8_t* tab_d = smem + L.tab_d;
    uint2* zero = reinterpret_cast<uint2*>(smem + L.zero);
    float* stage = reinterpret_cast<float*>(smem + L.stage);
    float* red = reinterpret_cast<float*>(smem + L.red);
    Meta* meta = reinterpret_cast<Meta*>(smem + L.meta);

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.S; ++s) {
            mbar_init(r.full0 + 8 * s, 1);
            mbar_init(r.empty0 + 8 * s, kCW);
        }
        mbar_init(xbar, 1);
        mbar_init(dbar0, 1);
        mbar_init(dbar0 + 8, 1);
        for (int s = 0; s < kNT; ++s) {
            mbar_init(tfull0 + 8 * s, kCW);
            mbar_init(tfree0 + 8 * s, 1);
        }
        mbar_fence_init();
        s_abort = 0;
        s_fnext = 0;
    }
    for (int i = threadIdx.x; i < table_entries_per_block<FD>(1); i += blockDim.x) zero[i] = make_uint2(0u, 0u);
    __syncthreads();

    if (warp == kCW) {  // ------------------------------------------------ producer
        Prod P;
        P.r = r;
        P.dbar0 = dbar0;
        P.tab_d = tab_d;
        P.loads0 = P.loads1 = 0;
        P.last0 = P.last1 = -1;
        bool ok = true;
        for (int l = 0; l < a.L && ok; ++l) ok = produce_layer<FA, FD>(P, s_desc, a, G, l, lane);
        drain_ring(P.r, P.r.round * P.r.S + P.r.slot);
        // the last table copies landed
        if (P.loads0 > 0) mbar_wait(dbar0, (P.loads0 - 1) & 1);
        if (P.loads1 > 0) mbar_wait(dbar0 + 8, (P.loads1 - 1) & 1);
        if (!ok && lane == 0) atomicOr(a.err, 2);
        return;
    }
    if (TP && warp == kCW + 1 + kFW) {  // ----------------------------- x-tile completer
        completer<FA, FD>(a, G, lane);
        return;
    }
    if (warp > kCW) {  // ------------------------------------------------ finishers
        finisher<FA, FD, TP>(a, G, &s_fnext, tfull0, tfree0, red, meta, &s_inv, stage, lane);
        return;
    }

    // --------------------------------------------------------------------- consumers
    // A warp that meets a timeout stops working (aborted) and tells the CTA (s_abort), but
    // every consumer warp still passes every named barrier of every layer in the same order,
    // so no barrier can wait for a warp that left.  At a chunk's last stage every warp drops its
    // partial sums into hand-over slot k % kNT and arrives on the slot's barrier; a finisher warp
    // completes the chunk.
    constexpr int kStep = kCW * 32;
    const int mt = warp_matrix(warp, true), jj = warp % stage_blocks(true);
    static_assert(FA::kLaneShares && FD::kLaneShares, "hand-over partials assume lane-distributed formats");
    int k = 0;  // chunks handed over so far (the same count in every consumer warp)
    int dloads0 = 0, dloads1 = 0;  // down-table copies waited for, per table slot
    bool aborted = false, bad = false;
    float yA = 0.f, yB = 0.f;
    float pA[1][1] = {{0.f}}, pB[1][1] = {{0.f}};
    auto fail = [&]() {
        aborted = true;
        if (lane == 0) {
            atomicOr(a.err, 2);
            s_abort = 1;
        }
    };
    // hand the current chunk (or an end marker) to its finisher; false on timeout
    auto hand_over = [&](const Meta& m, bool partials) -> bool {
        const int ts = k % kNT, use = k / kNT;
        if (use > 0 && !mbar_wait(tfree0 + 8 * ts, (use - 1) & 1)) return false;
        if (partials) warp_partials<FA, 1>(red + (size_t)(ts * kCW + warp) * 16, lane >> 2, lane & 3, yA, yB, pA, pB);
        if (warp == 0 && lane == 0) meta[ts] = m;
        __syncwarp();
        if (lane == 0) mbar_arrive(tfull0 + 8 * ts);
        ++k;
        return true;
    };
    for (int l = 0; l < a.L; ++l) {
        const Layer ly = a.layers[l];
        unsigned* cnt = a.cnt + (size_t)l * a.cstride;
        // ---- gate/up prologue: the fragment table of x * w and 1 / rms(x)
        if (l == 0) {
            float ssq = 0.f;
            for (int c = threadIdx.x; c < a.dm / 4; c += kStep) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(a.x) + c);
                const float4 w = ly.norm ? __ldg(reinterpret_cast<const float4*>(ly.norm) + c)
                                         : make_float4(1.f, 1.f, 1.f, 1.f);
                ssq += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
                const float xs[4] = {v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w};
                const int slot = chunk_slot<FA>(c);
                pack_chunk(xs, xt[slot], xt[slot + FA::kLoOff], bad);
                if constexpr (FA::kNeedSx) {  // 8 consecutive chunks form one 32-element sub-block
                    float s = (xs[0] + xs[1]) + (xs[2] + xs[3]);
                    s += __shfl_xor_sync(kFull, s, 1);
                    s += __shfl_xor_sync(kFull, s, 2);
                    s += __shfl_xor_sync(kFull, s, 4);
                    if ((threadIdx.x & 7) == 0) sx[c >> 3] = s;
                }
            }
            const float tot = block_sum(ssq, s_red, kStep, kBarPro);
            if (threadIdx.x == 0) s_inv = ly.norm ? 1.0f / sqrtf(tot / (float)a.dm + a.eps) : 1.0f;
            named_bar_sync(kBarPro, kStep);
            if (threadIdx.x == 0) red_rel(cnt + kCopied, 1u);  // done reading the caller's x
        } else {
            // every warp is done with the previous layer's gate/up table before it is replaced
            named_bar_sync(kBarPro, kStep);
            if (threadIdx.x == 0 && !s_abort) {
                const unsigned* prev = a.cnt + (size_t)(l - 1) * a.cstride;
                bool ok = wait_ge(prev + kXcnt, (unsigned)G.td, a.err);
                if (ok) {
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_expect_tx(xbar, (uint32_t)(G.tab_a + 2 * G.td * 4));
                    bulk_g2s(smem_addr(xt), a.xtab + (size_t)(l & 1) * (G.tab_a / 8), (uint32_t)G.tab_a, xbar);
                    bulk_g2s(smem_addr(stage), a.xs + (size_t)(l & 1) * 2 * G.td, (uint32_t)(2 * G.td * 4), xbar);
                    ok = mbar_wait(xbar, (l - 1) & 1);
                    if (!ok) atomicOr(a.err, 2);
                }
                if (ok) red_rel(cnt + kCopied, 1u);  // the global table may be rewritten
                else s_abort = 1;
            }
            named_bar_sync(kBarPro, kStep);
            if (s_abort) aborted = true;
            // the copied per-tile sums serve the Q4_K units as they are (sx16), and the finishers
            // take 1 / rms from the copied sums of squares: nothing else to wait for
        }
        // ---- gate/up units (h is completed by the finishers)
        {
            LaneCtx<1> ctx = make_ctx<FA, 1>(xt, zero, l == 0 ? sx : stage, a.dm, lane);
            if (l > 0) {
                ctx.sx16 = 1;
                ctx.sxs = a.dm / 16;
            }
            while (!aborted) {
                if (!mbar_wait(r.full0 + 8 * r.slot, r.round & 1)) {
                    fail();
                    break;
                }
                const Desc d = s_desc[r.slot];
                if (d.flags & kPhaseEnd) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
                    r.advance();
                    break;
                }
                if (jj < d.n)
                    stage_unit<FA, 1>(r.base + r.slot * r.slot_bytes + (mt * stage_blocks(true) + jj) * FA::kTile,
                                      d.kb + jj, ctx, yA, yB, pA, pB);
                __syncwarp();
                if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
                r.advance();
                if ((d.flags & kLastOfChunk) && !hand_over(Meta{d.tile, -1, l, 0}, true)) {
                    fail();
                    break;
                }
            }
        }
        // ---- down units: K-part partial sums (the finishers complete x)
        {
            int dcur = -1;  // the table part the consumers hold (parts restart every layer)
            LaneCtx<1> ctx = make_ctx<FD, 1>(reinterpret_cast<uint2*>(tab_d), zero, nullptr, a.ff, lane);
            while (!aborted) {
                if (!mbar_wait(r.full0 + 8 * r.slot, r.round & 1)) {
                    fail();
                    break;
                }
                const Desc d = s_desc[r.slot];
                if (d.flags & kPhaseEnd) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
                    r.advance();
                    break;
                }
                if (d.part != dcur) {  // a new table part: wait for its copy
                    const int ts = d.part & 1;
                    const int nl = ts ? ++dloads1 : ++dloads0;
                    if (!mbar_wait(dbar0 + 8 * ts, (nl - 1) & 1)) {
                        fail();
                        break;
                    }
                    ctx = make_ctx<FD, 1>(reinterpret_cast<uint2*>(tab_d + ts * G.tab_p), zero, nullptr, a.ff, lane);
                    dcur = d.part;
                }
                if (warp < d.n)
                    stage_unit<FD, 1>(r.base + r.slot * r.slot_bytes + warp * FD::kTile,
                                      d.kb - d.part * G.pb + warp, ctx, yA, yB, pA, pB);
                __syncwarp();
                if (lane == 0) mbar_arrive(r.empty0 + 8 * r.slot);
                r.advance();
                if ((d.flags & kLastOfChunk) && !hand_over(Meta{d.tile, d.part, l, 0}, true)) {
                    fail();
                    break;
                }
            }
        }
    }
    // ---- end markers (one per finisher), then x_L (in xbuf[L & 1]) into the caller's x once
    // every tile is final and every CTA has read x_0
    if (!aborted) {
        for (int f = 0; f < kFW && !aborted; ++f)
            if (!hand_over(Meta{0, 0, 0, 1}, false)) fail();
    }
    named_bar_sync(kBarPro, kStep);
    if (threadIdx.x == 0 && !s_abort) {
        bool ok = wait_ge(a.cnt + (size_t)(a.L - 1) * a.cstride + kXcnt, (unsigned)G.td, a.err);
        if (ok) ok = wait_ge(a.cnt + kCopied, gridDim.x, a.err);
        if (!ok) s_abort = 1;
    }
    named_bar_sync(kBarPro, kStep);
    if (!s_abort) {
        const float4* src = reinterpret_cast<const float4*>(a.xbuf + (size_t)(a.L & 1) * a.dm);
        const int n4 = a.dm / 4, C = gridDim.x;
        const int c0 = (int)((long long)blockIdx.x * n4 / C), c1 = (int)((long long)(blockIdx.x + 1) * n4 / C);
        for (int c = c0 + (int)threadIdx.x; c < c1; c += kStep) reinterpret_cast<float4*>(a.x)[c] = __ldcg(src + c);
    }
    if (bad) atomicOr(a.err, 1);
}

}  // namespace flow

// ------------------------------------------------------------------ host side
namespace {

struct FlowScratch {
    size_t cnt, xbuf, parts, htab, xtab, xs, total;
    int cstride;
};

template <class FA, class FD>
FlowScratch flow_scratch(int L, int dm, int ff) {
    const flow::Geo<FA, FD> G(dm, ff);
    FlowScratch s;
    s.cstride = (flow::kHcnt + G.np + G.td + 31) & ~31;
    size_t off = 0;
    auto take = [&off](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 255) & ~(size_t)255;
        return o;
    };
    s.cnt = take((size_t)L * s.cstride * 4);
    s.xbuf = take(2 * (size_t)dm * 4);
    s.parts = take((size_t)G.td * G.np * 16 * 4);
    s.htab = take((size_t)G.np * G.tab_p);
    s.xtab = take(2 * (size_t)G.tab_a);
    s.xs = take(2 * 2 * (size_t)G.td * 4);
    s.total = off;
    return s;
}

template <class FA, class FD>
cudaError_t launch_flow_t(const StackLaunch& s, int num_sms, int smem_limit, cudaStream_t stream, bool dry,
                          size_t* scratch_bytes) {
    using namespace flow;
    const bool tp = s.tp_size > 1;
    if (s.dm % FA::kBlockElems || s.ff % (FD::kBlockElems) || s.dm % 256 || s.ff % 256)
        return cudaErrorInvalidConfiguration;
    if (tp) {  // the exchange: per-tile counters and the double-buffered tile partials
        const Geo<FA, FD> g(s.dm, s.ff);
        if (s.tp_size > 8 || (size_t)g.td * 4 > kPeerTpParts - kPeerFlowTile ||
            (size_t)2 * g.td * s.tp_size * 16 * 4 > kPeerTpPartsBytes)
            return cudaErrorInvalidConfiguration;
    }
    (void)num_sms;  // any shape: CTAs without chunks of a phase pass its end marker
    // ring: slots of the larger stage; down stages of dsb blocks (16, else 12 or 8 to keep 3 slots)
    const int sa = 2 * stage_blocks(true) * FA::kTile;
    int dsb = 16, S = 0, slot = 0;
    for (; dsb >= 8; dsb -= 4) {
        slot = sa > dsb * FD::kTile ? sa : dsb * FD::kTile;
        const int fixed = smem_layout<FA, FD>(s.dm, s.ff, 0, slot).ring + 1024;  // + static shared
        S = (smem_limit - fixed) / slot;
        if (S > kMaxS) S = kMaxS;
        if (S >= 3) break;
    }
    if (S < 3) return cudaErrorInvalidConfiguration;
    const Smem L = smem_layout<FA, FD>(s.dm, s.ff, S, slot);
    auto kern = tp ? ffn_flow_kernel<FA, FD, true> : ffn_flow_kernel<FA, FD, false>;
    const int threads = tp ? kThreadsTP : kThreads;
    // the shared-memory opt-in and the one-CTA-per-SM check, once per kernel, device and size
    // (a stack call makes two launches of this function: the driver queries cost microseconds)
    static int checked[2][64];  // [tp][device]: the largest size configured and found to fit
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || checked[tp][dev] < L.total) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, L.total);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
        if (dev < 64) checked[tp][dev] = L.total;
    }
    const FlowScratch sc = flow_scratch<FA, FD>(s.L, s.dm, s.ff);
    if (dry) {
        if (scratch_bytes) *scratch_bytes = sc.total;
        return cudaSuccess;
    }
    uint8_t* base = static_cast<uint8_t*>(s.scratch);
    Args a{};
    a.layers = reinterpret_cast<const Layer*>(s.layers);
    a.L = s.L;
    a.dm = s.dm;
    a.ff = s.ff;
    a.ts_a = s.ts_a;
    a.ts_b = s.ts_b;
    a.x = s.x;
    a.xbuf = reinterpret_cast<float*>(base + sc.xbuf);
    a.parts = reinterpret_cast<float*>(base + sc.parts);
    a.htab = reinterpret_cast<uint2*>(base + sc.htab);
    a.xtab = reinterpret_cast<uint2*>(base + sc.xtab);
    a.xs = reinterpret_cast<float*>(base + sc.xs);
    a.cnt = reinterpret_cast<unsigned*>(base + sc.cnt);
    a.cstride = sc.cstride;
    a.eps = s.eps;
    a.err = s.err;
    a.S = S;
    a.slot_bytes = slot;
    a.dsb = dsb;
    a.regions = reinterpret_cast<char* const*>(s.tp_regions);
    a.tp_rank = tp ? s.tp_rank : 0;
    a.tp_size = tp ? s.tp_size : 1;
    a.tp_base = s.tp_base;
    a.flow_base = s.tp_flow_base;
    e = cudaMemsetAsync(a.cnt, 0, (size_t)s.L * sc.cstride * 4, stream);
    if (e != cudaSuccess) return e;
    void* args[] = {&a};
    e = cudaLaunchCooperativeKernel((const void*)kern, dim3(num_sms), dim3(threads), args, L.total, stream);
    if (e == cudaSuccess && s.flow_used) *s.flow_used = 1;
    return e;
}

}  // namespace

// The dataflow stack kernel covers stacks with a Q6_K down projection and Q4_K or Q6_K gate/up
// (d_model and d_ff whole super-blocks), on one GPU or tensor-parallel over up to 8;
// cudaErrorInvalidConfiguration otherwise.
cudaError_t launch_ffn_flow(int type_a, int type_d, const StackLaunch& s, int num_sms, int smem_limit,
                            cudaStream_t stream, bool dry, size_t* scratch_bytes) {
    if (type_d != T_Q6_K) return cudaErrorInvalidConfiguration;
    if (type_a == T_Q4_K) return launch_flow_t<FmtQ4K, FmtQ6K>(s, num_sms, smem_limit, stream, dry, scratch_bytes);
    if (type_a == T_Q6_K) return launch_flow_t<FmtQ6K, FmtQ6K>(s, num_sms, smem_limit, stream, dry, scratch_bytes);
    return cudaErrorInvalidConfiguration;
}

}  // namespace hc
