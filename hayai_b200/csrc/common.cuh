// common.cuh -- device helpers shared by the hayai_b200 kernels (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef __CUDACC__
#error "common.cuh is CUDA-only"
#endif

namespace hc {

// GgmlType ids (reference: crates/hayai-model/src/gguf_types.rs:6-40).
enum GgmlType : int {
    T_F32 = 0,
    T_Q4_0 = 2,
    T_Q4_1 = 3,
    T_Q5_0 = 6,
    T_Q5_1 = 7,
    T_Q8_0 = 8,
    T_Q2_K = 10,
    T_Q3_K = 11,
    T_Q4_K = 12,
    T_Q5_K = 13,
    T_Q6_K = 14,
    T_IQ2_XXS = 16,
    T_IQ2_XS = 17,
    T_IQ3_XXS = 18,
    T_IQ4_NL = 20,
    T_IQ3_S = 21,
    T_IQ2_S = 22,
    T_IQ4_XS = 23,
    T_F16 = 1,
    T_Q8_1 = 9,
    T_Q8_K = 15,
    T_BF16 = 30,
};

constexpr int QK_K = 256;

// The IQ2 / IQ3 codebook formats (tile-major layout, tensor-core GEMV).
__host__ __device__ constexpr bool is_iq_type(int t) {
    return t == T_IQ2_XXS || t == T_IQ2_XS || t == T_IQ2_S || t == T_IQ3_XXS || t == T_IQ3_S;
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// ---------------------------------------------------------------- loads
// Weights are streamed once per call: do not let them evict the activation
// working set from L1.
__device__ __forceinline__ uint4 ldg_stream128(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ldg_stream32(const void* p) {
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
    uint16_t r;
    asm("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ldg_u2(const void* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }

// ---------------------------------------------------------------- f16 packing
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    return h2_as_u32(__floats2half2_rn(lo, hi));
}

// x = hi + lo * 2^-11 with hi, lo in f16: hi = f16(x), lo = f16((x - hi) * 2^11).
// The residual is pre-scaled by 2^11 so it stays a normal f16 whenever x does,
// which gives ~22 significant bits for |x| < 65504.
__device__ __forceinline__ void split_f16(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn((x - __half2float(hi)) * 2048.0f);
}

// ---------------------------------------------------------------- byte tricks
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    // (a & mask) | orv  as one LOP3
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
    return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    return h2_as_u32(__hfma2(u32_as_h2(a), u32_as_h2(b), u32_as_h2(c)));
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    return h2_as_u32(__hsub2(u32_as_h2(a), u32_as_h2(b)));
}

// Unsigned byte `byte` of `word` as f32 without the conversion pipe: the byte becomes the low
// mantissa bits of 2^23 (one PRMT) and one FADD removes 2^23.  Exact.
__device__ __forceinline__ float u8_to_f32(uint32_t word, int byte) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(word), "r"(0x4B000000u), "r"(0x7440u | (uint32_t)byte));
    return __uint_as_float(d) - 8388608.0f;
}

// Signed byte `byte` of `word` as f32, without the conversion pipe: the byte, offset to
// unsigned, becomes the low mantissa bits of 2^23 (one PRMT on 0x80-flipped bytes), and one
// FADD removes 2^23 + 128.  Exact for every int8.  `flipped` = word ^ 0x80808080.
__device__ __forceinline__ float s8_to_f32_flipped(uint32_t flipped, int byte) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(flipped), "r"(0x4B000000u), "r"(0x7440u | (uint32_t)byte));
    return __uint_as_float(d) - 8388736.0f;
}

// ---------------------------------------------------------------- tensor core
// D = A(16x16 f16, row) * B(16x8 f16, col) + C, f32 accumulate.
// Fragment layout (PTX ISA, mma.m16n8k16): lane = 4*g + t;
//   A regs: {row g, k 2t..2t+1}, {row g+8, k 2t..2t+1}, {row g, k 2t+8..}, {row g+8, k 2t+8..}
//   B regs: {k 2t..2t+1, col g}, {k 2t+8..2t+9, col g}
//   C regs: (row g, col 2t), (row g, col 2t+1), (row g+8, col 2t), (row g+8, col 2t+1)
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(  // pure: no memory side effects, free to be scheduled around the loads
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- async copies
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy that bypasses L1 (weights are read once).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Wait until at most n of this thread's committed groups are still pending (n in [0, 7]).
__device__ __forceinline__ void cp_async_wait(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
        case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
    }
}

// ---------------------------------------------------------------- mbarrier + bulk copy (TMA)
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// One bounded probe: true once the phase with parity `parity` has completed.  Each probe
// may suspend the thread for up to ~10 us.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 10000;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait (<= ~2^17 probes, about a second): false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < (1 << 17); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Bounded wait by polling (non-blocking probes, no suspension): for handoffs that are usually
// not complete yet when the wait starts, where a suspended thread's wake-up would add latency.
// ~2^25 probes: about a second.  False on timeout.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < (1 << 25); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Global -> shared bulk copy through the TMA engine, completing `bytes` on mbarrier `bar`.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    // crates/hayai-core/src/stream_infer.rs:3836-3840: (g / (1 + exp(-g))) * u
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))) * u;
}

}  // namespace hc
