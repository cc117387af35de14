// repack.cu -- one-time upload transform from raw GGUF rows to the GPU layouts.
//
// GGUF Q6_K (210 B) and Q8_0 (34 B) blocks are only 2-byte aligned inside a row, which
// rules out 128-bit loads.  At upload the rows are rewritten (same byte count, or a
// few bytes of padding per row) so that every lane of the tensor-core GEMV reads its
// codes with 16-byte vector loads:
//
//  Q6_K row:  nb x 208 B {ql_perm[4][8 words] | qh_perm[4][4 words] | scales[16]}
//             + d plane (nb f16, padded to 16 B).
//             ql word (t, wq=4h+2qq+lh) = ql bytes 64h+32qq+16lh+4t..+3
//             qh word (t, wh=2h+lh)     = qh bytes 32h+16lh+4t..+3
//  Q8_0 row:  ng = ceil(nb/4) groups x 128 B {qs_perm[4][8 words]} + d plane (4 f16 per
//             group, padded to 16 B).  word (t, w) = codes 16(w&1)+4t..+3 of block 4G+w/2;
//             missing blocks of the last group are zero (d = 0).
//  Q4_K, F32, IQ*: raw layout (Q4_K's 144 B blocks are already 16-byte aligned).
//
// Layout of the GGUF blocks: q6k.rs:26-57 (ql/qh/scales/d), quant.rs:598-615 (Q8_0).
#include "common.cuh"
#include "gemv_launch.h"

namespace hc {

static inline size_t pad16(size_t b) { return (b + 15) / 16 * 16; }

size_t raw_row_bytes(int type, int K) {
    switch (type) {
        case T_F32: return (size_t)K * 4;
        case T_Q8_0: return (size_t)K / 32 * 34;
        case T_Q4_K: return (size_t)K / 256 * 144;
        case T_Q6_K: return (size_t)K / 256 * 210;
        case T_IQ2_XXS: return (size_t)K / 256 * 66;
        case T_IQ2_XS: return (size_t)K / 256 * 74;
        case T_IQ2_S: return (size_t)K / 256 * 82;
        case T_IQ3_XXS: return (size_t)K / 256 * 98;
        case T_IQ3_S: return (size_t)K / 256 * 110;
        default: return 0;
    }
}

size_t gpu_row_stride(int type, int K) {
    if (type == T_Q6_K) {
        const size_t nb = (size_t)K / 256;
        return nb * 208 + pad16(nb * 2);
    }
    if (type == T_Q8_0) {
        const size_t ng = ((size_t)K / 32 + 3) / 4;
        return ng * 128 + pad16(ng * 8);
    }
    return raw_row_bytes(type, K);
}

__device__ __forceinline__ uint32_t rd4(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// one thread per destination 32-bit word of the block area, plus one per d entry
__global__ void repack_q6k_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ gpu, int M, int nb,
                                  size_t raw_rb, size_t gpu_rb) {
    const size_t total = (size_t)M * nb * 53;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int w = (int)(i % 53);
        const size_t rb = i / 53;
        const int b = (int)(rb % nb);
        const size_t row = rb / nb;
        const uint8_t* src = raw + row * raw_rb + (size_t)b * 210;
        uint8_t* dst = gpu + row * gpu_rb + (size_t)b * 208;
        if (w < 32) {
            const int t = w >> 3, wq = w & 7, h = wq >> 2, qq = (wq >> 1) & 1, lh = wq & 1;
            *reinterpret_cast<uint32_t*>(dst + 32 * t + 4 * wq) = rd4(src + 64 * h + 32 * qq + 16 * lh + 4 * t);
        } else if (w < 48) {
            const int j = w - 32, t = j >> 2, wh = j & 3, h = wh >> 1, lh = wh & 1;
            *reinterpret_cast<uint32_t*>(dst + 128 + 16 * t + 4 * wh) = rd4(src + 128 + 32 * h + 16 * lh + 4 * t);
        } else if (w < 52) {
            const int j = w - 48;
            *reinterpret_cast<uint32_t*>(dst + 192 + 4 * j) = rd4(src + 192 + 4 * j);
        } else {
            uint8_t* dp = gpu + row * gpu_rb + (size_t)nb * 208 + 2 * b;
            dp[0] = src[208];
            dp[1] = src[209];
        }
    }
}

__global__ void repack_q80_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ gpu, int M, int nb, int ng,
                                  size_t raw_rb, size_t gpu_rb) {
    const size_t total = (size_t)M * ng * 36;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int w = (int)(i % 36);
        const size_t rg = i / 36;
        const int G = (int)(rg % ng);
        const size_t row = rg / ng;
        const uint8_t* srow = raw + row * raw_rb;
        uint8_t* drow = gpu + row * gpu_rb;
        if (w < 32) {
            const int t = w >> 3, wi = w & 7, blk = 4 * G + (wi >> 1), half = wi & 1;
            uint32_t v = 0;
            if (blk < nb) v = rd4(srow + (size_t)blk * 34 + 2 + 16 * half + 4 * t);
            *reinterpret_cast<uint32_t*>(drow + (size_t)G * 128 + 32 * t + 4 * wi) = v;
        } else {
            const int blk = 4 * G + (w - 32);
            uint8_t* dp = drow + (size_t)ng * 128 + 2 * blk;
            dp[0] = blk < nb ? srow[(size_t)blk * 34] : 0;
            dp[1] = blk < nb ? srow[(size_t)blk * 34 + 1] : 0;
        }
    }
}

cudaError_t launch_repack(int type, const uint8_t* raw, uint8_t* gpu, int M, int K, cudaStream_t stream) {
    const size_t rrb = raw_row_bytes(type, K), grb = gpu_row_stride(type, K);
    if (type == T_Q6_K) {
        const int nb = K / 256;
        // zero the d-plane padding first
        cudaError_t e = cudaMemsetAsync(gpu, 0, (size_t)M * grb, stream);
        if (e != cudaSuccess) return e;
        const size_t total = (size_t)M * nb * 53;
        const unsigned blocks = (unsigned)((total + 255) / 256 < 65535 * 8 ? (total + 255) / 256 : 65535 * 8);
        repack_q6k_kernel<<<blocks, 256, 0, stream>>>(raw, gpu, M, nb, rrb, grb);
        return cudaGetLastError();
    }
    if (type == T_Q8_0) {
        const int nb = K / 32, ng = (nb + 3) / 4;
        cudaError_t e = cudaMemsetAsync(gpu, 0, (size_t)M * grb, stream);
        if (e != cudaSuccess) return e;
        const size_t total = (size_t)M * ng * 36;
        const unsigned blocks = (unsigned)((total + 255) / 256 < 65535 * 8 ? (total + 255) / 256 : 65535 * 8);
        repack_q80_kernel<<<blocks, 256, 0, stream>>>(raw, gpu, M, nb, ng, rrb, grb);
        return cudaGetLastError();
    }
    return cudaMemcpyAsync(gpu, raw, (size_t)M * rrb, cudaMemcpyDeviceToDevice, stream);
}

}  // namespace hc
