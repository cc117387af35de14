// gemv_simple.cu -- CUDA-core kernels on the raw GGUF layout: F32, the IQ2/IQ3 codebook
// formats, the toy LUT-Q4 matmul, and the elementwise SwiGLU combine.
//
// Reference semantics: gemv_f32 (crates/hayai-model/src/quant.rs:358-369), the IQ2 block
// decoders (crates/hayai-model/src/iq2.rs:504-573, gemv macro :591-626), the IQ3 block
// decoders (crates/hayai-model/src/iq3.rs:147-220, gemv :258-331), cpu_lut_matmul_q4
// (crates/hayai-cpu/src/matmul.rs:48-82).
#include "common.cuh"
#include "gemv_launch.h"

#define HC_IQ_QUAL static __device__ const
#include "_gen/iq_tables.h"

namespace hc {

// Sign byte of a 7-bit index: the index with bit 7 = its parity (iq2.rs:18-27).
__device__ __forceinline__ uint32_t ksigns(uint32_t i) { return (i & 127u) | ((__popc(i & 127u) & 1u) << 7); }

__device__ __forceinline__ uint32_t ldb(const uint8_t* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t ld_u16u(const uint8_t* p) { return ldb(p) | (ldb(p + 1) << 8); }
__device__ __forceinline__ uint32_t ld_u32u(const uint8_t* p) { return ld_u16u(p) | (ld_u16u(p + 2) << 16); }
__device__ __forceinline__ float ld_f16u(const uint8_t* p) { return h2f((uint16_t)ld_u16u(p)); }

// sum over 8 codebook values: db * g_j * sign_j * x_j
__device__ __forceinline__ float dot8_grid(float db, uint64_t grid, uint32_t signs, const float* x) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float g = (float)((grid >> (8 * j)) & 0xffu);
        const float v = (signs >> j) & 1u ? -db * g : db * g;
        s += v * x[j];
    }
    return s;
}

__device__ __forceinline__ float dot4_grid(float db, uint32_t grid, uint32_t signs, const float* x) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float g = (float)((grid >> (8 * j)) & 0xffu);
        const float v = (signs >> j) & 1u ? -db * g : db * g;
        s += v * x[j];
    }
    return s;
}

// One 32-element group (ib32) of an IQ block, dotted with x[0..32).
template <int TYPE>
__device__ __forceinline__ float iq_group_dot(const uint8_t* blk, int ib32, const float* x) {
    const float d = ld_f16u(blk);
    float s = 0.f;
    if constexpr (TYPE == T_IQ2_XXS) {
        const uint32_t aux0 = ld_u32u(blk + 2 + 8 * ib32), aux1 = ld_u32u(blk + 2 + 8 * ib32 + 4);
        const float db = d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
#pragma unroll
        for (int l = 0; l < 4; ++l)
            s += dot8_grid(db, hc_iq2xxs_grid[(aux0 >> (8 * l)) & 0xff], ksigns(aux1 >> (7 * l)), x + 8 * l);
    } else if constexpr (TYPE == T_IQ2_XS) {
        const uint32_t sc = ldb(blk + 66 + ib32);
        const float db0 = d * (0.5f + (float)(sc & 0xf)) * 0.25f, db1 = d * (0.5f + (float)(sc >> 4)) * 0.25f;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t q = ld_u16u(blk + 2 + 2 * (4 * ib32 + l));
            s += dot8_grid(l < 2 ? db0 : db1, hc_iq2xs_grid[q & 511], ksigns(q >> 9), x + 8 * l);
        }
    } else if constexpr (TYPE == T_IQ2_S) {
        const uint32_t sc = ldb(blk + 74 + ib32), qh = ldb(blk + 66 + ib32);
        const float db0 = d * (0.5f + (float)(sc & 0xf)) * 0.25f, db1 = d * (0.5f + (float)(sc >> 4)) * 0.25f;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t idx = ldb(blk + 2 + 4 * ib32 + l) | ((qh << (8 - 2 * l)) & 0x300u);
            s += dot8_grid(l < 2 ? db0 : db1, hc_iq2s_grid[idx], ldb(blk + 34 + 4 * ib32 + l), x + 8 * l);
        }
    } else if constexpr (TYPE == T_IQ3_XXS) {
        const uint32_t aux = ld_u32u(blk + 66 + 4 * ib32);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t sg = ksigns(aux >> (7 * l));
            s += dot4_grid(db, hc_iq3xxs_grid[ldb(blk + 2 + 8 * ib32 + 2 * l)], sg, x + 8 * l);
            s += dot4_grid(db, hc_iq3xxs_grid[ldb(blk + 2 + 8 * ib32 + 2 * l + 1)], sg >> 4, x + 8 * l + 4);
        }
    } else if constexpr (TYPE == T_IQ3_S) {
        const uint32_t sc = ldb(blk + 106 + ib32 / 2), qh = ldb(blk + 66 + ib32);
        const float db = d * (1.0f + 2.0f * (float)((sc >> (4 * (ib32 & 1))) & 0xf));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t i1 = ldb(blk + 2 + 8 * ib32 + 2 * l) | ((qh << (8 - 2 * l)) & 256u);
            const uint32_t i2 = ldb(blk + 2 + 8 * ib32 + 2 * l + 1) | ((qh << (7 - 2 * l)) & 256u);
            const uint32_t sg = ldb(blk + 74 + 4 * ib32 + l);
            s += dot4_grid(db, hc_iq3s_grid[i1], sg, x + 8 * l);
            s += dot4_grid(db, hc_iq3s_grid[i2], sg >> 4, x + 8 * l + 4);
        }
    }
    return s;
}

template <int TYPE, int BLK>
__global__ void __launch_bounds__(256) gemv_iq_kernel(const uint8_t* __restrict__ w, size_t row_bytes, int M,
                                                       int K, const float* __restrict__ x, int ldx,
                                                       float* __restrict__ y, int ldy, const float* resid, int ldr,
                                                       int nvec) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int nb = K / 256;
    for (int rv = warp; rv < M * nvec; rv += nwarps) {
        const int row = rv % M, v = rv / M;
        const uint8_t* wr = w + (size_t)row * row_bytes;
        const float* xv = x + (size_t)v * ldx;
        float s = 0.f;
        for (int gi = lane; gi < nb * 8; gi += 32) {
            const int b = gi >> 3, ib32 = gi & 7;
            float xs[32];
            const float4* xp = reinterpret_cast<const float4*>(xv + b * 256 + 32 * ib32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 a = __ldg(xp + q);
                xs[4 * q] = a.x;
                xs[4 * q + 1] = a.y;
                xs[4 * q + 2] = a.z;
                xs[4 * q + 3] = a.w;
            }
            s += iq_group_dot<TYPE>(wr + (size_t)b * BLK, ib32, xs);
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

static int grid_for(int work_warps) {
    int blocks = (work_warps + 7) / 8;
    return blocks < 1 ? 1 : (blocks > 65535 ? 65535 : blocks);
}

bool gemv_simple_supported(int type) {
    return type == T_F32 || type == T_IQ2_XXS || type == T_IQ2_XS || type == T_IQ2_S || type == T_IQ3_XXS ||
           type == T_IQ3_S;
}

cudaError_t launch_gemv_simple(int type, const uint8_t* w, size_t row_bytes, int M, int K, const float* x, int ldx,
                               float* y, int ldy, const float* resid, int ldr, int nvec, cudaStream_t stream) {
    const int grid = grid_for(M * nvec);
    switch (type) {
        case T_F32:
            gemv_f32_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float*>(w), row_bytes / 4, M, K, x, ldx,
                                                      y, ldy, resid, ldr, nvec);
            break;
        case T_IQ2_XXS:
            gemv_iq_kernel<T_IQ2_XXS, 66><<<grid, 256, 0, stream>>>(w, row_bytes, M, K, x, ldx, y, ldy, resid, ldr, nvec);
            break;
        case T_IQ2_XS:
            gemv_iq_kernel<T_IQ2_XS, 74><<<grid, 256, 0, stream>>>(w, row_bytes, M, K, x, ldx, y, ldy, resid, ldr, nvec);
            break;
        case T_IQ2_S:
            gemv_iq_kernel<T_IQ2_S, 82><<<grid, 256, 0, stream>>>(w, row_bytes, M, K, x, ldx, y, ldy, resid, ldr, nvec);
            break;
        case T_IQ3_XXS:
            gemv_iq_kernel<T_IQ3_XXS, 98><<<grid, 256, 0, stream>>>(w, row_bytes, M, K, x, ldx, y, ldy, resid, ldr, nvec);
            break;
        case T_IQ3_S:
            gemv_iq_kernel<T_IQ3_S, 110><<<grid, 256, 0, stream>>>(w, row_bytes, M, K, x, ldx, y, ldy, resid, ldr, nvec);
            break;
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
                                                      float* __restrict__ y) {
    __shared__ float lut[16];
    if (threadIdx.x < 16) lut[threadIdx.x] = lut16[threadIdx.x];
    __syncthreads();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int pc = N / 2;
    for (int row = warp; row < M; row += nwarps) {
        const uint8_t* wr = w + (size_t)row * pc;
        float s = 0.f;
        for (int c = lane; c < pc; c += 32) {
            const uint32_t b = __ldg(wr + c);
            s += __ldg(x + 2 * c) * lut[b & 15] + __ldg(x + 2 * c + 1) * lut[b >> 4];
        }
        s = warp_sum(s);
        if (lane == 0) y[row] = s;
    }
}

cudaError_t launch_lut_matmul_q4(const uint8_t* w, int M, int N, const float* lut16, const float* x, float* y,
                                 cudaStream_t stream) {
    lut_q4_kernel<<<grid_for(M), 256, 0, stream>>>(w, M, N, lut16, x, y);
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
