// synth.cu -- seeded synthetic inputs and weight quantizers on the device.
//
// quantize_q4_k restates the reference quantizer (crates/hayai-model/src/q4k.rs:85-160,
// f32_to_f16 :46-79) bit-exactly: every f32 operation is written with explicit
// round-to-nearest intrinsics so the compiler cannot contract them into FMAs.  The Q6_K
// and Q8_0 quantizers are this project's own (the reference ships none); the CPU oracle
// holds the same rules.  The normal generator evaluates splitmix64 at a position and
// applies Box-Muller in double precision, like the oracle's or_fill_normal.
#include "../../include/hayai_cuda.h"
#include "common.cuh"
#include "engine.h"

using namespace hc;

namespace hc {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void synth_normal_kernel(uint64_t seed, size_t n, float mean, float stdv, float* __restrict__ out) {
    const uint64_t key = mix64(seed);
    const size_t pairs = (n + 1) / 2;
    for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < pairs; p += (size_t)gridDim.x * blockDim.x) {
        const uint64_t a = mix64(key + (2 * p + 1) * 0x9E3779B97F4A7C15ull);
        const uint64_t b = mix64(key + (2 * p + 2) * 0x9E3779B97F4A7C15ull);
        const double u1 = ((double)(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        const double u2 = ((double)(b >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        const double r = sqrt(-2.0 * log(u1));
        double s, c;
        sincospi(2.0 * u2, &s, &c);
        out[2 * p] = (float)((double)mean + (double)stdv * (r * c));
        if (2 * p + 1 < n) out[2 * p + 1] = (float)((double)mean + (double)stdv * (r * s));
    }
}

// q4k.rs:46-79
__device__ uint16_t f32_to_f16_ref(float value) {
    const uint32_t f = __float_as_uint(value);
    const uint32_t sign = (f >> 16) & 0x8000u;
    int exponent = (int)((f >> 23) & 0xffu) - 127 + 15;
    const uint32_t mantissa = f & 0x7fffffu;
    if (exponent <= 0) {
        if (exponent < -10) return (uint16_t)sign;
        uint32_t m = mantissa | 0x800000u;
        const uint32_t shift = (uint32_t)(14 - exponent);
        m >>= shift;
        const uint32_t sb = shift > 0 ? shift - 1 : 0;
        if (mantissa & (1u << sb)) m += 1;
        return (uint16_t)(sign | m);
    }
    if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t m = mantissa >> 13;
    if (mantissa & 0x1000u) m += 1;
    if ((m & 0x400u) == 0x400u) {
        m = 0;
        exponent += 1;
    }
    if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)exponent << 10) | m);
}

__device__ __forceinline__ float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// q4k.rs:98-160, one thread per 256-element block
__global__ void quantize_q4k_kernel(const float* __restrict__ x, size_t nblk, uint8_t* __restrict__ out) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblk; b += (size_t)gridDim.x * blockDim.x) {
        const float* xb = x + b * 256;
        uint8_t* o = out + b * 144;
        float scales[8], mins[8];
        for (int j = 0; j < 8; ++j) {
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 32; ++i) {
                const float v = xb[j * 32 + i];
                mn = fminf(mn, v);
                mx = fmaxf(mx, v);
            }
            scales[j] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
            mins[j] = mn;
        }
        float max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; ++j) max_scale = fmaxf(max_scale, scales[j]);
        max_scale = fmaxf(max_scale, 1e-30f);
        for (int j = 0; j < 8; ++j) max_min = fmaxf(max_min, fabsf(mins[j]));
        max_min = fmaxf(max_min, 1e-30f);
        const float d = __fdiv_rn(max_scale, 63.0f), dmin = __fdiv_rn(max_min, 63.0f);
        uint8_t ls[8], lm[8];
        for (int j = 0; j < 8; ++j) {
            ls[j] = (uint8_t)clampf(roundf(__fdiv_rn(__fmul_rn(scales[j], 63.0f), max_scale)), 0.0f, 63.0f);
            lm[j] = (uint8_t)clampf(roundf(__fdiv_rn(__fmul_rn(-mins[j], 63.0f), max_min)), 0.0f, 63.0f);
        }
        uint8_t sp[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 8; ++j) {
            const uint8_t sc = ls[j], m = lm[j];
            if (j < 4) {
                sp[j] = sc;
                sp[j + 4] = m;
            } else {
                sp[j + 4] = (uint8_t)((sc & 0xF) | ((m & 0xF) << 4));
                sp[j - 4] |= (uint8_t)((sc >> 4) << 6);
                sp[j] |= (uint8_t)((m >> 4) << 6);
            }
        }
        const uint16_t hd = f32_to_f16_ref(d), hm = f32_to_f16_ref(dmin);
        o[0] = (uint8_t)(hd & 0xff);
        o[1] = (uint8_t)(hd >> 8);
        o[2] = (uint8_t)(hm & 0xff);
        o[3] = (uint8_t)(hm >> 8);
        for (int i = 0; i < 12; ++i) o[4 + i] = sp[i];
        for (int c = 0; c < 4; ++c) {
            const int j0 = 2 * c, j1 = 2 * c + 1;
            const float d1a = __fmul_rn(d, (float)ls[j0]), d1b = __fmul_rn(d, (float)ls[j1]);
            const float dma = __fmul_rn(dmin, (float)lm[j0]), dmb = __fmul_rn(dmin, (float)lm[j1]);
            for (int ii = 0; ii < 32; ++ii) {
                uint8_t qa = 0, qb = 0;
                if (d1a != 0.0f) qa = (uint8_t)clampf(roundf(__fdiv_rn(__fadd_rn(xb[j0 * 32 + ii], dma), d1a)), 0.f, 15.f);
                if (d1b != 0.0f) qb = (uint8_t)clampf(roundf(__fdiv_rn(__fadd_rn(xb[j1 * 32 + ii], dmb), d1b)), 0.f, 15.f);
                o[16 + 32 * c + ii] = (uint8_t)(qa | (qb << 4));
            }
        }
    }
}

// Project Q6_K quantizer (same rule as the oracle's or_quantize_q6_k).
__global__ void quantize_q6k_kernel(const float* __restrict__ x, size_t nblk, uint8_t* __restrict__ out) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblk; b += (size_t)gridDim.x * blockDim.x) {
        const float* xb = x + b * 256;
        uint8_t* o = out + b * 210;
        float gs[16], maxs = 0.0f;
        for (int g = 0; g < 16; ++g) {
            float am = 0.0f;
            for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(xb[g * 16 + i]));
            gs[g] = __fdiv_rn(am, 31.0f);
            maxs = fmaxf(maxs, gs[g]);
        }
        maxs = fmaxf(maxs, 1e-30f);
        const uint16_t hd = f32_to_f16_ref(__fdiv_rn(maxs, 127.0f));
        const float dq = __half2float(__ushort_as_half(hd));
        for (int i = 0; i < 210; ++i) o[i] = 0;
        int8_t ls[16];
        for (int g = 0; g < 16; ++g) {
            const float a = dq > 0.0f ? roundf(__fdiv_rn(gs[g], dq)) : 0.0f;
            ls[g] = (int8_t)clampf(a, -128.f, 127.f);
            o[192 + g] = (uint8_t)ls[g];
        }
        for (int e = 0; e < 256; ++e) {
            const float den = __fmul_rn(dq, (float)ls[e / 16]);
            int q = 0;
            if (den != 0.0f) q = (int)clampf(roundf(__fdiv_rn(xb[e], den)), -32.f, 31.f);
            const int u = q + 32, h = e / 128, r = e % 128, qi = r / 32, l = r % 32;
            const int qlidx = 64 * h + l + ((qi & 1) ? 32 : 0);
            o[qlidx] |= (uint8_t)(qi < 2 ? (u & 15) : ((u & 15) << 4));
            o[128 + 32 * h + l] |= (uint8_t)((u >> 4) << (2 * qi));
        }
        o[208] = (uint8_t)(hd & 0xff);
        o[209] = (uint8_t)(hd >> 8);
    }
}

// Project Q8_0 quantizer (ggml's rule): d = amax/127, q = round(x/d).
__global__ void quantize_q80_kernel(const float* __restrict__ x, size_t nblk, uint8_t* __restrict__ out) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblk; b += (size_t)gridDim.x * blockDim.x) {
        const float* xb = x + b * 32;
        uint8_t* o = out + b * 34;
        float am = 0.0f;
        for (int j = 0; j < 32; ++j) am = fmaxf(am, fabsf(xb[j]));
        const float d = __fdiv_rn(am, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const uint16_t hd = f32_to_f16_ref(d);
        o[0] = (uint8_t)(hd & 0xff);
        o[1] = (uint8_t)(hd >> 8);
        for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(int8_t)clampf(roundf(__fmul_rn(xb[j], id)), -127.f, 127.f);
    }
}

}  // namespace hc

extern "C" int hc_synth_normal_dev(hc_engine* e, uint64_t seed, size_t n, float mean, float stdv, float* out) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!out) return hc_set_error(HC_ERR_INVALID, "null output");
    if (n == 0) return HC_OK;
    const size_t pairs = (n + 1) / 2;
    unsigned blocks = (unsigned)((pairs + 255) / 256 < 148u * 16 ? (pairs + 255) / 256 : 148u * 16);
    synth_normal_kernel<<<blocks, 256, 0, e->stream>>>(seed, n, mean, stdv, out);
    cudaError_t ce = cudaGetLastError();
    return ce == cudaSuccess ? HC_OK : hc_cuda_error(ce, "synth_normal launch");
}

extern "C" int hc_quantize_dev(hc_engine* e, int type, const float* x, size_t n, uint8_t* out) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!x || !out) return hc_set_error(HC_ERR_INVALID, "null argument");
    const size_t qk = type == T_Q8_0 ? 32 : 256;
    if (type != T_Q4_K && type != T_Q6_K && type != T_Q8_0)
        return hc_set_error(HC_ERR_UNSUPPORTED, "no quantizer for %s", hc_type_label(type));
    if (n % qk) return hc_set_error(HC_ERR_INVALID, "quantize: n=%zu not a multiple of %zu", n, qk);
    const size_t nblk = n / qk;
    if (nblk == 0) return HC_OK;
    unsigned blocks = (unsigned)((nblk + 127) / 128 < 148u * 32 ? (nblk + 127) / 128 : 148u * 32);
    if (type == T_Q4_K) quantize_q4k_kernel<<<blocks, 128, 0, e->stream>>>(x, nblk, out);
    else if (type == T_Q6_K) quantize_q6k_kernel<<<blocks, 128, 0, e->stream>>>(x, nblk, out);
    else quantize_q80_kernel<<<blocks, 128, 0, e->stream>>>(x, nblk, out);
    cudaError_t ce = cudaGetLastError();
    return ce == cudaSuccess ? HC_OK : hc_cuda_error(ce, "quantize launch");
}
