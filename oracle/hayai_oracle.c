/*
 * hayai_oracle.c -- CPU restatement of the reference's quantized-FFN arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the CUDA
 * library in hayai_b200/.  Only tests/, __graft_entry__.smoke() and the CPU
 * baseline legs of bench.py may load it, and only as the checker (or as the
 * timed CPU baseline).  Nothing in the product path calls it.
 *
 * The reference (aitups/hayai v0.2.3) is Rust; its workspace cannot be built
 * in this environment (no cargo, un-vendored crates.io dependencies), so this
 * is a line-by-line restatement of its CPU code with Rust's f32 semantics:
 *   - every operation in f32, no FMA contraction (build with -ffp-contract=off);
 *   - left-to-right evaluation exactly as written in the Rust source;
 *   - per-row sequential sums, so results do not depend on the thread count
 *     (rows are spread over OpenMP threads like rayon's par_iter_mut);
 *   - f32::round == roundf (half away from zero), f32::exp == expf.
 * Each function cites the reference file:line it restates (paths relative to
 * the reference repository root).
 *
 * Quantizers for Q6_K and Q8_0 are NOT in the reference (it ships only
 * quantize_q4_k); the two here are simple deterministic quantizers of this
 * project, used to produce valid packed bytes.  Parity is defined on identical
 * packed bytes, so the quantizer choice does not affect the parity contract.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "iq_tables.h" /* generated at build time from the reference's codebooks */
#ifdef _OPENMP
#include <omp.h>
#endif

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int or_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

#define QK_K 256
#define Q4_K_BLOCK 144
#define Q6_K_BLOCK 210
#define Q8_0_BLOCK 34
#define IQ2_XXS_BLOCK 66
#define IQ2_XS_BLOCK 74
#define IQ2_S_BLOCK 82
#define IQ3_XXS_BLOCK 98
#define IQ3_S_BLOCK 110

#define Q4_0_BLOCK 18
#define Q4_1_BLOCK 20
#define Q5_0_BLOCK 22
#define Q5_1_BLOCK 24
#define Q2_K_BLOCK 84
#define Q3_K_BLOCK 110
#define Q5_K_BLOCK 176
#define IQ4_NL_BLOCK 18
#define IQ4_XS_BLOCK 136
#define Q8_1_BLOCK 36
#define Q8_K_BLOCK 292

/* GgmlType ids, crates/hayai-model/src/gguf_types.rs:6-40 */
enum {
    T_F32 = 0, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11,
    T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18, T_IQ4_NL = 20,
    T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23, T_F16 = 1, T_Q8_1 = 9, T_Q8_K = 15, T_BF16 = 30
};

/* ------------------------------------------------------------------------ */
/* f16 <-> f32                                                               */
/* ------------------------------------------------------------------------ */

static inline float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* crates/hayai-model/src/gguf.rs:521-545 (IEEE binary16 -> f32, exact). */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign << 31;
        } else {
            uint32_t m = mant, e = 127 - 15 + 1;
            while ((m & 0x400u) == 0) { m <<= 1; e -= 1; }
            m &= 0x3FFu;
            bits = (sign << 31) | (e << 23) | (m << 13);
        }
    } else if (exp == 31) {
        bits = (sign << 31) | (0xFFu << 23) | (mant << 13);
    } else {
        bits = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    return bits_f32(bits);
}

/* crates/hayai-model/src/q4k.rs:46-79 (the reference's own f32 -> f16 rounding). */
uint16_t or_f32_to_f16(float value) {
    uint32_t f = f32_bits(value);
    uint32_t sign = (f >> 16) & 0x8000u;
    int32_t exponent = (int32_t)((f >> 23) & 0xffu) - 127 + 15;
    uint32_t mantissa = f & 0x7fffffu;
    if (exponent <= 0) {
        if (exponent < -10) return (uint16_t)sign;
        uint32_t m = mantissa | 0x800000u;
        uint32_t shift = (uint32_t)(14 - exponent);
        m = m >> shift;
        uint32_t sb = shift > 0 ? shift - 1 : 0; /* saturating_sub(1) */
        if (mantissa & (1u << sb)) m += 1;
        return (uint16_t)(sign | m);
    }
    if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t m = mantissa >> 13;
    if (mantissa & 0x1000u) m += 1;
    if ((m & 0x400u) == 0x400u) { m = 0; exponent += 1; }
    if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)exponent << 10) | m);
}

static inline float rd_f16(const uint8_t* p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------------------------ */
/* Seeded synthetic data: splitmix64 evaluated at a position, Box-Muller.   */
/* Shared by oracle-side tests and the bench so inputs are reproducible.    */
/* ------------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Output i of the splitmix64 stream whose state starts at mix64(seed). */
uint64_t or_rng_u64(uint64_t seed, uint64_t i) {
    return mix64(mix64(seed) + (i + 1) * 0x9E3779B97F4A7C15ull);
}

static inline double u01(uint64_t seed, uint64_t i) {
    return ((double)(or_rng_u64(seed, i) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

/* out[j] = mean + std * N(0,1), pair p = (2p, 2p+1) from uniforms (2p, 2p+1). */
void or_fill_normal(uint64_t seed, size_t n, float mean, float std, float* out) {
    const double two_pi = 6.283185307179586476925286766559;
    #pragma omp parallel for schedule(static)
    for (size_t p = 0; p < (n + 1) / 2; p++) {
        double u1 = u01(seed, 2 * p), u2 = u01(seed, 2 * p + 1);
        double r = sqrt(-2.0 * log(u1));
        double th = two_pi * u2;
        out[2 * p] = (float)((double)mean + (double)std * (r * cos(th)));
        if (2 * p + 1 < n) out[2 * p + 1] = (float)((double)mean + (double)std * (r * sin(th)));
    }
}

void or_fill_bytes(uint64_t seed, size_t n, uint8_t* out) {
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) out[i] = (uint8_t)(or_rng_u64(seed, i) >> 56);
}

/* ------------------------------------------------------------------------ */
/* Q4_K                                                                      */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/q4k.rs:34-43 */
static inline void get_scale_min_k4(int j, const uint8_t* s, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *d = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* crates/hayai-model/src/q4k.rs:98-160 (quantize_q4_k_block, non-ggml simple quantizer). */
static void quantize_q4_k_block(const float* x, uint8_t* out) {
    float scales[8], mins[8];
    uint8_t l[QK_K];
    for (int j = 0; j < 8; j++) {
        float mn = INFINITY, mx = -INFINITY;
        for (int i = 0; i < 32; i++) {
            float v = x[j * 32 + i];
            mn = fminf(mn, v); /* f32::min/max ignore NaN like fminf/fmaxf */
            mx = fmaxf(mx, v);
        }
        scales[j] = (mx - mn) / 15.0f;
        mins[j] = mn;
    }
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) max_scale = fmaxf(max_scale, scales[j]);
    max_scale = fmaxf(max_scale, 1e-30f);
    for (int j = 0; j < 8; j++) max_min = fmaxf(max_min, fabsf(mins[j]));
    max_min = fmaxf(max_min, 1e-30f);
    float d = max_scale / 63.0f;
    float dmin = max_min / 63.0f;
    uint8_t ls[8], lm[8];
    for (int j = 0; j < 8; j++) {
        float a = roundf(scales[j] * 63.0f / max_scale);
        a = a < 0.0f ? 0.0f : (a > 63.0f ? 63.0f : a);
        ls[j] = (uint8_t)a;
        float b = roundf(-mins[j] * 63.0f / max_min);
        b = b < 0.0f ? 0.0f : (b > 63.0f ? 63.0f : b);
        lm[j] = (uint8_t)b;
    }
    for (int j = 0; j < 8; j++) {
        float d1 = d * (float)ls[j];
        if (d1 == 0.0f) {
            for (int ii = 0; ii < 32; ii++) l[j * 32 + ii] = 0;
            continue;
        }
        float dm = dmin * (float)lm[j];
        for (int ii = 0; ii < 32; ii++) {
            float q = roundf((x[j * 32 + ii] + dm) / d1);
            q = q < 0.0f ? 0.0f : (q > 15.0f ? 15.0f : q);
            l[j * 32 + ii] = (uint8_t)q;
        }
    }
    uint16_t hd = or_f32_to_f16(d), hm = or_f32_to_f16(dmin);
    out[0] = (uint8_t)(hd & 0xff); out[1] = (uint8_t)(hd >> 8);
    out[2] = (uint8_t)(hm & 0xff); out[3] = (uint8_t)(hm >> 8);
    uint8_t sp[12];
    memset(sp, 0, sizeof sp);
    for (int j = 0; j < 8; j++) {
        uint8_t sc = ls[j], m = lm[j];
        if (j < 4) {
            sp[j] = sc;
            sp[j + 4] = m;
        } else {
            sp[j + 4] = (uint8_t)((sc & 0xF) | ((m & 0xF) << 4));
            sp[j - 4] |= (uint8_t)((sc >> 4) << 6);
            sp[j] |= (uint8_t)((m >> 4) << 6);
        }
    }
    memcpy(out + 4, sp, 12);
    for (int j = 0; j < QK_K; j += 64) {
        int base = j / 64 * 32;
        for (int ii = 0; ii < 32; ii++) out[16 + base + ii] = (uint8_t)(l[j + ii] | (l[j + ii + 32] << 4));
    }
}

/* crates/hayai-model/src/q4k.rs:85-96 */
int or_quantize_q4_k(const float* x, size_t n, uint8_t* out) {
    if (n % QK_K) return -1;
    size_t blocks = n / QK_K;
    #pragma omp parallel for schedule(static)
    for (size_t b = 0; b < blocks; b++) quantize_q4_k_block(x + b * QK_K, out + b * Q4_K_BLOCK);
    return 0;
}

/* crates/hayai-model/src/q4k.rs:163-203 */
static void dequant_q4_k_block(const uint8_t* block, float* y) {
    float d = rd_f16(block), mn = rd_f16(block + 2);
    const uint8_t* sc = block + 4;
    const uint8_t* q = block + 16;
    int is = 0, yo = 0;
    for (int c = 0; c < QK_K / 64; c++) {
        uint8_t sc0, m0, sc1, m1;
        get_scale_min_k4(is, sc, &sc0, &m0);
        get_scale_min_k4(is + 1, sc, &sc1, &m1);
        float d1 = d * (float)sc0, m1v = mn * (float)m0;
        float d2 = d * (float)sc1, m2v = mn * (float)m1;
        for (int l = 0; l < 32; l++) y[yo + l] = d1 * (float)(q[l] & 0x0F) - m1v;
        yo += 32;
        for (int l = 0; l < 32; l++) y[yo + l] = d2 * (float)(q[l] >> 4) - m2v;
        yo += 32;
        q += 32;
        is += 2;
    }
}

int or_dequant_q4_k(const uint8_t* bytes, size_t n, float* out) {
    if (n % QK_K) return -1;
    for (size_t i = 0; i < n / QK_K; i++) dequant_q4_k_block(bytes + i * Q4_K_BLOCK, out + i * QK_K);
    return 0;
}

/* crates/hayai-model/src/q4k.rs:10-32: eight f32 lanes accumulate (f*d - m)*x over
 * 4 chunks of 8, then reduce_sum (ordered, from 0.0). */
static inline float gemv_q4k_sub32(float d, float minv, const uint8_t* q, const float* x, int high) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int chunk = 0; chunk < 4; chunk++) {
        int o = chunk * 8;
        for (int lane = 0; lane < 8; lane++) {
            uint8_t b = q[o + lane];
            float f = (float)(high ? (b >> 4) : (b & 0x0F));
            float wv = f * d - minv;
            acc[lane] += wv * x[o + lane];
        }
    }
    float s = 0.0f;
    for (int lane = 0; lane < 8; lane++) s += acc[lane];
    return s;
}

/* crates/hayai-model/src/q4k.rs:206-256 */
int or_gemv_q4_k(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % QK_K) return -1;
    size_t bpr = ncols / QK_K, rb = bpr * Q4_K_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* block = data + row * rb + b * Q4_K_BLOCK;
            float d = rd_f16(block), mn = rd_f16(block + 2);
            const uint8_t* sc = block + 4;
            const uint8_t* q = block + 16;
            int is = 0;
            size_t xb = b * QK_K, xo = 0;
            for (int c = 0; c < QK_K / 64; c++) {
                uint8_t sc0, m0, sc1, m1;
                get_scale_min_k4(is, sc, &sc0, &m0);
                get_scale_min_k4(is + 1, sc, &sc1, &m1);
                float d1 = d * (float)sc0, m1v = mn * (float)m0;
                float d2 = d * (float)sc1, m2v = mn * (float)m1;
                sum += gemv_q4k_sub32(d1, m1v, q, input + xb + xo, 0);
                xo += 32;
                sum += gemv_q4k_sub32(d2, m2v, q, input + xb + xo, 1);
                xo += 32;
                q += 32;
                is += 2;
            }
        }
        output[row] = sum;
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Q6_K                                                                      */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/q6k.rs:26-57 */
static void dequant_q6_k_block(const uint8_t* block, float* y) {
    const uint8_t* ql = block;
    const uint8_t* qh = block + 128;
    const int8_t* sc = (const int8_t*)(block + 192);
    float d = rd_f16(block + 208);
    int yo = 0, qlo = 0, qho = 0, sco = 0;
    for (int h = 0; h < QK_K / 128; h++) {
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = (int)(int8_t)((ql[qlo + l] & 0x0F) | (((qh[qho + l] >> 0) & 3) << 4)) - 32;
            int q2 = (int)(int8_t)((ql[qlo + l + 32] & 0x0F) | (((qh[qho + l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)(int8_t)((ql[qlo + l] >> 4) | (((qh[qho + l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)(int8_t)((ql[qlo + l + 32] >> 4) | (((qh[qho + l] >> 6) & 3) << 4)) - 32;
            float s0 = (float)sc[sco + is], s2 = (float)sc[sco + is + 2];
            float s4 = (float)sc[sco + is + 4], s6 = (float)sc[sco + is + 6];
            y[yo + l] = d * s0 * (float)q1;
            y[yo + l + 32] = d * s2 * (float)q2;
            y[yo + l + 64] = d * s4 * (float)q3;
            y[yo + l + 96] = d * s6 * (float)q4;
        }
        yo += 128; qlo += 64; qho += 32; sco += 8;
    }
}

int or_dequant_q6_k(const uint8_t* bytes, size_t n, float* out) {
    if (n % QK_K) return -1;
    for (size_t i = 0; i < n / QK_K; i++) dequant_q6_k_block(bytes + i * Q6_K_BLOCK, out + i * QK_K);
    return 0;
}

/* crates/hayai-model/src/q6k.rs:59-90: dequantize the row, then a sequential dot. */
int or_gemv_q6_k(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % QK_K) return -1;
    size_t bpr = ncols / QK_K, rb = bpr * Q6_K_BLOCK;
    #pragma omp parallel
    {
        float* vals = (float*)malloc(ncols * sizeof(float));
        #pragma omp for schedule(static)
        for (size_t row = 0; row < nrows; row++) {
            for (size_t b = 0; b < bpr; b++) dequant_q6_k_block(data + row * rb + b * Q6_K_BLOCK, vals + b * QK_K);
            float sum = 0.0f;
            for (size_t c = 0; c < ncols; c++) sum += vals[c] * input[c];
            output[row] = sum;
        }
        free(vals);
    }
    return 0;
}

/* Project quantizer (no reference counterpart): per 16-element group the scale is
 * amax/31 so codes stay in [-31, 31]; the block keeps d = max_scale/127 (f16, the
 * reference's rounding) and int8 group scales ls = round(scale/d). */
int or_quantize_q6_k(const float* x, size_t n, uint8_t* out) {
    if (n % QK_K) return -1;
    size_t blocks = n / QK_K;
    #pragma omp parallel for schedule(static)
    for (size_t bi = 0; bi < blocks; bi++) {
        const float* xb = x + bi * QK_K;
        uint8_t* o = out + bi * Q6_K_BLOCK;
        float gs[16], maxs = 0.0f;
        for (int g = 0; g < 16; g++) {
            float am = 0.0f;
            for (int i = 0; i < 16; i++) am = fmaxf(am, fabsf(xb[g * 16 + i]));
            gs[g] = am / 31.0f;
            maxs = fmaxf(maxs, gs[g]);
        }
        maxs = fmaxf(maxs, 1e-30f);
        float d = maxs / 127.0f;
        uint16_t hd = or_f32_to_f16(d);
        float dq = or_f16_to_f32(hd);
        memset(o, 0, Q6_K_BLOCK);
        for (int g = 0; g < 16; g++) {
            float a = dq > 0.0f ? roundf(gs[g] / dq) : 0.0f;
            a = a < -128.0f ? -128.0f : (a > 127.0f ? 127.0f : a);
            o[192 + g] = (uint8_t)(int8_t)a;
        }
        for (int e = 0; e < QK_K; e++) {
            int ls = (int)(int8_t)o[192 + e / 16];
            float den = dq * (float)ls;
            int q = 0;
            if (den != 0.0f) {
                float r = roundf(xb[e] / den);
                r = r < -32.0f ? -32.0f : (r > 31.0f ? 31.0f : r);
                q = (int)r;
            }
            int u = q + 32, h = e / 128, r = e % 128, qi = r / 32, l = r % 32;
            int lo4 = u & 15, hi2 = u >> 4;
            int qlidx = 64 * h + l + ((qi & 1) ? 32 : 0);
            if (qi < 2) o[qlidx] |= (uint8_t)lo4; else o[qlidx] |= (uint8_t)(lo4 << 4);
            o[128 + 32 * h + l] |= (uint8_t)(hi2 << (2 * qi));
        }
        o[208] = (uint8_t)(hd & 0xff);
        o[209] = (uint8_t)(hd >> 8);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Q8_0                                                                      */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/quant.rs:598-615: sum += (q as f32) * d * x, left to right. */
int or_gemv_q8_0(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 32) return -1;
    size_t bpr = ncols / 32, rb = bpr * Q8_0_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q8_0_BLOCK;
            float d = rd_f16(base);
            size_t xb = b * 32;
            for (int j = 0; j < 32; j++) sum += (float)(int8_t)base[2 + j] * d * input[xb + j];
        }
        output[row] = sum;
    }
    return 0;
}

/* crates/hayai-model/src/quant.rs:652-665 */
int or_dequant_q8_0(const uint8_t* bytes, size_t n, float* out) {
    if (n % 32) return -1;
    for (size_t b = 0; b < n / 32; b++) {
        float d = rd_f16(bytes + b * Q8_0_BLOCK);
        for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)(int8_t)bytes[b * Q8_0_BLOCK + 2 + j] * d;
    }
    return 0;
}

/* Project quantizer (ggml's Q8_0 rule): d = amax/127, q = round(x/d), d kept as f16. */
int or_quantize_q8_0(const float* x, size_t n, uint8_t* out) {
    if (n % 32) return -1;
    #pragma omp parallel for schedule(static)
    for (size_t b = 0; b < n / 32; b++) {
        const float* xb = x + b * 32;
        float am = 0.0f;
        for (int j = 0; j < 32; j++) am = fmaxf(am, fabsf(xb[j]));
        float d = am / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t hd = or_f32_to_f16(d);
        uint8_t* o = out + b * Q8_0_BLOCK;
        o[0] = (uint8_t)(hd & 0xff);
        o[1] = (uint8_t)(hd >> 8);
        for (int j = 0; j < 32; j++) {
            float q = roundf(xb[j] * id);
            q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
            o[2 + j] = (uint8_t)(int8_t)q;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* F32 (router)                                                              */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/quant.rs:358-369: sum += w * x, sequential, no FMA. */
int or_gemv_f32(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    const float* w = (const float*)data;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t c = 0; c < ncols; c++) sum += w[row * ncols + c] * input[c];
        output[row] = sum;
    }
    return 0;
}

/* crates/hayai-model/src/quant.rs:371-382: w = f16_to_f32(bits), sum += w * x, sequential. */
int or_gemv_f16(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t c = 0; c < ncols; c++) sum += rd_f16(data + (row * ncols + c) * 2) * input[c];
        output[row] = sum;
    }
    return 0;
}

static inline float rd_bf16(const uint8_t* p) {
    uint32_t bits = ((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* crates/hayai-model/src/quant.rs:384-395: w = f32::from_bits(bits << 16). */
int or_gemv_bf16(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t c = 0; c < ncols; c++) sum += rd_bf16(data + (row * ncols + c) * 2) * input[c];
        output[row] = sum;
    }
    return 0;
}

/* crates/hayai-model/src/quant.rs:458-475: {f16 d, f16 s, int8 qs[32]}; sum += (q as f32) * d * x
 * (s, the block's sum, is not read). */
int or_gemv_q8_1(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 32) return -1;
    size_t bpr = ncols / 32, rb = bpr * Q8_1_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q8_1_BLOCK;
            float d = rd_f16(base);
            for (int j = 0; j < 32; j++) sum += (float)(int8_t)base[4 + j] * d * input[b * 32 + j];
        }
        output[row] = sum;
    }
    return 0;
}

/* crates/hayai-model/src/quant.rs:477-501: {f32 d, int8 qs[256], int16 bsums[16]};
 * sum += (q as f32) * d * x (bsums are not read). */
int or_gemv_q8_k(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 256) return -1;
    size_t bpr = ncols / 256, rb = bpr * Q8_K_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q8_K_BLOCK;
            float d;
            memcpy(&d, base, 4);
            for (int j = 0; j < 256; j++) sum += (float)(int8_t)base[4 + j] * d * input[b * 256 + j];
        }
        output[row] = sum;
    }
    return 0;
}

static void dequant_q8_1_block(const uint8_t* b, float* y) {
    float d = rd_f16(b);
    for (int j = 0; j < 32; j++) y[j] = (float)(int8_t)b[4 + j] * d;
}

static void dequant_q8_k_block(const uint8_t* b, float* y) {
    float d;
    memcpy(&d, b, 4);
    for (int j = 0; j < 256; j++) y[j] = (float)(int8_t)b[4 + j] * d;
}

static void dequant_f16_elem(const uint8_t* b, float* y) { y[0] = rd_f16(b); }
static void dequant_bf16_elem(const uint8_t* b, float* y) { y[0] = rd_bf16(b); }

/* ------------------------------------------------------------------------ */
/* IQ2 / IQ3 codebook formats                                                */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/iq2.rs:18-27: sign byte for a 7-bit index = index with
 * bit 7 = parity of the index. */
static inline uint8_t ksigns(uint32_t i) {
    i &= 127u;
    return (uint8_t)(i | ((uint32_t)(__builtin_popcount(i) & 1) << 7));
}

/* crates/hayai-model/src/iq2.rs:497-503 (signed_mul): db * g * s. */
static inline float signed_mul(float db, uint8_t g, uint8_t signs, int j) {
    float s = (signs & (1u << j)) ? -1.0f : 1.0f;
    return db * (float)g * s;
}

static inline uint32_t rd_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

static inline uint8_t grid8_byte(uint64_t g, int j) { return (uint8_t)(g >> (8 * j)); }
static inline uint8_t grid4_byte(uint32_t g, int j) { return (uint8_t)(g >> (8 * j)); }

/* crates/hayai-model/src/iq2.rs:504-523 */
static void dequant_iq2_xxs_block(const uint8_t* block, float* y) {
    float d = rd_f16(block);
    const uint8_t* qs = block + 2;
    int yo = 0;
    for (int ib32 = 0; ib32 < 8; ib32++) {
        uint32_t aux0 = rd_u32(qs + 8 * ib32), aux1 = rd_u32(qs + 8 * ib32 + 4);
        float db = d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            uint64_t g = hc_iq2xxs_grid[(aux0 >> (8 * l)) & 0xff];
            uint8_t signs = ksigns((aux1 >> (7 * l)) & 127);
            for (int j = 0; j < 8; j++) y[yo + j] = signed_mul(db, grid8_byte(g, j), signs, j);
            yo += 8;
        }
    }
}

/* crates/hayai-model/src/iq2.rs:525-544 */
static void dequant_iq2_xs_block(const uint8_t* block, float* y) {
    float d = rd_f16(block);
    const uint8_t* qs = block + 2;
    const uint8_t* scales = block + 66;
    int yo = 0;
    for (int ib32 = 0; ib32 < 8; ib32++) {
        float db0 = d * (0.5f + (float)(scales[ib32] & 0x0f)) * 0.25f;
        float db1 = d * (0.5f + (float)(scales[ib32] >> 4)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            uint16_t q = (uint16_t)(qs[8 * ib32 + 2 * l] | (qs[8 * ib32 + 2 * l + 1] << 8));
            uint64_t g = hc_iq2xs_grid[q & 511];
            uint8_t signs = ksigns(q >> 9);
            float db = l < 2 ? db0 : db1;
            for (int j = 0; j < 8; j++) y[yo + j] = signed_mul(db, grid8_byte(g, j), signs, j);
            yo += 8;
        }
    }
}

/* crates/hayai-model/src/iq2.rs:546-573 */
static void dequant_iq2_s_block(const uint8_t* block, float* y) {
    float d = rd_f16(block);
    const uint8_t* qs = block + 2;
    const uint8_t* signs_all = block + 34;
    const uint8_t* qh = block + 66;
    const uint8_t* scales = block + 74;
    int yo = 0, qoff = 0, soff = 0;
    for (int ib32 = 0; ib32 < 8; ib32++) {
        float db0 = d * (0.5f + (float)(scales[ib32] & 0x0f)) * 0.25f;
        float db1 = d * (0.5f + (float)(scales[ib32] >> 4)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            float db = l < 2 ? db0 : db1;
            uint32_t idx = (uint32_t)qs[qoff + l] | (((uint32_t)qh[ib32] << (8 - 2 * l)) & 0x300u);
            uint64_t g = hc_iq2s_grid[idx];
            uint8_t signs = signs_all[soff + l];
            for (int j = 0; j < 8; j++) y[yo + j] = signed_mul(db, grid8_byte(g, j), signs, j);
            yo += 8;
        }
        qoff += 4;
        soff += 4;
    }
}

/* crates/hayai-model/src/iq3.rs:147-173 */
static void dequant_iq3_xxs_block(const uint8_t* block, float* y) {
    float d = rd_f16(block);
    const uint8_t* qs = block + 2;
    const uint8_t* sas = block + 66;
    int yo = 0, qoff = 0;
    for (int ib32 = 0; ib32 < 8; ib32++) {
        uint32_t aux32 = rd_u32(sas + 4 * ib32);
        float db = d * (0.5f + (float)(aux32 >> 28)) * 0.5f;
        for (int l = 0; l < 4; l++) {
            uint8_t signs = ksigns((aux32 >> (7 * l)) & 127);
            uint32_t g1 = hc_iq3xxs_grid[qs[qoff + 2 * l]], g2 = hc_iq3xxs_grid[qs[qoff + 2 * l + 1]];
            for (int j = 0; j < 4; j++) {
                y[yo + j] = signed_mul(db, grid4_byte(g1, j), signs, j);
                y[yo + 4 + j] = signed_mul(db, grid4_byte(g2, j), signs, j + 4);
            }
            yo += 8;
        }
        qoff += 8;
    }
}

/* crates/hayai-model/src/iq3.rs:175-220 */
static void dequant_iq3_s_block(const uint8_t* block, float* y) {
    float d = rd_f16(block);
    const uint8_t* qs_all = block + 2;
    const uint8_t* qh_all = block + 66;
    const uint8_t* signs_all = block + 74;
    const uint8_t* scales = block + 106;
    int yo = 0, qoff = 0, soff = 0, qh_off = 0;
    for (int ib32 = 0; ib32 < 8; ib32 += 2) {
        float db1 = d * (1.0f + 2.0f * (float)(scales[ib32 / 2] & 0x0f));
        float db2 = d * (1.0f + 2.0f * (float)(scales[ib32 / 2] >> 4));
        for (int half = 0; half < 2; half++) {
            uint32_t qh = qh_all[qh_off + half];
            float db = half ? db2 : db1;
            for (int l = 0; l < 4; l++) {
                uint32_t idx1 = (uint32_t)qs_all[qoff + 2 * l] | ((qh << (8 - 2 * l)) & 256u);
                uint32_t idx2 = (uint32_t)qs_all[qoff + 2 * l + 1] | ((qh << (7 - 2 * l)) & 256u);
                uint32_t g1 = hc_iq3s_grid[idx1], g2 = hc_iq3s_grid[idx2];
                uint8_t signs = signs_all[soff + l];
                for (int j = 0; j < 4; j++) {
                    y[yo + j] = signed_mul(db, grid4_byte(g1, j), signs, j);
                    y[yo + 4 + j] = signed_mul(db, grid4_byte(g2, j), signs, j + 4);
                }
                yo += 8;
            }
            qoff += 8;
            soff += 4;
        }
        qh_off += 2;
    }
}

typedef void (*block_fn)(const uint8_t*, float*);

/* crates/hayai-model/src/iq2.rs:591-626 (macro gemv) and iq3.rs:258-331: dequantize
 * each block into tmp[256], then a sequential dot continuing one running sum. */
static int gemv_blockwise(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output,
                          block_fn fn, size_t blk) {
    if (ncols % QK_K) return -1;
    size_t bpr = ncols / QK_K, rb = bpr * blk;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float tmp[QK_K];
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            fn(data + row * rb + b * blk, tmp);
            for (int j = 0; j < QK_K; j++) sum += tmp[j] * input[b * QK_K + j];
        }
        output[row] = sum;
    }
    return 0;
}

int or_gemv_iq2_xxs(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blockwise(m, n, w, x, y, dequant_iq2_xxs_block, IQ2_XXS_BLOCK); }
int or_gemv_iq2_xs(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blockwise(m, n, w, x, y, dequant_iq2_xs_block, IQ2_XS_BLOCK); }
int or_gemv_iq2_s(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blockwise(m, n, w, x, y, dequant_iq2_s_block, IQ2_S_BLOCK); }
int or_gemv_iq3_xxs(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blockwise(m, n, w, x, y, dequant_iq3_xxs_block, IQ3_XXS_BLOCK); }
int or_gemv_iq3_s(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blockwise(m, n, w, x, y, dequant_iq3_s_block, IQ3_S_BLOCK); }

/* ------------------------------------------------------------------------ */
/* Q4_0, Q4_1, Q5_0, Q5_1 (32-element blocks)                                */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/quant.rs:617-632 (extract_q4_0_row) */
static void dequant_q4_0_block(const uint8_t* b, float* y) {
    float d = rd_f16(b);
    const uint8_t* qs = b + 2;
    for (int j = 0; j < 16; j++) {
        y[j] = (float)((int)(qs[j] & 0x0F) - 8) * d;
        y[j + 16] = (float)((int)(qs[j] >> 4) - 8) * d;
    }
}

/* crates/hayai-model/src/quant.rs:538-574: per block, two 8-lane chunks accumulate
 * (ql*d)*xl + (qh*d)*xh lane by lane; the lanes' reduce_sum (taken in lane order here)
 * joins the row sum. */
int or_gemv_q4_0(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 32) return -1;
    size_t bpr = ncols / 32, rb = bpr * Q4_0_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q4_0_BLOCK;
            float d = rd_f16(base);
            const uint8_t* qs = base + 2;
            const float* x = input + b * 32;
            float ql[16], qh[16], acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j < 16; j++) {
                ql[j] = (float)((int)(qs[j] & 0x0F) - 8);
                qh[j] = (float)((int)(qs[j] >> 4) - 8);
            }
            for (int c = 0; c < 2; c++) {
                int o = c * 8;
                for (int i = 0; i < 8; i++) acc[i] += ql[o + i] * d * x[o + i] + qh[o + i] * d * x[16 + o + i];
            }
            float r = 0.0f;
            for (int i = 0; i < 8; i++) r += acc[i];
            sum += r;
        }
        output[row] = sum;
    }
    return 0;
}

/* crates/hayai-model/src/quant.rs:634-650 (extract_q4_1_row) */
static void dequant_q4_1_block(const uint8_t* b, float* y) {
    float d = rd_f16(b), m = rd_f16(b + 2);
    const uint8_t* qs = b + 4;
    for (int j = 0; j < 16; j++) {
        y[j] = (float)(qs[j] & 0x0F) * d + m;
        y[j + 16] = (float)(qs[j] >> 4) * d + m;
    }
}

/* crates/hayai-model/src/quant.rs:576-596 */
int or_gemv_q4_1(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 32) return -1;
    size_t bpr = ncols / 32, rb = bpr * Q4_1_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q4_1_BLOCK;
            float d = rd_f16(base), m = rd_f16(base + 2);
            const uint8_t* qs = base + 4;
            const float* x = input + b * 32;
            for (int j = 0; j < 16; j++) {
                sum += ((float)(qs[j] & 0x0F) * d + m) * x[j];
                sum += ((float)(qs[j] >> 4) * d + m) * x[j + 16];
            }
        }
        output[row] = sum;
    }
    return 0;
}

/* The fifth bits of Q5_0 / Q5_1 element j and j + 16 (crates/hayai-model/src/q5.rs:30-33). */
static inline int q5_hi0(uint32_t qh, int j) { return (int)(((qh >> j) << 4) & 0x10); }
static inline int q5_hi1(uint32_t qh, int j) { return (int)((qh >> (j + 12)) & 0x10); }

/* crates/hayai-model/src/q5.rs:26-38 */
static void dequant_q5_0_block(const uint8_t* b, float* y) {
    float d = rd_f16(b);
    uint32_t qh = rd_u32(b + 2);
    const uint8_t* qs = b + 6;
    for (int j = 0; j < 16; j++) {
        int x0 = ((qs[j] & 0x0F) | q5_hi0(qh, j)) - 16;
        int x1 = ((qs[j] >> 4) | q5_hi1(qh, j)) - 16;
        y[j] = (float)x0 * d;
        y[j + 16] = (float)x1 * d;
    }
}

/* crates/hayai-model/src/q5.rs:40-76 */
int or_gemv_q5_0(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 32) return -1;
    size_t bpr = ncols / 32, rb = bpr * Q5_0_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q5_0_BLOCK;
            float d = rd_f16(base);
            uint32_t qh = rd_u32(base + 2);
            const uint8_t* qs = base + 6;
            const float* x = input + b * 32;
            for (int j = 0; j < 16; j++) {
                int x0 = ((qs[j] & 0x0F) | q5_hi0(qh, j)) - 16;
                int x1 = ((qs[j] >> 4) | q5_hi1(qh, j)) - 16;
                sum += (float)x0 * d * x[j];
                sum += (float)x1 * d * x[j + 16];
            }
        }
        output[row] = sum;
    }
    return 0;
}

/* crates/hayai-model/src/q5.rs:96-122 */
static void dequant_q5_1_block(const uint8_t* b, float* y) {
    float d = rd_f16(b), m = rd_f16(b + 2);
    uint32_t qh = rd_u32(b + 4);
    const uint8_t* qs = b + 8;
    for (int j = 0; j < 16; j++) {
        int x0 = (qs[j] & 0x0F) | q5_hi0(qh, j);
        int x1 = (qs[j] >> 4) | q5_hi1(qh, j);
        y[j] = (float)x0 * d + m;
        y[j + 16] = (float)x1 * d + m;
    }
}

/* crates/hayai-model/src/q5.rs:124-158 */
int or_gemv_q5_1(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output) {
    if (ncols % 32) return -1;
    size_t bpr = ncols / 32, rb = bpr * Q5_1_BLOCK;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            const uint8_t* base = data + row * rb + b * Q5_1_BLOCK;
            float d = rd_f16(base), m = rd_f16(base + 2);
            uint32_t qh = rd_u32(base + 4);
            const uint8_t* qs = base + 8;
            const float* x = input + b * 32;
            for (int j = 0; j < 16; j++) {
                int x0 = (qs[j] & 0x0F) | q5_hi0(qh, j);
                int x1 = (qs[j] >> 4) | q5_hi1(qh, j);
                sum += ((float)x0 * d + m) * x[j];
                sum += ((float)x1 * d + m) * x[j + 16];
            }
        }
        output[row] = sum;
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Q2_K, Q3_K, Q5_K (256-element super-blocks)                               */
/* ------------------------------------------------------------------------ */

/* The elements of a K-quant super-block in the reference's order, each computed by
 * `elem` exactly as the reference's GEMV forms it, then summed into one running sum:
 * crates/hayai-model/src/q2k.rs:60-118, q3k.rs:93-146, q5k.rs:69-127 (their dequant
 * blocks :26-58, :52-84, :36-66 produce the same values). */
static void dequant_q2_k_block(const uint8_t* b, float* y) {
    const uint8_t* scales = b;
    const uint8_t* q = b + 16;
    float d = rd_f16(b + 80), mn = rd_f16(b + 82);
    int yo = 0, is = 0;
    for (int n = 0; n < QK_K / 128; n++) {
        for (int j = 0; j < 4; j++) {
            int shift = 2 * j;
            for (int h = 0; h < 2; h++) {
                uint8_t sc = scales[is++];
                float dl = d * (float)(sc & 0xF), ml = mn * (float)(sc >> 4);
                for (int l = 0; l < 16; l++) y[yo + l] = dl * (float)((q[l + 16 * h] >> shift) & 3) - ml;
                yo += 16;
            }
        }
        q += 32;
    }
}

/* crates/hayai-model/src/q3k.rs:10-30 (unpack_q3_k_scales) */
static void unpack_q3_k_scales(const uint8_t* s12, int8_t* out) {
    const uint32_t kmask1 = 0x03030303u, kmask2 = 0x0f0f0f0fu;
    uint32_t aux[4];
    aux[0] = rd_u32(s12);
    aux[1] = rd_u32(s12 + 4);
    aux[2] = rd_u32(s12 + 8);
    uint32_t tmp = aux[2];
    aux[2] = ((aux[0] >> 4) & kmask2) | (((tmp >> 4) & kmask1) << 4);
    aux[3] = ((aux[1] >> 4) & kmask2) | (((tmp >> 6) & kmask1) << 4);
    aux[0] = (aux[0] & kmask2) | (((tmp >> 0) & kmask1) << 4);
    aux[1] = (aux[1] & kmask2) | (((tmp >> 2) & kmask1) << 4);
    for (int i = 0; i < 4; i++)
        for (int j = 0; j < 4; j++) out[4 * i + j] = (int8_t)(uint8_t)(aux[i] >> (8 * j));
}

static void dequant_q3_k_block(const uint8_t* b, float* y) {
    const uint8_t* hmask = b;
    const uint8_t* q = b + 32;
    int8_t scales[16];
    unpack_q3_k_scales(b + 96, scales);
    float d_all = rd_f16(b + 108);
    int yo = 0, is = 0;
    uint8_t m = 1;
    for (int n = 0; n < QK_K / 128; n++) {
        for (int j = 0; j < 4; j++) {
            int shift = 2 * j;
            for (int h = 0; h < 2; h++) {
                float dl = d_all * (float)((int)scales[is++] - 32);
                for (int l = 0; l < 16; l++) {
                    int qv = (q[l + 16 * h] >> shift) & 3;
                    int hm = (hmask[l + 16 * h] & m) ? 0 : 4;
                    y[yo + l] = dl * (float)(qv - hm);
                }
                yo += 16;
            }
            m <<= 1;
        }
        q += 32;
    }
}

/* crates/hayai-model/src/q5k.rs:10-18 (scale_min) is get_scale_min_k4 above. */
static void dequant_q5_k_block(const uint8_t* b, float* y) {
    float d = rd_f16(b), mn = rd_f16(b + 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* ql = b + 48;
    int yo = 0, is = 0;
    uint8_t u1 = 1, u2 = 2;
    for (int c = 0; c < QK_K / 64; c++) {
        uint8_t sc0, m0, sc1, m1;
        get_scale_min_k4(is, scales, &sc0, &m0);
        get_scale_min_k4(is + 1, scales, &sc1, &m1);
        float d1 = d * (float)sc0, m1v = mn * (float)m0, d2 = d * (float)sc1, m2v = mn * (float)m1;
        for (int l = 0; l < 32; l++) y[yo + l] = d1 * (float)((ql[l] & 0x0F) + ((qh[l] & u1) ? 16 : 0)) - m1v;
        yo += 32;
        for (int l = 0; l < 32; l++) y[yo + l] = d2 * (float)((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2v;
        yo += 32;
        ql += 32;
        is += 2;
        u1 <<= 2;
        u2 <<= 2;
    }
}

/* ------------------------------------------------------------------------ */
/* IQ4_NL (32-element blocks), IQ4_XS (256)                                  */
/* ------------------------------------------------------------------------ */

/* crates/hayai-model/src/iq4.rs:36-42 */
static void dequant_iq4_nl_block(const uint8_t* b, float* y) {
    float d = rd_f16(b);
    const uint8_t* qs = b + 2;
    for (int j = 0; j < 16; j++) {
        y[j] = d * (float)hc_iq4nl_values[qs[j] & 0x0F];
        y[j + 16] = d * (float)hc_iq4nl_values[qs[j] >> 4];
    }
}

/* crates/hayai-model/src/iq4.rs:121-138 */
static void dequant_iq4_xs_block(const uint8_t* b, float* y) {
    float d = rd_f16(b);
    uint32_t scales_h = (uint32_t)(b[2] | (b[3] << 8));
    const uint8_t* scales_l = b + 4;
    const uint8_t* qs = b + 8;
    for (int ib = 0; ib < 8; ib++) {
        int ls = ((scales_l[ib / 2] >> (4 * (ib % 2))) & 0x0F) | (int)(((scales_h >> (2 * ib)) & 3) << 4);
        float dl = d * (float)(ls - 32);
        for (int j = 0; j < 16; j++) {
            y[32 * ib + j] = dl * (float)hc_iq4nl_values[qs[j] & 0x0F];
            y[32 * ib + 16 + j] = dl * (float)hc_iq4nl_values[qs[j] >> 4];
        }
        qs += 16;
    }
}

/* One running sum over each block's values in element order, the block decoded exactly as the
 * reference's GEMV forms each product's weight: crates/hayai-model/src/q2k.rs:60-118,
 * q3k.rs:93-146, q5k.rs:69-127, iq4.rs:44-78 (IQ4_NL, 32-element blocks; the reference sums
 * element j, then j + 16, per j), iq4.rs:140-186 (IQ4_XS). */
static int gemv_blocks_seq(size_t nrows, size_t ncols, const uint8_t* data, const float* input, float* output,
                           block_fn fn, size_t qk, size_t blk) {
    if (ncols % qk) return -1;
    size_t bpr = ncols / qk, rb = bpr * blk;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < nrows; row++) {
        float tmp[QK_K];
        float sum = 0.0f;
        for (size_t b = 0; b < bpr; b++) {
            fn(data + row * rb + b * blk, tmp);
            const float* x = input + b * qk;
            if (qk == 32) {  /* IQ4_NL: j then j + 16 */
                for (int j = 0; j < 16; j++) {
                    sum += tmp[j] * x[j];
                    sum += tmp[j + 16] * x[j + 16];
                }
            } else if (fn == dequant_iq4_xs_block) {  /* IQ4_XS: per 32-group, j then j + 16 */
                for (int ib = 0; ib < 8; ib++)
                    for (int j = 0; j < 16; j++) {
                        sum += tmp[32 * ib + j] * x[32 * ib + j];
                        sum += tmp[32 * ib + 16 + j] * x[32 * ib + 16 + j];
                    }
            } else {
                for (int j = 0; j < (int)qk; j++) sum += tmp[j] * x[j];
            }
        }
        output[row] = sum;
    }
    return 0;
}

int or_gemv_q2_k(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blocks_seq(m, n, w, x, y, dequant_q2_k_block, QK_K, Q2_K_BLOCK); }
int or_gemv_q3_k(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blocks_seq(m, n, w, x, y, dequant_q3_k_block, QK_K, Q3_K_BLOCK); }
int or_gemv_q5_k(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blocks_seq(m, n, w, x, y, dequant_q5_k_block, QK_K, Q5_K_BLOCK); }
int or_gemv_iq4_nl(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blocks_seq(m, n, w, x, y, dequant_iq4_nl_block, 32, IQ4_NL_BLOCK); }
int or_gemv_iq4_xs(size_t m, size_t n, const uint8_t* w, const float* x, float* y) { return gemv_blocks_seq(m, n, w, x, y, dequant_iq4_xs_block, QK_K, IQ4_XS_BLOCK); }

/* Block dequantizers exported for layout cross-checks against an independent decoder. */
int or_dequant(int type, const uint8_t* bytes, size_t n, float* out) {
    block_fn fn = NULL;
    size_t blk = 0;
    size_t qk = QK_K;
    switch (type) {
        case T_Q4_K: return or_dequant_q4_k(bytes, n, out);
        case T_Q6_K: return or_dequant_q6_k(bytes, n, out);
        case T_Q8_0: return or_dequant_q8_0(bytes, n, out);
        case T_IQ2_XXS: fn = dequant_iq2_xxs_block; blk = IQ2_XXS_BLOCK; break;
        case T_IQ2_XS: fn = dequant_iq2_xs_block; blk = IQ2_XS_BLOCK; break;
        case T_IQ2_S: fn = dequant_iq2_s_block; blk = IQ2_S_BLOCK; break;
        case T_IQ3_XXS: fn = dequant_iq3_xxs_block; blk = IQ3_XXS_BLOCK; break;
        case T_IQ3_S: fn = dequant_iq3_s_block; blk = IQ3_S_BLOCK; break;
        case T_Q4_0: fn = dequant_q4_0_block; blk = Q4_0_BLOCK; qk = 32; break;
        case T_Q4_1: fn = dequant_q4_1_block; blk = Q4_1_BLOCK; qk = 32; break;
        case T_Q5_0: fn = dequant_q5_0_block; blk = Q5_0_BLOCK; qk = 32; break;
        case T_Q5_1: fn = dequant_q5_1_block; blk = Q5_1_BLOCK; qk = 32; break;
        case T_IQ4_NL: fn = dequant_iq4_nl_block; blk = IQ4_NL_BLOCK; qk = 32; break;
        case T_Q2_K: fn = dequant_q2_k_block; blk = Q2_K_BLOCK; break;
        case T_Q3_K: fn = dequant_q3_k_block; blk = Q3_K_BLOCK; break;
        case T_Q5_K: fn = dequant_q5_k_block; blk = Q5_K_BLOCK; break;
        case T_IQ4_XS: fn = dequant_iq4_xs_block; blk = IQ4_XS_BLOCK; break;
        case T_Q8_1: fn = dequant_q8_1_block; blk = Q8_1_BLOCK; qk = 32; break;
        case T_Q8_K: fn = dequant_q8_k_block; blk = Q8_K_BLOCK; break;
        case T_F16: fn = dequant_f16_elem; blk = 2; qk = 1; break;
        case T_BF16: fn = dequant_bf16_elem; blk = 2; qk = 1; break;
        default: return -2;
    }
    if (n % qk) return -1;
    for (size_t i = 0; i < n / qk; i++) fn(bytes + i * blk, out + i * qk);
    return 0;
}

/* crates/hayai-model/src/quant.rs:278-354 (QuantMatrix::gemv dispatch on GgmlType). */
int or_gemv(int type, size_t nrows, size_t ncols, const uint8_t* w, const float* x, float* y) {
    switch (type) {
        case T_F32: return or_gemv_f32(nrows, ncols, w, x, y);
        case T_Q8_0: return or_gemv_q8_0(nrows, ncols, w, x, y);
        case T_Q4_K: return or_gemv_q4_k(nrows, ncols, w, x, y);
        case T_Q6_K: return or_gemv_q6_k(nrows, ncols, w, x, y);
        case T_IQ2_XXS: return or_gemv_iq2_xxs(nrows, ncols, w, x, y);
        case T_IQ2_XS: return or_gemv_iq2_xs(nrows, ncols, w, x, y);
        case T_IQ2_S: return or_gemv_iq2_s(nrows, ncols, w, x, y);
        case T_IQ3_XXS: return or_gemv_iq3_xxs(nrows, ncols, w, x, y);
        case T_IQ3_S: return or_gemv_iq3_s(nrows, ncols, w, x, y);
        case T_Q4_0: return or_gemv_q4_0(nrows, ncols, w, x, y);
        case T_Q4_1: return or_gemv_q4_1(nrows, ncols, w, x, y);
        case T_Q5_0: return or_gemv_q5_0(nrows, ncols, w, x, y);
        case T_Q5_1: return or_gemv_q5_1(nrows, ncols, w, x, y);
        case T_Q2_K: return or_gemv_q2_k(nrows, ncols, w, x, y);
        case T_Q3_K: return or_gemv_q3_k(nrows, ncols, w, x, y);
        case T_Q5_K: return or_gemv_q5_k(nrows, ncols, w, x, y);
        case T_IQ4_NL: return or_gemv_iq4_nl(nrows, ncols, w, x, y);
        case T_IQ4_XS: return or_gemv_iq4_xs(nrows, ncols, w, x, y);
        case T_F16: return or_gemv_f16(nrows, ncols, w, x, y);
        case T_BF16: return or_gemv_bf16(nrows, ncols, w, x, y);
        case T_Q8_1: return or_gemv_q8_1(nrows, ncols, w, x, y);
        case T_Q8_K: return or_gemv_q8_k(nrows, ncols, w, x, y);
        default: return -2;
    }
}

/* ------------------------------------------------------------------------ */
/* Toy LUT-Q4 matmul                                                         */
/* ------------------------------------------------------------------------ */

/* crates/hayai-cpu/src/matmul.rs:48-82 */
void or_lut_matmul_q4(size_t m, size_t n, const uint8_t* w, const float* lut, const float* input, float* output) {
    size_t pc = n / 2;
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < m; row++) {
        float sum = 0.0f;
        for (size_t c = 0; c < pc; c++) {
            uint8_t p = w[row * pc + c];
            float w0 = lut[p & 0x0F], w1 = lut[(p >> 4) & 0x0F];
            float x0 = input[c * 2], x1 = input[c * 2 + 1];
            sum += x0 * w0 + x1 * w1;
        }
        output[row] = sum;
    }
}

/* crates/hayai-cpu/src/matmul.rs:5-18 */
void or_fp32_matmul(size_t m, size_t n, const float* w, const float* input, float* output) {
    #pragma omp parallel for schedule(static)
    for (size_t row = 0; row < m; row++) {
        float sum = 0.0f;
        for (size_t c = 0; c < n; c++) sum += w[row * n + c] * input[c];
        output[row] = sum;
    }
}

/* ------------------------------------------------------------------------ */
/* RMSNorm                                                                   */
/* ------------------------------------------------------------------------ */

/* crates/hayai-cpu/src/simd_ops.rs:10-25 (simd_mean_square): eight f32 lanes accumulate
 * v*v over chunks of 8, ordered reduce_sum, then the scalar tail, then / len. */
float or_mean_square(const float* x, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[l] += x[i + l] * x[i + l];
    float ms = 0.0f;
    for (int l = 0; l < 8; l++) ms += acc[l];
    for (; i < n; i++) ms += x[i] * x[i];
    return ms / (float)n;
}

/* crates/hayai-cpu/src/attention.rs:142-147 (rms_norm) with simd_scale_mul
 * (simd_ops.rs:28-42): x[i] = (x[i] * inv) * w[i], inv = 1 / sqrt(ms + eps).  Out of place. */
void or_rms_norm(const float* x, const float* w, size_t n, float eps, float* out) {
    float ms = or_mean_square(x, n);
    float inv = 1.0f / sqrtf(ms + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* ------------------------------------------------------------------------ */
/* SwiGLU FFN block                                                          */
/* ------------------------------------------------------------------------ */

/* crates/hayai-core/src/stream_infer.rs:3836-3840 (and moe_infer.rs:364-366):
 * g = (g / (1 + exp(-g))) * u. */
void or_swiglu(const float* g, const float* u, float* h, size_t n) {
    for (size_t j = 0; j < n; j++) h[j] = (g[j] / (1.0f + expf(-g[j]))) * u[j];
}

/* crates/hayai-core/src/stream_infer.rs:574-606 (run_ffn_block): gate and up GEMVs
 * over x (k_in columns), SiLU(g)*u, then the down GEMV (n_out rows over d_ff
 * columns).  y receives the FFN output; the residual add is the caller's. */
int or_ffn_swiglu(int tg, const uint8_t* wg, int tu, const uint8_t* wu, int td, const uint8_t* wd,
                  size_t k_in, size_t d_ff, size_t n_out, const float* x, float* y) {
    float* g = (float*)malloc(d_ff * sizeof(float));
    float* u = (float*)malloc(d_ff * sizeof(float));
    int rc = or_gemv(tg, d_ff, k_in, wg, x, g);
    if (!rc) rc = or_gemv(tu, d_ff, k_in, wu, x, u);
    if (!rc) {
        or_swiglu(g, u, g, d_ff);
        rc = or_gemv(td, n_out, d_ff, wd, g, y);
    }
    free(g);
    free(u);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* MoE routing + expert FFN                                                  */
/* ------------------------------------------------------------------------ */

/* Stable sort of idx[0..n) by key descending (ties keep their order), i.e. Rust's
 * stable sort_by with b.partial_cmp(a) on non-NaN keys.  Insertion sort: n <= 256. */
static void stable_sort_desc(int32_t* idx, size_t n, const float* key) {
    for (size_t i = 1; i < n; i++) {
        int32_t v = idx[i];
        size_t j = i;
        while (j > 0 && key[idx[j - 1]] < key[v]) { idx[j] = idx[j - 1]; j--; }
        idx[j] = v;
    }
}

/* crates/hayai-core/src/moe_infer.rs:868-935 (route_experts) with top_k_indices
 * :852-862; meta fields as MoeMeta, crates/hayai-core/src/exec_plan.rs:244-272.
 * ids/weights receive k entries; returns k (or <0 on error). */
int or_route_experts(const float* scores, const float* bias, size_t n, size_t top_k, size_t n_group,
                     size_t topk_group, int gating, int norm_topk_prob, float routed_scaling_factor,
                     int32_t* ids, float* weights) {
    if (n == 0) return 0;
    float* choice = (float*)malloc(n * sizeof(float));
    int32_t* idx = (int32_t*)malloc(n * sizeof(int32_t));
    for (size_t i = 0; i < n; i++) choice[i] = bias ? scores[i] + bias[i] : scores[i];
    size_t k;
    int grouped = n_group > 0 && topk_group > 0 && n % n_group == 0;
    if (grouped) {
        size_t gs = n / n_group;
        float* gsc = (float*)malloc(n_group * sizeof(float));
        int32_t* gidx = (int32_t*)malloc(n_group * sizeof(int32_t));
        float* vals = (float*)malloc(gs * sizeof(float));
        int32_t* vi = (int32_t*)malloc(gs * sizeof(int32_t));
        for (size_t g = 0; g < n_group; g++) {
            for (size_t j = 0; j < gs; j++) { vals[j] = choice[g * gs + j]; vi[j] = (int32_t)j; }
            stable_sort_desc(vi, gs, vals);
            float s = 0.0f;
            for (size_t j = 0; j < gs && j < 2; j++) s += vals[vi[j]];
            gsc[g] = s;
            gidx[g] = (int32_t)g;
        }
        stable_sort_desc(gidx, n_group, gsc);
        size_t nc = 0;
        for (size_t t = 0; t < topk_group && t < n_group; t++)
            for (size_t j = 0; j < gs; j++) idx[nc++] = (int32_t)(gidx[t] * gs + j);
        k = top_k > 0 ? top_k : 1;
        size_t cap = nc > 0 ? nc : 1;
        if (k > cap) k = cap;
        stable_sort_desc(idx, nc, choice);
        if (k > nc) k = nc;
        free(gsc); free(gidx); free(vals); free(vi);
    } else {
        for (size_t i = 0; i < n; i++) idx[i] = (int32_t)i;
        stable_sort_desc(idx, n, choice);
        k = top_k < n ? top_k : n;
        if (k < 1) k = 1;
    }
    for (size_t i = 0; i < k; i++) ids[i] = idx[i];
    if (gating == 1) {
        for (size_t i = 0; i < k; i++) weights[i] = 1.0f / (1.0f + expf(-scores[ids[i]]));
    } else {
        float mx = -INFINITY;
        for (size_t i = 0; i < n; i++) mx = fmaxf(mx, scores[i]);
        float sum = 0.0f;
        float* ex = (float*)malloc(n * sizeof(float));
        for (size_t i = 0; i < n; i++) { ex[i] = expf(scores[i] - mx); sum += ex[i]; }
        float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (size_t i = 0; i < k; i++) weights[i] = ex[ids[i]] * inv;
        free(ex);
    }
    if (norm_topk_prob) {
        float s = 0.0f;
        for (size_t i = 0; i < k; i++) s += weights[i];
        if (s > 0.0f)
            for (size_t i = 0; i < k; i++) weights[i] /= s;
    }
    if (fabsf(routed_scaling_factor - 1.0f) > 1e-9f)
        for (size_t i = 0; i < k; i++) weights[i] *= routed_scaling_factor;
    free(choice);
    free(idx);
    return (int)k;
}

/* crates/hayai-core/src/moe_infer.rs:221-264 (router GEMV + routing) and :342-376,
 * :449-455 (per-expert SwiGLU, acc += w_i * d_i in top-k order), for n_tok tokens.
 * Expert e's gate/up/down live at wg + e*stride_g etc.  y[t] receives acc (no
 * residual); ids_out/w_out receive the routing per token (top_k each). */
int or_moe_ffn(const float* router_w, const float* router_bias, size_t n_expert, size_t top_k, int norm_topk_prob,
               float scaling, int tg, const uint8_t* wg, size_t stride_g, int tu, const uint8_t* wu, size_t stride_u,
               int td, const uint8_t* wd, size_t stride_d, size_t d_model, size_t d_ff, size_t n_tok,
               const float* x, float* y, int32_t* ids_out, float* w_out) {
    float* scores = (float*)malloc(n_expert * sizeof(float));
    float* d = (float*)malloc(d_model * sizeof(float));
    int rc = 0;
    for (size_t t = 0; t < n_tok && !rc; t++) {
        const float* xt = x + t * d_model;
        float* yt = y + t * d_model;
        or_gemv_f32(n_expert, d_model, (const uint8_t*)router_w, xt, scores);
        int32_t* ids = ids_out + t * top_k;
        float* ws = w_out + t * top_k;
        int k = or_route_experts(scores, router_bias, n_expert, top_k, 0, 0, 0, norm_topk_prob, scaling, ids, ws);
        if (k != (int)top_k) { rc = -3; break; }
        for (size_t j = 0; j < d_model; j++) yt[j] = 0.0f;
        for (int i = 0; i < k && !rc; i++) {
            size_t e = (size_t)ids[i];
            rc = or_ffn_swiglu(tg, wg + e * stride_g, tu, wu + e * stride_u, td, wd + e * stride_d, d_model, d_ff,
                               d_model, xt, d);
            for (size_t j = 0; j < d_model; j++) yt[j] += ws[i] * d[j];
        }
    }
    free(scores);
    free(d);
    return rc;
}
