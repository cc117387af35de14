// repack.cu -- one-time upload transform from raw GGUF rows to the GPU layouts.
//
// Q4_K, Q6_K, Q8_0 and the IQ2 / IQ3 formats are stored tile-major: the matrix is cut into 16-row tiles, and the
// 16 rows x one kernel block (256 elements; 128 for Q8_0) of a tile form one contiguous
// "tile-block" image.  The blocks of a tile follow one another, so any run of blocks of a
// tile is a single contiguous range: the GEMV moves a whole pipeline stage with one TMA
// bulk copy per matrix.  Inside an image, every 16-byte piece a lane reads sits at
// (4 * row + lane_in_group) * 16 within its region, so the 32 lanes of a warp read 32
// consecutive pieces (conflict-free shared-memory reads) and 128-bit loads are always
// aligned.  Rows past M are zero.
//
//  Q4_K image (2304 B):  [hdr: row r at 16r: d, dmin (f16), then the 6-bit scales and mins
//                         regrouped per lane: bytes 4 + 3t..+2 hold sc(2t) | sc(2t+1) << 6 |
//                         m(2t) << 12 | m(2t+1) << 18 (get_scale_min_k4, q4k.rs:34-43)]
//                        [q0: (r,t) at 256 + 16(4r+t) = qs bytes 32t..32t+15]
//                        [q1: (r,t) at 1280 + 16(4r+t) = qs bytes 32t+16..32t+31]
//  Q6_K image (3360 B), lane-distributed: lane t of a row owns half h = t >> 1, l in
//                        [16s, 16s + 16), s = t & 1 (the 4 scale groups 8h + 2q + s, q < 4):
//                        [l0: (r,t) at 16(4r+t) = ql bytes 64h + 16s .. +15]
//                        [l1: at 1024 + 16(4r+t) = ql bytes 64h + 32 + 16s .. +15]
//                        [qh: at 2048 + 16(4r+t) = qh bytes 32h + 16s .. +15]
//                        [sc: row r at 3072 + 16r, word t = scales 8h + s + 2q in byte q]
//                        [d: row r at 3328 + 2r]
//  Q8_0 image (2176 B), one group = 4 GGUF blocks = 128 elements:
//                        [q0: (r,t) at 16(4r+t)][q1: at 1024 + 16(4r+t)][d: row r at 2048 + 8r]
//                        word wi of lane t (q0: wi < 4, q1: wi - 4) = codes 16(wi & 1) + 4t..+3 of
//                        block 4G + wi / 2; d = the group's 4 f16 scales; missing blocks are zero.
//  IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S images (1056 / 1184 / 1312 / 1568 / 1760 B):
//                        [d: row r at 2r][piece (r,t) at 32 + 16(4r+t) = lane t's groups 2t,
//                        2t+1: block bytes 2 + 16t..+15 (IQ2_S: grid-index bytes 2 + 8t..+7,
//                        then sign bytes 34 + 8t..+7)][extras from 1056: IQ2_XS scales (8 B
//                        per row); IQ2_S qh, scales (16 B per row); IQ3_XXS scale-and-sign
//                        words (32 B per row); IQ3_S signs (32 B per row), qh (8 B per row at
//                        1568), scales (4 B per row at 1696)] (iq2.rs:504-573, iq3.rs:147-220).
//  F32, F16, BF16 and the other block formats: raw GGUF rows.
//
// Layout of the GGUF blocks: q4k.rs:11-43 (Q4_K), q6k.rs:26-57 (ql/qh/scales/d),
// quant.rs:598-615 (Q8_0).
#include "common.cuh"
#include "gemv_launch.h"

namespace hc {

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
        case T_Q4_0: return (size_t)K / 32 * 18;
        case T_Q4_1: return (size_t)K / 32 * 20;
        case T_Q5_0: return (size_t)K / 32 * 22;
        case T_Q5_1: return (size_t)K / 32 * 24;
        case T_IQ4_NL: return (size_t)K / 32 * 18;
        case T_Q2_K: return (size_t)K / 256 * 84;
        case T_Q3_K: return (size_t)K / 256 * 110;
        case T_Q5_K: return (size_t)K / 256 * 176;
        case T_IQ4_XS: return (size_t)K / 256 * 136;
        case T_F16: case T_BF16: return (size_t)K * 2;
        case T_Q8_1: return (size_t)K / 32 * 36;
        case T_Q8_K: return (size_t)K / 256 * 292;
        default: return 0;
    }
}

bool tiled_type(int type) { return type == T_Q4_K || type == T_Q6_K || type == T_Q8_0 || is_iq_type(type); }

size_t tile_block_bytes(int type) {
    switch (type) {
        case T_Q4_K: return 2304;
        case T_Q6_K: return 3360;
        case T_Q8_0: return 2176;
        case T_IQ2_XXS: return 1056;
        case T_IQ2_XS: return 1184;
        case T_IQ2_S: return 1312;
        case T_IQ3_XXS: return 1568;
        case T_IQ3_S: return 1760;
        default: return 0;
    }
}

// kernel blocks per row: 256-element super-blocks, or 128-element groups for Q8_0
static size_t kernel_blocks(int type, int K) {
    return type == T_Q8_0 ? ((size_t)K / 32 + 3) / 4 : (size_t)K / 256;
}

size_t gpu_stride(int type, int K) {
    if (tiled_type(type)) return kernel_blocks(type, K) * tile_block_bytes(type);
    return raw_row_bytes(type, K);
}

size_t gpu_weight_bytes(int type, int M, int K) {
    if (tiled_type(type)) return (size_t)((M + 15) / 16) * gpu_stride(type, K);
    return (size_t)M * raw_row_bytes(type, K);
}

__device__ __forceinline__ uint32_t rd4(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__device__ __forceinline__ uint32_t rd2(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// One thread per 32-bit word of the tiled image.  Word w of tile-block (tile, kb); the
// source row is tile * 16 + r (zero when >= M).
template <int kType>
__device__ __forceinline__ uint32_t tiled_word(const uint8_t* __restrict__ raw, size_t raw_rb, int M, int nb, int tile,
                                               int kb, int w) {
    if constexpr (kType == T_Q4_K) {
        int r, off;
        if (w < 64) {
            r = w >> 2;
            const int row = tile * 16 + r;
            if (row >= M) return 0u;
            const uint8_t* blk = raw + (size_t)row * raw_rb + (size_t)kb * 144;
            if ((w & 3) == 0) return rd4(blk);  // d, dmin
            // the 12 packed scale bytes, regrouped: lane t's 24 bits at byte 3t
            const uint8_t* q = blk + 4;
            uint8_t f[12];
            for (int t = 0; t < 4; ++t) {
                uint32_t v = 0;
                for (int h = 0; h < 2; ++h) {
                    const int j = 2 * t + h;
                    const uint32_t sc = j < 4 ? (q[j] & 63u) : ((q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4));
                    const uint32_t mn = j < 4 ? (q[j + 4] & 63u) : ((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
                    v |= sc << (6 * h);
                    v |= mn << (12 + 6 * h);
                }
                f[3 * t] = (uint8_t)v;
                f[3 * t + 1] = (uint8_t)(v >> 8);
                f[3 * t + 2] = (uint8_t)(v >> 16);
            }
            return rd4(f + 4 * ((w & 3) - 1));
        } else {
            const int q = w >= 320, p = (w - (q ? 320 : 64)) >> 2, j = w & 3, t = p & 3;
            r = p >> 2;
            off = 16 + 32 * t + 16 * q + 4 * j;
        }
        const int row = tile * 16 + r;
        return row < M ? rd4(raw + (size_t)row * raw_rb + (size_t)kb * 144 + off) : 0u;
    } else if constexpr (kType == T_Q6_K) {
        if (w >= 832) {  // d of rows 2k, 2k+1
            const int k = w - 832;
            uint32_t v = 0;
            for (int h = 0; h < 2; ++h) {
                const int row = tile * 16 + 2 * k + h;
                if (row < M) v |= rd2(raw + (size_t)row * raw_rb + (size_t)kb * 210 + 208) << (16 * h);
            }
            return v;
        }
        const int seg = w >> 8, p = (w & 255) >> 2, j = w & 3;
        const int r = seg < 3 ? p >> 2 : (w - 768) >> 2;
        const int t = seg < 3 ? p & 3 : w & 3, h = t >> 1, s = t & 1;
        const int row = tile * 16 + r;
        if (row >= M) return 0u;
        const uint8_t* blk = raw + (size_t)row * raw_rb + (size_t)kb * 210;
        if (seg == 0) return rd4(blk + 64 * h + 16 * s + 4 * j);
        if (seg == 1) return rd4(blk + 64 * h + 32 + 16 * s + 4 * j);
        if (seg == 2) return rd4(blk + 128 + 32 * h + 16 * s + 4 * j);
        uint32_t v = 0;  // the lane's 4 int8 scales, group q in byte q
        for (int q = 0; q < 4; ++q) v |= (uint32_t)blk[192 + 8 * h + s + 2 * q] << (8 * q);
        return v;
    } else if constexpr (is_iq_type(kType)) {
        // [d of 16 rows][piece (r, t): 16 B][extras], gemv_iq.cuh
        constexpr int kBlk = kType == T_IQ2_XXS ? 66 : kType == T_IQ2_XS ? 74 : kType == T_IQ2_S ? 82
                             : kType == T_IQ3_XXS ? 98 : 110;
        int r, off;
        if (w < 8) {  // d of rows 2w, 2w + 1
            uint32_t v = 0;
            for (int h = 0; h < 2; ++h) {
                const int row = tile * 16 + 2 * w + h;
                if (row < M) v |= rd2(raw + (size_t)row * raw_rb + (size_t)kb * kBlk) << (16 * h);
            }
            return v;
        } else if (w < 264) {  // piece (r, t), word j
            const int p = (w - 8) >> 2, j = w & 3, t = p & 3;
            r = p >> 2;
            if constexpr (kType == T_IQ2_S) off = j < 2 ? 2 + 8 * t + 4 * j : 34 + 8 * t + 4 * (j - 2);
            else off = 2 + 16 * t + 4 * j;
        } else {
            const int e = w - 264;
            if constexpr (kType == T_IQ2_XS) {  // scales: 8 B per row
                r = e >> 1;
                off = 66 + 4 * (e & 1);
            } else if constexpr (kType == T_IQ2_S) {  // qh[8] then scales[8]: 16 B per row
                r = e >> 2;
                off = (e & 3) < 2 ? 66 + 4 * (e & 3) : 74 + 4 * ((e & 3) - 2);
            } else if constexpr (kType == T_IQ3_XXS) {  // scale-and-sign words: 32 B per row
                r = e >> 3;
                off = 66 + 4 * (e & 7);
            } else {  // IQ3_S: signs (32 B per row), qh (8 B), scales (4 B)
                if (e < 128) {
                    r = e >> 3;
                    off = 74 + 4 * (e & 7);
                } else if (e < 160) {
                    r = (e - 128) >> 1;
                    off = 66 + 4 * ((e - 128) & 1);
                } else {
                    r = e - 160;
                    off = 106;
                }
            }
        }
        const int row = tile * 16 + r;
        return row < M ? rd4(raw + (size_t)row * raw_rb + (size_t)kb * kBlk + off) : 0u;
    } else {  // Q8_0, kb = group of 4 blocks
        if (w >= 512) {  // d: row r = k / 2, blocks 4G + 2(k & 1) + {0, 1}
            const int k = w - 512, row = tile * 16 + (k >> 1);
            uint32_t v = 0;
            for (int h = 0; h < 2; ++h) {
                const int blk = 4 * kb + 2 * (k & 1) + h;
                if (row < M && blk < nb) v |= rd2(raw + (size_t)row * raw_rb + (size_t)blk * 34) << (16 * h);
            }
            return v;
        }
        const int q = w >= 256, p = (w & 255) >> 2, j = w & 3, t = p & 3, r = p >> 2;
        const int wi = 4 * q + j, blk = 4 * kb + (wi >> 1), half = wi & 1;
        const int row = tile * 16 + r;
        return (row < M && blk < nb) ? rd4(raw + (size_t)row * raw_rb + (size_t)blk * 34 + 2 + 16 * half + 4 * t)
                                     : 0u;
    }
}

template <int kType>
__global__ void repack_tiled_kernel(const uint8_t* __restrict__ raw, uint32_t* __restrict__ gpu, int M, int nb,
                                    int nkb, size_t raw_rb, int words) {
    const int ntiles = (M + 15) / 16;
    const size_t total = (size_t)ntiles * nkb * words;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int w = (int)(i % words);
        const size_t tb = i / words;
        const int kb = (int)(tb % nkb), tile = (int)(tb / nkb);
        gpu[i] = tiled_word<kType>(raw, raw_rb, M, nb, tile, kb, w);
    }
}

cudaError_t launch_repack(int type, const uint8_t* raw, uint8_t* gpu, int M, int K, cudaStream_t stream) {
    const size_t rrb = raw_row_bytes(type, K);
    if (!tiled_type(type)) return cudaMemcpyAsync(gpu, raw, (size_t)M * rrb, cudaMemcpyDeviceToDevice, stream);
    const int nb = type == T_Q8_0 ? K / 32 : K / 256;
    const int nkb = (int)kernel_blocks(type, K);
    const int words = (int)(tile_block_bytes(type) / 4);
    const size_t total = (size_t)((M + 15) / 16) * nkb * words;
    const unsigned blocks = (unsigned)((total + 255) / 256 < 65535 * 8 ? (total + 255) / 256 : 65535 * 8);
    uint32_t* out = reinterpret_cast<uint32_t*>(gpu);
    switch (type) {
        case T_Q4_K: repack_tiled_kernel<T_Q4_K><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        case T_Q6_K: repack_tiled_kernel<T_Q6_K><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        case T_IQ2_XXS: repack_tiled_kernel<T_IQ2_XXS><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        case T_IQ2_XS: repack_tiled_kernel<T_IQ2_XS><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        case T_IQ2_S: repack_tiled_kernel<T_IQ2_S><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        case T_IQ3_XXS: repack_tiled_kernel<T_IQ3_XXS><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        case T_IQ3_S: repack_tiled_kernel<T_IQ3_S><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
        default: repack_tiled_kernel<T_Q8_0><<<blocks, 256, 0, stream>>>(raw, out, M, nb, nkb, rrb, words); break;
    }
    return cudaGetLastError();
}

}  // namespace hc
