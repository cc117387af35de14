// tp_reduce.cu -- the exchange step of a tensor-parallel FFN layer at batch > 1.
//
// Rank p holds gate/up rows and down columns [p F/P, (p+1) F/P), so its down GEMV yields a
// partial y_p of every output row; the layer output is x + sum_p y_p on every rank (the
// reference's residual add, crates/hayai-core/src/stream_infer.rs:2166, after an all-reduce
// of the down output).  One kernel does the all-reduce over NVLink peer memory: each CTA stores
// its slice of y_p into slot p of every rank's exchange region (plain stores, remote for the
// peers), signals every rank with a system-scope release, waits (bounded) until all ranks'
// CTAs have signalled, and adds the slots of its slice in rank order to x.  Every rank sums
// the same values in the same order, so x stays bit-identical across ranks.
//
// Buffers alternate with the exchange count (the epoch, kept on the device so a captured
// graph replays correctly): a rank writes buffer e & 1 again only in exchange e + 2, which it
// reaches after every rank has signalled exchange e + 1, i.e. after every rank's exchange-e
// kernel, the last reader of that buffer, has completed.
#include "common.cuh"
#include "gemv_launch.h"

namespace hc {
namespace {

constexpr int kXrCtas = 64;  // fixed: the counter target counts every rank's CTAs
constexpr int kXrThreads = 256;

__global__ void __launch_bounds__(kXrThreads) tp_allreduce_kernel(const float4* __restrict__ yp, float4* x, int n4,
                                                                  char* const* regions, int rank, int world, int* err) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    char* own = regions[rank];
    if (threadIdx.x == 0) s_epoch = __ldcg(reinterpret_cast<const unsigned*>(own + kPeerTpbEpoch));
    __syncthreads();
    const unsigned epoch = s_epoch;
    const size_t buf = (size_t)(epoch & 1u) * world;  // first slot of this exchange's buffer
    const int lo = (int)((long long)n4 * blockIdx.x / gridDim.x);
    const int hi = (int)((long long)n4 * (blockIdx.x + 1) / gridDim.x);

    // 1. this rank's slice into slot `rank` of every region
    for (int i = lo + (int)threadIdx.x; i < hi; i += blockDim.x) {
        const float4 v = __ldcg(yp + i);
        for (int r = 0; r < world; ++r)
            reinterpret_cast<float4*>(regions[r] + kPeerTpbData)[(buf + rank) * n4 + i] = v;
    }
    __threadfence_system();
    __syncthreads();

    // 2. signal every rank; wait for all ranks' CTAs (one second; error bit 1)
    if ((int)threadIdx.x < world)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(regions[threadIdx.x] + kPeerTpbBar) : "memory");
    if (threadIdx.x == 0) {
        const unsigned target = (epoch + 1u) * (unsigned)(gridDim.x * world);
        const unsigned* bar = reinterpret_cast<const unsigned*>(own + kPeerTpbBar);
        unsigned long long t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        int ok = 1;
        while (true) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if ((int)(v - target) >= 0) break;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > 1000000000ull) {
                ok = 0;
                if (err) atomicOr(err, 2);
                break;
            }
        }
        s_ok = ok;
    }
    __syncthreads();

    // 3. x += y_0 + y_1 + ... + y_{P-1} over this CTA's slice
    if (s_ok) {
        const float4* src = reinterpret_cast<const float4*>(own + kPeerTpbData) + buf * n4;
        for (int i = lo + (int)threadIdx.x; i < hi; i += blockDim.x) {
            float4 s = __ldcg(src + i);
            for (int r = 1; r < world; ++r) {
                const float4 v = __ldcg(src + (size_t)r * n4 + i);
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
            float4 a = x[i];
            a.x += s.x;
            a.y += s.y;
            a.z += s.z;
            a.w += s.w;
            x[i] = a;
        }
    }

    // 4. the last CTA to finish advances the epoch (every CTA read it before arriving here)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned* done = reinterpret_cast<unsigned*>(own + kPeerTpbDone);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            atomicExch(done, 0u);
            atomicExch(reinterpret_cast<unsigned*>(own + kPeerTpbEpoch), epoch + 1u);
        }
    }
}

}  // namespace

size_t tp_exchange_bytes(int world, size_t n) { return kPeerTpbData + 2 * (size_t)world * n * 4; }

cudaError_t launch_tp_allreduce(const float* yp, float* x, size_t n, void* const* regions, int rank, int world,
                                int* err, cudaStream_t stream) {
    if (n % 4 || n / 4 > 0x7FFFFFFF || ((uintptr_t)yp | (uintptr_t)x) % 16) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    tp_allreduce_kernel<<<kXrCtas, kXrThreads, 0, stream>>>(reinterpret_cast<const float4*>(yp),
                                                             reinterpret_cast<float4*>(x), (int)(n / 4),
                                                             reinterpret_cast<char* const*>(regions), rank, world, err);
    return cudaGetLastError();
}

}  // namespace hc
