// gemv_launch.h -- host-side entry points of the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hc {

struct GemvArgs;

// Tensor-core GEMV / fused SwiGLU gate-up for Q4_K, Q6_K, Q8_0 (weights in the GPU layout).
cudaError_t launch_gemv_mma(int type, const GemvArgs& a, int nvec, bool fused, int num_sms, int smem_limit,
                            cudaStream_t stream);
bool gemv_mma_supported(int type);
// Workspace of the stream-K split for an M x K launch: partial-sum floats and tile counters.
void gemv_sk_workspace(int type, int M, int K, bool fused, int num_sms, size_t* ws_floats, size_t* counters);
// Stream-K slots per tile (most CTAs sharing one tile) of an M x K GEMV on num_sms CTAs.
int gemv_sk_slots(int type, int M, int K, int num_sms);

// A batch-1 residual SwiGLU FFN stack in one persistent kernel (ffn_stack.cu).
// Layout of the peer exchange region (identical on every rank of a group).
constexpr size_t kPeerTpBar = 0;                  // u32: cross-GPU counter of the TP stack
constexpr size_t kPeerEpBar = 128;                // u32: cross-GPU counter of the EP MoE
constexpr size_t kPeerEpEpoch = 256;              // u32: EP MoE phases this rank has signalled (local)
constexpr size_t kPeerFlowTile = 1024;            // u32 per 16-row tile of x (<= 768 tiles): the dataflow TP
                                                  // stack's per-tile exchange counters
constexpr size_t kPeerTpParts = 4096;             // TP stack: down partials [2][d_model/16][parts][16] f32
constexpr size_t kPeerTpPartsBytes = 4u << 20;    // d_model x parts (<= 8) x 2 buffers x 4 B up to 65536 x 8
constexpr size_t kPeerEpData = kPeerTpParts + kPeerTpPartsBytes;  // EP MoE exchange data [2][T*k][d_model] f32
constexpr size_t kPeerEpDataBytes = 24u << 20;    // e.g. 2 x 384 routed rows x 8192 x 4 B
constexpr size_t kPeerRegionMin = kPeerEpData + kPeerEpDataBytes;
constexpr size_t kPeerTpbBar = 384;             // u32: cross-GPU counter of the batched TP exchange
constexpr size_t kPeerTpbEpoch = 512;           // u32: batched TP exchanges this rank has completed (local)
constexpr size_t kPeerTpbDone = 640;            // u32: CTAs of the running exchange that finished (local)
constexpr size_t kPeerTpbData = kPeerRegionMin; // batched TP: down partials [2][ranks][rows x d_model] f32

// The all-reduce of a tensor-parallel FFN layer at any batch (tp_reduce.cu): x[n] += the sum
// over ranks (in rank order) of every rank's yp[n], through the exchange regions.  Every rank
// calls it with the same n; the region must hold tp_exchange_bytes(world, n).
size_t tp_exchange_bytes(int world, size_t n);
cudaError_t launch_tp_allreduce(const float* yp, float* x, size_t n, void* const* regions, int rank, int world,
                                int* err, cudaStream_t stream);

struct StackLaunch {
    const void* layers;  // device array, per layer {gate, up, down, norm weight} pointers
    int L, dm, ff;
    long long ts_a, ts_b;  // tile strides of gate/up and of down
    float* x;              // [dm], updated in place
    float eps;
    int* err;
    void* scratch;  // launch_ffn_stack(dry) reports its size
    // tensor parallelism over tp_size ranks (1 = off): the layers are this rank's d_ff shard,
    // the down partials go to every rank's exchange region
    int tp_rank, tp_size;
    void* const* tp_regions;  // device array [tp_size] of the ranks' regions as mapped here
    unsigned tp_base;         // cross-GPU phases completed before this launch
    unsigned tp_flow_base;    // of those, the phases the dataflow kernel ran (its per-tile counters)
    int* flow_used;           // set to 1 when the dataflow kernel took the launch (may be null)
};
// cudaErrorInvalidConfiguration: the shapes or formats are not covered (use the per-layer
// kernels).  dry = only check that the launch is possible and report the scratch bytes.
// Stacks the dataflow kernel covers (ffn_flow.cu; one GPU or tensor-parallel) run on it, the
// others on the phase-barrier kernel (ffn_stack.cu); HAYAI_FLOW_KERNEL=0 in the environment
// keeps every stack on the latter.
cudaError_t launch_ffn_stack(int type_a, int type_d, const StackLaunch& s, int num_sms, int smem_limit,
                             cudaStream_t stream, bool dry, size_t* scratch_bytes);
cudaError_t launch_ffn_flow(int type_a, int type_d, const StackLaunch& s, int num_sms, int smem_limit,
                            cudaStream_t stream, bool dry, size_t* scratch_bytes);

// Batched GEMV on the tcgen05 tensor cores (gemm_tc.cu) for Q8_0, Q4_K and Q6_K, 8..128 rows of
// x, M a multiple of 128 and K of the format's tile-block image (128 or 256).  w2 != nullptr:
// fused gate/up, y = silu(G x') * (U x') with x' = rms_norm(x) when norm_w is given.
// ws: tc_workspace_bytes(...) bytes of scratch.
bool tc_gemm_supported(int type, int M, int K, int nvec);
size_t tc_workspace_bytes(int type, int M, int K, int nvec, int num_sms, int mats);
cudaError_t launch_tc_gemm(int type, const uint8_t* w, const uint8_t* w2, long long tstride, int M, int K,
                           const float* x, int ldx, int nvec, float* y, int ldy, const float* resid, int ldr,
                           const float* norm_w, int norm_len, float eps, void* ws, int* err, int num_sms,
                           int smem_limit, cudaStream_t stream);

// CUDA-core GEMV on the raw GGUF layout for F32 and the IQ2/IQ3 codebook formats.
cudaError_t launch_gemv_simple(int type, const uint8_t* w, size_t row_bytes, int M, int K, const float* x,
                               int ldx, float* y, int ldy, const float* resid, int ldr, int nvec,
                               cudaStream_t stream);
bool gemv_simple_supported(int type);

// Toy LUT-Q4 matmul (16-entry LUT, two nibbles per byte, low nibble first).
cudaError_t launch_lut_matmul_q4(const uint8_t* w, int M, int N, const float* lut16, const float* x, float* y,
                                 cudaStream_t stream);

// RMSNorm rows: out[v][i] = (x[v][i] * inv_v) * w[i] for i < len, 0 for len <= i < K.
cudaError_t launch_rms_norm(const float* x, int ldx, const float* w, int len, int K, float eps, float* out, int ldo,
                            int nvec, cudaStream_t stream);

// Elementwise SwiGLU h = silu(g) * u, with an optional residual for out = resid + ...
cudaError_t launch_swiglu(const float* g, const float* u, float* h, size_t n, cudaStream_t stream);

// Upload repack: raw GGUF rows -> GPU layout.  Q4_K, Q6_K and Q8_0 become tile-major
// (16-row tiles of contiguous tile-block images); the other formats keep their rows.
bool tiled_type(int type);
size_t tile_block_bytes(int type);                 // bytes of one 16-row x kernel-block image
size_t gpu_stride(int type, int K);                // bytes per tile (tiled) or per row
size_t gpu_weight_bytes(int type, int M, int K);   // bytes of the whole GPU image
size_t raw_row_bytes(int type, int K);
cudaError_t launch_repack(int type, const uint8_t* raw, uint8_t* gpu, int M, int K, cudaStream_t stream);

}  // namespace hc
