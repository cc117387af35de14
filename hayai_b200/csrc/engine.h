// engine.h -- internal definitions of the C-ABI objects (not part of the public header).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <unordered_map>

struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    int ensure(size_t n);
    void release();
};

struct HostBuf {
    void* p = nullptr;
    size_t cap = 0;
    int ensure(size_t n);
    void release();
};

// Exchange region shared with the other ranks of a tensor- or expert-parallel group (one
// process per GPU; the regions are mapped into each other's address space with CUDA IPC, so
// kernels store into a peer's region over NVLink).  Every rank's region has the same layout
// (gemv_launch.h, kPeer*).
constexpr int kMaxPeers = 8;
struct PeerState {
    int rank = 0, world = 1;
    void* region = nullptr;      // this rank's region (exported)
    size_t bytes = 0;
    void* peer[kMaxPeers] = {};  // every rank's region as mapped here (peer[rank] = region)
    void** d_peer = nullptr;     // device copy of peer[]
    bool connected = false;
    uint32_t tp_phases = 0;      // cross-GPU phases of the TP stack run so far (equal on every rank)
    uint32_t flow_phases = 0;    // of those, the phases run by the dataflow stack kernel
};

// One GPU + stream: the counterpart of OpenClEngine (crates/hayai-opencl/src/context.rs:23).
struct hc_engine {
    int device = 0;
    int num_sms = 0;
    int smem_optin = 0;
    cudaStream_t stream = nullptr;      // stream all work is enqueued on
    cudaStream_t own_stream = nullptr;  // the engine's own stream
    int* d_err = nullptr;               // device error flags (bit 0: f16 range, bit 1: wait timeout)
    int* h_err = nullptr;               // pinned host copy of d_err, read back with a call's results
    bool use_graphs = true;
    // grow-on-demand workspaces (the reference's GemvSyncWorkspace, compute.rs:10-17)
    DevBuf ws_raw, ws_gpu, ws_x, ws_y, ws_h, ws_g, ws_u, ws_misc;
    // stream-K partial sums and per-tile counters (counters zeroed once; kernels re-arm them)
    DevBuf sk_ws, sk_cnt;
    DevBuf stack_bar;             // grid-barrier counter of the persistent FFN-stack kernel
    DevBuf ws_tc;                 // batched Q8_0 tensor-core GEMM: canonical activations + partials
    DevBuf ws_tp;                 // tensor parallelism at batch > 1: this rank's down partial
    bool use_stack_kernel = true; // batch-1 stacks run as one persistent kernel when they fit
    bool use_tc = true;           // batches of 8+ rows of Q8_0/Q4_K/Q6_K on the tcgen05 GEMM
    HostBuf hs_out;
    std::unordered_map<uint64_t, cudaGraphExec_t> graphs;  // captured FFN stacks
    std::unordered_map<uint64_t, void*> ptr_tables;        // device tables of expert pointers
    PeerState peer;                                        // tensor/expert-parallel group
};

// A resident weight matrix in the GPU layout of its format.
struct hc_weights {
    int type = 0;
    size_t m = 0, n = 0;
    size_t stride = 0;  // bytes per row in the GPU layout
    size_t bytes = 0;
    void* dev = nullptr;
    int device = 0;
};

// internal helpers shared by the translation units of the C ABI
int hc_set_error(int code, const char* fmt, ...);
int hc_cuda_error(cudaError_t e, const char* what);

#define HC_CUDA(call)                                           \
    do {                                                        \
        cudaError_t _e = (call);                                \
        if (_e != cudaSuccess) return hc_cuda_error(_e, #call); \
    } while (0)

void hc_peer_release(hc_engine* e);  // unmap the peers' regions and free this rank's
int hc_engine_activate(hc_engine* e);
int hc_check_device_error(hc_engine* e);
// Synchronises the engine's stream and reports the device error flag, read back behind the
// work already enqueued (one stream synchronisation instead of two round trips).
int hc_finish_sync(hc_engine* e);
int hc_launch_gemv(hc_engine* e, const hc_weights* w, const float* x, size_t ldx, float* y, size_t ldy,
                   const float* resid, size_t ldr, size_t nvec);
int hc_launch_gateup(hc_engine* e, const hc_weights* g, const hc_weights* u, const float* x, size_t ldx, float* h,
                     size_t nvec, const float* norm_w, size_t norm_len, float eps);
int hc_launch_ffn(hc_engine* e, const hc_weights* g, const hc_weights* u, const hc_weights* d, const float* x,
                  size_t ldx, float* y, size_t ldy, const float* resid, size_t ldr, float* h_ws, size_t nvec,
                  const float* norm_w, size_t norm_len, float eps);
const char* hc_type_label(int t);
// Make the stream-K workspace large enough for an M x K launch of `type`; a reallocation
// drops the captured CUDA graphs (they hold the old addresses).
int hc_sk_prepare(hc_engine* e, int type, size_t M, size_t K, bool fused, float** ws, int** cnt);
void hc_drop_graphs(hc_engine* e);
// Scratch of the batched Q8_0 tensor-core GEMM (grows on demand; a reallocation drops the
// captured CUDA graphs).
int hc_tc_prepare(hc_engine* e, int type, size_t M, size_t K, size_t nvec, int mats, void** ws);
