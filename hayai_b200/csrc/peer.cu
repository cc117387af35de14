// peer.cu -- the exchange region of a tensor- or expert-parallel group (C ABI).
//
// One process drives one GPU.  Each rank allocates a region, exports it as a CUDA IPC handle,
// and maps every other rank's region from the handles the caller gathered (over its own
// process group).  Kernels then store partial results straight into the peers' regions over
// NVLink and signal with system-scope atomics on a counter in each region; the fused
// collective (gemv output -> every rank) needs no separate library call.  No reference
// counterpart: the reference has no multi-GPU FFN path.
#include <cuda_runtime.h>
#include <string.h>

#include "engine.h"
#include "gemv_launch.h"
#include "hayai_cuda.h"

using hc::kPeerRegionMin;

void hc_peer_release(hc_engine* e) {
    PeerState& p = e->peer;
    for (int r = 0; r < kMaxPeers; ++r) {
        if (p.peer[r] && r != p.rank && p.connected) cudaIpcCloseMemHandle(p.peer[r]);
        p.peer[r] = nullptr;
    }
    if (p.d_peer) cudaFree(p.d_peer);
    if (p.region) cudaFree(p.region);
    p = PeerState{};
}

extern "C" int hc_peer_open(hc_engine* e, int rank, int world, size_t bytes, void* handle_out) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
        return hc_set_error(HC_ERR_INVALID, "peer group: rank %d of %d (1..%d ranks)", rank, world, kMaxPeers);
    if (bytes < kPeerRegionMin)
        return hc_set_error(HC_ERR_INVALID, "peer region of %zu bytes is below the %zu-byte minimum", bytes,
                            (size_t)kPeerRegionMin);
    if (!handle_out) return hc_set_error(HC_ERR_INVALID, "null handle");
    HC_CUDA(cudaStreamSynchronize(e->stream));
    hc_peer_release(e);
    PeerState& p = e->peer;
    HC_CUDA(cudaMalloc(&p.region, bytes));
    p.bytes = bytes;
    p.rank = rank;
    p.world = world;
    cudaError_t ce = cudaMemset(p.region, 0, bytes);  // counters start at zero on every rank
    cudaIpcMemHandle_t h;
    if (ce == cudaSuccess) ce = cudaIpcGetMemHandle(&h, p.region);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) {
        hc_peer_release(e);
        return hc_cuda_error(ce, "peer region");
    }
    memcpy(handle_out, &h, sizeof(h));
    return HC_OK;
}

extern "C" int hc_peer_connect(hc_engine* e, const void* handles) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    PeerState& p = e->peer;
    if (!p.region) return hc_set_error(HC_ERR_INVALID, "peer group not opened");
    if (!handles) return hc_set_error(HC_ERR_INVALID, "null handles");
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) {
            p.peer[r] = p.region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
        cudaError_t ce = cudaIpcOpenMemHandle(&p.peer[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (ce != cudaSuccess) {
            p.peer[r] = nullptr;
            for (int q = 0; q < r; ++q)
                if (q != p.rank && p.peer[q]) {
                    cudaIpcCloseMemHandle(p.peer[q]);
                    p.peer[q] = nullptr;
                }
            return hc_cuda_error(ce, "mapping a peer's region");
        }
    }
    p.connected = true;
    HC_CUDA(cudaMalloc(&p.d_peer, kMaxPeers * sizeof(void*)));
    HC_CUDA(cudaMemcpy(p.d_peer, p.peer, kMaxPeers * sizeof(void*), cudaMemcpyHostToDevice));
    return HC_OK;
}

extern "C" int hc_peer_close(hc_engine* e) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    HC_CUDA(cudaStreamSynchronize(e->stream));
    hc_peer_release(e);
    return HC_OK;
}

extern "C" int hc_peer_region(hc_engine* e, void** region, size_t* bytes) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!region || !bytes) return hc_set_error(HC_ERR_INVALID, "null argument");
    if (!e->peer.region) return hc_set_error(HC_ERR_INVALID, "peer group not opened");
    *region = e->peer.region;
    *bytes = e->peer.bytes;
    return HC_OK;
}

extern "C" int hc_peer_handle_bytes(size_t* out) {
    if (!out) return hc_set_error(HC_ERR_INVALID, "null argument");
    *out = sizeof(cudaIpcMemHandle_t);
    return HC_OK;
}
