// capi.cu -- the C ABI (include/hayai_cuda.h): engine, resident weights, GEMV and FFN
// entry points.  Host logic mirrors hayai-opencl's OpenClEngine
// (crates/hayai-opencl/src/compute.rs, async_gemv.rs): the same validation and error
// behaviour, with CUDA streams and one-time resident uploads instead of per-call
// buffer creation.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/hayai_cuda.h"
#include "common.cuh"
#include "engine.h"
#include "gemv_launch.h"
#include "gemv_mma.cuh"

using namespace hc;

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

int hc_set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int hc_cuda_error(cudaError_t e, const char* what) {
    return hc_set_error(HC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" const char* hc_last_error(void) { return g_last_error.c_str(); }

// ------------------------------------------------------------------ labels / row bytes
const char* hc_type_label(int t) {
    switch (t) {
        case T_F32: return "f32";
        case T_Q8_0: return "q8_0";
        case T_Q4_K: return "q4_k";
        case T_Q6_K: return "q6_k";
        case T_IQ2_XXS: return "iq2_xxs";
        case T_IQ2_XS: return "iq2_xs";
        case T_IQ2_S: return "iq2_s";
        case T_IQ3_XXS: return "iq3_xxs";
        case T_IQ3_S: return "iq3_s";
        case T_Q4_0: return "q4_0";
        case T_Q4_1: return "q4_1";
        case T_Q5_0: return "q5_0";
        case T_Q5_1: return "q5_1";
        case T_Q2_K: return "q2_k";
        case T_Q3_K: return "q3_k";
        case T_Q5_K: return "q5_k";
        case T_IQ4_NL: return "iq4_nl";
        case T_IQ4_XS: return "iq4_xs";
        case T_F16: return "f16";
        case T_BF16: return "bf16";
        case T_Q8_1: return "q8_1";
        case T_Q8_K: return "q8_k";
        default: return "unknown";
    }
}

static int block_elems(int t) {
    switch (t) {
        case T_F32: case T_F16: case T_BF16: return 1;
        case T_Q8_0: case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_IQ4_NL: case T_Q8_1: return 32;
        case T_Q4_K: case T_Q6_K: case T_IQ2_XXS: case T_IQ2_XS: case T_IQ2_S: case T_IQ3_XXS: case T_IQ3_S:
        case T_Q2_K: case T_Q3_K: case T_Q5_K: case T_IQ4_XS: case T_Q8_K:
            return 256;
        default: return 0;
    }
}

// gemv_row_bytes (compute.rs:877-907) restricted to the formats with a kernel here.
extern "C" int hc_gemv_row_bytes(int ggml_type, size_t n, size_t* out) {
    const int qk = block_elems(ggml_type);
    if (qk == 0) return hc_set_error(HC_ERR_UNSUPPORTED, "CUDA GEMV missing for ggml type %d", ggml_type);
    if (n % (size_t)qk != 0)
        return hc_set_error(HC_ERR_INVALID, "ggml_gemv_%s: n=%zu is not a valid column count for this layout",
                            hc_type_label(ggml_type), n);
    if (out) *out = raw_row_bytes(ggml_type, (int)n);
    return HC_OK;
}

// validate_gemv_shape (compute.rs:937-951)
int hc_validate_shape(int type, size_t m, size_t n) {
    if (block_elems(type) == 0) return hc_set_error(HC_ERR_UNSUPPORTED, "CUDA GEMV missing for ggml type %d", type);
    if (m == 0 || n == 0)
        return hc_set_error(HC_ERR_INVALID, "ggml_gemv_%s: empty shape m=%zu n=%zu", hc_type_label(type), m, n);
    if (m > (size_t)INT32_MAX || n > (size_t)INT32_MAX)
        return hc_set_error(HC_ERR_INVALID, "ggml_gemv_%s: shape too large m=%zu n=%zu", hc_type_label(type), m, n);
    if (n % (size_t)block_elems(type) != 0)
        return hc_set_error(HC_ERR_INVALID,
                            "ggml_gemv_%s: n=%zu is not a valid column count (multiple of the block size)",
                            hc_type_label(type), n);
    return HC_OK;
}

// validate_gemv_weights (compute.rs:912-933)
int hc_validate_weights(int type, size_t m, size_t n, size_t len) {
    int rc = hc_validate_shape(type, m, n);
    if (rc) return rc;
    const size_t row = raw_row_bytes(type, (int)n);
    if (row != 0 && m > SIZE_MAX / row)
        return hc_set_error(HC_ERR_INVALID, "ggml_gemv_%s: weight size overflow for %zux%zu", hc_type_label(type), m, n);
    const size_t expected = m * row;
    if (len < expected)
        return hc_set_error(HC_ERR_INVALID, "ggml_gemv_%s: weight buffer %zu B < %zu B required for %zux%zu",
                            hc_type_label(type), len, expected, m, n);
    return HC_OK;
}

// ------------------------------------------------------------------ engine
int DevBuf::ensure(size_t n) {
    if (n <= cap) return HC_OK;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    cudaError_t e = cudaMalloc(&p, n);
    if (e != cudaSuccess) {
        p = nullptr;
        return hc_cuda_error(e, "workspace cudaMalloc");
    }
    cap = n;
    return HC_OK;
}

void DevBuf::release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
}

int HostBuf::ensure(size_t n) {
    if (n <= cap) return HC_OK;
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
    cudaError_t e = cudaMallocHost(&p, n);
    if (e != cudaSuccess) {
        p = nullptr;
        return hc_cuda_error(e, "pinned cudaMallocHost");
    }
    cap = n;
    return HC_OK;
}

void HostBuf::release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
}

int hc_engine_activate(hc_engine* e) {
    if (!e) return hc_set_error(HC_ERR_INVALID, "null engine");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != e->device) HC_CUDA(cudaSetDevice(e->device));
    return HC_OK;
}

extern "C" int hc_device_count(int* out) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        if (out) *out = 0;
        return hc_cuda_error(e, "cudaGetDeviceCount");
    }
    if (out) *out = n;
    return HC_OK;
}

extern "C" int hc_engine_init(int device, hc_engine** out) {
    if (!out) return hc_set_error(HC_ERR_INVALID, "null out pointer");
    *out = nullptr;
    int n = 0;
    HC_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return hc_set_error(HC_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    HC_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    HC_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return hc_set_error(HC_ERR_UNSUPPORTED, "device %d (%s, sm_%d%d) is not an sm_100 part", device, prop.name,
                            prop.major, prop.minor);
    hc_engine* e = new hc_engine();
    e->device = device;
    e->num_sms = prop.multiProcessorCount;
    e->smem_optin = (int)prop.sharedMemPerBlockOptin;
    cudaError_t ce = cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking);
    if (ce != cudaSuccess) {
        delete e;
        return hc_cuda_error(ce, "cudaStreamCreate");
    }
    e->stream = e->own_stream;
    // HAYAI_STACK_KERNEL=0 keeps batch-1 FFN stacks on the per-layer kernels
    const char* sk = getenv("HAYAI_STACK_KERNEL");
    if (sk && sk[0] == '0') e->use_stack_kernel = false;
    // HAYAI_TC_GEMM=0 keeps batches on the mma.sync GEMV (one weight pass per 4 rows)
    const char* tc = getenv("HAYAI_TC_GEMM");
    if (tc && tc[0] == '0') e->use_tc = false;
    ce = cudaMalloc(&e->d_err, 16);
    if (ce == cudaSuccess) ce = cudaMemset(e->d_err, 0, 16);
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->h_err, 16);
    if (ce != cudaSuccess) {
        if (e->d_err) cudaFree(e->d_err);
        cudaStreamDestroy(e->own_stream);
        delete e;
        return hc_cuda_error(ce, "error flag allocation");
    }
    *out = e;
    return HC_OK;
}

extern "C" int hc_engine_free(hc_engine* e) {
    if (!e) return HC_OK;
    hc_engine_activate(e);
    cudaStreamSynchronize(e->stream);
    hc_drop_graphs(e);
    e->sk_ws.release();
    e->sk_cnt.release();
    e->stack_bar.release();
    e->ws_tc.release();
    hc_peer_release(e);
    for (auto& kv : e->ptr_tables) cudaFree(kv.second);
    e->ptr_tables.clear();
    e->ws_raw.release();
    e->ws_gpu.release();
    e->ws_x.release();
    e->ws_y.release();
    e->ws_h.release();
    e->ws_g.release();
    e->ws_u.release();
    e->ws_misc.release();
    e->hs_out.release();
    if (e->d_err) cudaFree(e->d_err);
    if (e->h_err) cudaFreeHost(e->h_err);
    if (e->own_stream) cudaStreamDestroy(e->own_stream);
    delete e;
    return HC_OK;
}

void hc_drop_graphs(hc_engine* e) {
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
}

int hc_tc_prepare(hc_engine* e, int type, size_t M, size_t K, size_t nvec, int mats, void** ws) {
    const size_t need = tc_workspace_bytes(type, (int)M, (int)K, (int)nvec, e->num_sms, mats);
    if (need > e->ws_tc.cap) {
        cudaStreamSynchronize(e->stream);
        hc_drop_graphs(e);  // graphs captured earlier hold the old address
        e->ws_tc.release();
        int rc = e->ws_tc.ensure(need);
        if (rc) return rc;
    }
    *ws = e->ws_tc.p;
    return HC_OK;
}

int hc_sk_prepare(hc_engine* e, int type, size_t M, size_t K, bool fused, float** ws, int** cnt) {
    size_t nws = 0, ncnt = 0;
    gemv_sk_workspace(type, (int)M, (int)K, fused, e->num_sms, &nws, &ncnt);
    nws *= sizeof(float);
    ncnt *= sizeof(int);
    if (nws > e->sk_ws.cap || ncnt > e->sk_cnt.cap) {
        // graphs captured earlier hold the old addresses
        cudaStreamSynchronize(e->stream);
        hc_drop_graphs(e);
        const size_t want_ws = nws > e->sk_ws.cap ? nws : e->sk_ws.cap;
        const size_t want_cnt = ncnt > e->sk_cnt.cap ? ncnt : e->sk_cnt.cap;
        e->sk_ws.release();
        e->sk_cnt.release();
        int rc = e->sk_ws.ensure(want_ws);
        if (!rc) rc = e->sk_cnt.ensure(want_cnt);
        if (rc) return rc;
        HC_CUDA(cudaMemset(e->sk_cnt.p, 0, e->sk_cnt.cap));
    }
    *ws = (float*)e->sk_ws.p;
    *cnt = (int*)e->sk_cnt.p;
    return HC_OK;
}

extern "C" int hc_engine_set_stream(hc_engine* e, void* stream) {
    if (!e) return hc_set_error(HC_ERR_INVALID, "null engine");
    // NULL is CUDA's legacy default stream (the stream torch calls "default"), used as is
    e->stream = stream ? (cudaStream_t)stream : cudaStreamLegacy;
    return HC_OK;
}

extern "C" int hc_engine_use_own_stream(hc_engine* e) {
    if (!e) return hc_set_error(HC_ERR_INVALID, "null engine");
    e->stream = e->own_stream;
    return HC_OK;
}

extern "C" int hc_engine_get_stream(hc_engine* e, void** stream) {
    if (!e || !stream) return hc_set_error(HC_ERR_INVALID, "null argument");
    *stream = (void*)e->stream;
    return HC_OK;
}

// Read (and clear) the device error flag.  Call only after the stream is synchronised.
static int flag_error(hc_engine* e, int flag);

int hc_check_device_error(hc_engine* e) {
    int flag = 0;
    HC_CUDA(cudaMemcpy(&flag, e->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    return flag_error(e, flag);
}

// The end of a host-buffer call: the error flag travels back on the stream behind the call's
// results, so one stream synchronisation covers both.
int hc_finish_sync(hc_engine* e) {
    HC_CUDA(cudaMemcpyAsync(e->h_err, e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    HC_CUDA(cudaStreamSynchronize(e->stream));
    return flag_error(e, *e->h_err);
}

static int flag_error(hc_engine* e, int flag) {
    if (flag) {
        HC_CUDA(cudaMemset(e->d_err, 0, sizeof(int)));
        if (flag & 1)
            return hc_set_error(HC_ERR_RANGE,
                                "an activation magnitude reached 65504 (outside the f16 range of the tensor-core split)");
        if (flag & 2) return hc_set_error(HC_ERR_TIMEOUT, "a bounded device wait expired");
        return hc_set_error(HC_ERR_CUDA, "device error flag 0x%x", flag);
    }
    return HC_OK;
}

extern "C" int hc_sync(hc_engine* e) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    return hc_finish_sync(e);
}

// ------------------------------------------------------------------ weights
static int weights_make(hc_engine* e, int type, size_t m, size_t n, const void* src, size_t len, bool from_host,
                        hc_weights** out) {
    if (!out) return hc_set_error(HC_ERR_INVALID, "null out pointer");
    *out = nullptr;
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    rc = hc_validate_weights(type, m, n, len);
    if (rc) return rc;
    if (!src) return hc_set_error(HC_ERR_INVALID, "null weight bytes");
    const size_t raw_rb = raw_row_bytes(type, (int)n);
    const size_t gpu_rb = gpu_stride(type, (int)n);
    const size_t raw_bytes = m * raw_rb, gpu_bytes = gpu_weight_bytes(type, (int)m, (int)n);
    hc_weights* w = new hc_weights();
    w->type = type;
    w->m = m;
    w->n = n;
    w->stride = gpu_rb;
    w->bytes = gpu_bytes;
    w->device = e->device;
    cudaError_t ce = cudaMalloc(&w->dev, gpu_bytes + 16);
    if (ce != cudaSuccess) {
        delete w;
        return hc_cuda_error(ce, "weights cudaMalloc");
    }
    const uint8_t* raw_dev = nullptr;
    void* tmp = nullptr;
    const bool same_layout = !tiled_type(type);
    if (from_host) {
        if (same_layout) {
            ce = cudaMemcpyAsync(w->dev, src, raw_bytes, cudaMemcpyHostToDevice, e->stream);
        } else {
            ce = cudaMalloc(&tmp, raw_bytes);
            if (ce == cudaSuccess) ce = cudaMemcpyAsync(tmp, src, raw_bytes, cudaMemcpyHostToDevice, e->stream);
            raw_dev = (const uint8_t*)tmp;
        }
    } else {
        raw_dev = (const uint8_t*)src;
        if (same_layout) ce = cudaMemcpyAsync(w->dev, src, raw_bytes, cudaMemcpyDeviceToDevice, e->stream);
    }
    if (ce == cudaSuccess && !same_layout) ce = launch_repack(type, raw_dev, (uint8_t*)w->dev, (int)m, (int)n, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    if (tmp) cudaFree(tmp);
    if (ce != cudaSuccess) {
        cudaFree(w->dev);
        delete w;
        return hc_cuda_error(ce, "weights upload");
    }
    *out = w;
    return HC_OK;
}

extern "C" int hc_weights_upload(hc_engine* e, int type, size_t m, size_t n, const void* host, size_t len,
                                 hc_weights** out) {
    return weights_make(e, type, m, n, host, len, true, out);
}

extern "C" int hc_weights_from_device(hc_engine* e, int type, size_t m, size_t n, const void* dev, size_t len,
                                      hc_weights** out) {
    return weights_make(e, type, m, n, dev, len, false, out);
}

extern "C" int hc_weights_free(hc_weights* w) {
    if (!w) return HC_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    const bool other = cur != w->device;
    if (other) cudaSetDevice(w->device);
    cudaFree(w->dev);
    if (other && cur >= 0) cudaSetDevice(cur);  // leave the caller's device current
    delete w;
    return HC_OK;
}

extern "C" int hc_weights_info(const hc_weights* w, int* type, size_t* m, size_t* n, size_t* bytes) {
    if (!w) return hc_set_error(HC_ERR_INVALID, "null weights");
    if (type) *type = w->type;
    if (m) *m = w->m;
    if (n) *n = w->n;
    if (bytes) *bytes = w->bytes;
    return HC_OK;
}

// ------------------------------------------------------------------ GEMV core
int hc_launch_gemv(hc_engine* e, const hc_weights* w, const float* x, size_t ldx, float* y, size_t ldy,
                   const float* resid, size_t ldr, size_t nvec) {
    if (!w || !x || !y) return hc_set_error(HC_ERR_INVALID, "null argument");
    if (w->device != e->device) return hc_set_error(HC_ERR_INVALID, "weights live on device %d, engine on %d", w->device, e->device);
    if (nvec == 0) return HC_OK;
    if (ldx < w->n || ldy < w->m || (resid && ldr < w->m))
        return hc_set_error(HC_ERR_INVALID, "leading dimension smaller than the row length");
    // the element formats take any row length (their kernels fall back to scalar loads); the
    // block formats' kernels read x as float4
    const bool elem = w->type == T_F32 || w->type == T_F16 || w->type == T_BF16;
    if (!elem && (((uintptr_t)x & 15) || (ldx & 3)))
        return hc_set_error(HC_ERR_INVALID, "x must be 16-byte aligned with ldx a multiple of 4");
    cudaError_t ce;
    if (e->use_tc && tc_gemm_supported(w->type, (int)w->m, (int)w->n, (int)nvec)) {
        // batches of 8+ rows: one pass over the weights on the tcgen05 tensor cores
        void* ws;
        int rc = hc_tc_prepare(e, w->type, w->m, w->n, nvec, 1, &ws);
        if (rc) return rc;
        ce = launch_tc_gemm(w->type, (const uint8_t*)w->dev, nullptr, (long long)w->stride, (int)w->m, (int)w->n, x, (int)ldx,
                            (int)nvec, y, (int)ldy, resid, (int)ldr, nullptr, 0, 0.f, ws, e->d_err, e->num_sms,
                            e->smem_optin, e->stream);
    } else if (gemv_mma_supported(w->type)) {
        GemvArgs a{};
        a.w = (const uint8_t*)w->dev;
        a.row_stride = (long long)w->stride;
        a.M = (int)w->m;
        a.K = (int)w->n;
        a.x = x;
        a.ldx = (int)ldx;
        a.y = y;
        a.ldy = (int)ldy;
        a.resid = resid;
        a.ldr = (int)ldr;
        a.w2 = nullptr;
        a.err = e->d_err;
        int rc = hc_sk_prepare(e, w->type, w->m, w->n, false, &a.sk_ws, &a.sk_cnt);
        if (rc) return rc;
        ce = launch_gemv_mma(w->type, a, (int)nvec, false, e->num_sms, e->smem_optin, e->stream);
    } else if (gemv_simple_supported(w->type)) {
        ce = launch_gemv_simple(w->type, (const uint8_t*)w->dev, w->stride, (int)w->m, (int)w->n, x, (int)ldx, y,
                                (int)ldy, resid, (int)ldr, (int)nvec, e->stream);
    } else {
        return hc_set_error(HC_ERR_UNSUPPORTED, "CUDA GEMV missing for %s", hc_type_label(w->type));
    }
    if (ce != cudaSuccess) return hc_cuda_error(ce, "gemv launch");
    return HC_OK;
}

extern "C" int hc_gemv_dev(hc_engine* e, const hc_weights* w, const float* x, size_t ldx, float* y, size_t ldy,
                           const float* resid, size_t ldr, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    return hc_launch_gemv(e, w, x, ldx, y, ldy, resid, ldr, nvec);
}

// Blocking host-buffer GEMV through resident weights.
static int gemv_host(hc_engine* e, const hc_weights* w, const float* in, float* out, size_t nvec) {
    if (!w || !in || !out) return hc_set_error(HC_ERR_INVALID, "null argument");
    const size_t n = w->n, m = w->m;
    int rc = e->ws_x.ensure(nvec * n * 4);
    if (!rc) rc = e->ws_y.ensure(nvec * m * 4);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(e->ws_x.p, in, nvec * n * 4, cudaMemcpyHostToDevice, e->stream));
    rc = hc_launch_gemv(e, w, (const float*)e->ws_x.p, n, (float*)e->ws_y.p, m, nullptr, 0, nvec);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(out, e->ws_y.p, nvec * m * 4, cudaMemcpyDeviceToHost, e->stream));
    return hc_finish_sync(e);
}

extern "C" int hc_ggml_gemv_bound(hc_engine* e, const hc_weights* w, const float* in, float* out) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    return gemv_host(e, w, in, out, 1);
}

extern "C" int hc_ggml_gemv_batched(hc_engine* e, const hc_weights* w, const float* in, float* out, size_t batch) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (batch == 0) return HC_OK;
    return gemv_host(e, w, in, out, batch);
}

// ggml_gemv_dispatch: host weights are staged into the engine workspace every call
// (the reference does the same with its GemvSyncWorkspace, compute.rs:302-333).
extern "C" int hc_ggml_gemv_dispatch(hc_engine* e, int type, size_t m, size_t n, const uint8_t* weights, size_t len,
                                     const float* in, float* out) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    rc = hc_validate_weights(type, m, n, len);
    if (rc) return rc;
    if (!weights || !in || !out) return hc_set_error(HC_ERR_INVALID, "null argument");
    const size_t raw_bytes = m * raw_row_bytes(type, (int)n), gpu_rb = gpu_stride(type, (int)n);
    const size_t gpu_bytes = gpu_weight_bytes(type, (int)m, (int)n);
    rc = e->ws_raw.ensure(raw_bytes);
    if (!rc) rc = e->ws_gpu.ensure(gpu_bytes + 16);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(e->ws_raw.p, weights, raw_bytes, cudaMemcpyHostToDevice, e->stream));
    cudaError_t ce = launch_repack(type, (const uint8_t*)e->ws_raw.p, (uint8_t*)e->ws_gpu.p, (int)m, (int)n, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "repack");
    hc_weights tmp;
    tmp.type = type;
    tmp.m = m;
    tmp.n = n;
    tmp.stride = gpu_rb;
    tmp.bytes = gpu_bytes;
    tmp.dev = e->ws_gpu.p;
    tmp.device = e->device;
    return gemv_host(e, &tmp, in, out, 1);
}

// ------------------------------------------------------------------ async
struct hc_pending {
    hc_engine* eng = nullptr;
    void* d_x = nullptr;
    float* d_y = nullptr;
    float* h_y = nullptr;
    size_t m = 0;
    cudaEvent_t done = nullptr;
    bool waited = false;
};

extern "C" int hc_ggml_gemv_async(hc_engine* e, const hc_weights* w, const float* in, hc_pending** out) {
    if (!out) return hc_set_error(HC_ERR_INVALID, "null out pointer");
    *out = nullptr;
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!w || !in) return hc_set_error(HC_ERR_INVALID, "null argument");
    hc_pending* p = new hc_pending();
    p->eng = e;
    p->m = w->m;
    cudaError_t ce = cudaMalloc(&p->d_x, w->n * 4);
    if (ce == cudaSuccess) ce = cudaMalloc((void**)&p->d_y, w->m * 4);
    if (ce == cudaSuccess) ce = cudaMallocHost((void**)&p->h_y, w->m * 4);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(p->d_x, in, w->n * 4, cudaMemcpyHostToDevice, e->stream);
    if (ce != cudaSuccess) {
        hc_pending_free(p);
        return hc_cuda_error(ce, "async gemv setup");
    }
    rc = hc_launch_gemv(e, w, (const float*)p->d_x, w->n, p->d_y, w->m, nullptr, 0, 1);
    if (rc) {
        hc_pending_free(p);
        return rc;
    }
    ce = cudaMemcpyAsync(p->h_y, p->d_y, w->m * 4, cudaMemcpyDeviceToHost, e->stream);
    if (ce == cudaSuccess) ce = cudaEventRecord(p->done, e->stream);
    if (ce != cudaSuccess) {
        hc_pending_free(p);
        return hc_cuda_error(ce, "async gemv enqueue");
    }
    *out = p;
    return HC_OK;
}

extern "C" int hc_pending_wait(hc_pending* p, float* output, size_t m) {
    if (!p) return hc_set_error(HC_ERR_INVALID, "null pending");
    int rc = hc_engine_activate(p->eng);
    if (rc) return rc;
    if (!p->waited) {
        HC_CUDA(cudaEventSynchronize(p->done));
        p->waited = true;
        rc = hc_check_device_error(p->eng);
        if (rc) return rc;
    }
    if (output) {
        if (m < p->m) return hc_set_error(HC_ERR_INVALID, "output holds %zu floats, GEMV produced %zu", m, p->m);
        memcpy(output, p->h_y, p->m * 4);
    }
    return HC_OK;
}

extern "C" int hc_pending_free(hc_pending* p) {
    if (!p) return HC_OK;
    if (p->eng) hc_engine_activate(p->eng);
    // never free buffers a copy may still target (PendingGemv::drop, async_gemv.rs:48-57)
    if (p->done && !p->waited) cudaEventSynchronize(p->done);
    if (p->done) cudaEventDestroy(p->done);
    if (p->d_x) cudaFree(p->d_x);
    if (p->d_y) cudaFree(p->d_y);
    if (p->h_y) cudaFreeHost(p->h_y);
    delete p;
    return HC_OK;
}

// ------------------------------------------------------------------ LUT-Q4
extern "C" int hc_lut_matmul_q4_dev(hc_engine* e, size_t m, size_t n, const uint8_t* w, const float* lut16,
                                    const float* x, float* y) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (m == 0 || n == 0 || n % 2) return hc_set_error(HC_ERR_INVALID, "lut_matmul_q4: N must be even and non-zero");
    if (!w || !lut16 || !x || !y) return hc_set_error(HC_ERR_INVALID, "null argument");
    cudaError_t ce = launch_lut_matmul_q4(w, (int)m, (int)n, lut16, x, y, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "lut_matmul_q4 launch");
    return HC_OK;
}

extern "C" int hc_lut_matmul_q4(hc_engine* e, size_t m, size_t n, const uint8_t* w, const float* lut16,
                                const float* x, float* y) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (m == 0 || n == 0 || n % 2) return hc_set_error(HC_ERR_INVALID, "lut_matmul_q4: N must be even and non-zero");
    if (!w || !lut16 || !x || !y) return hc_set_error(HC_ERR_INVALID, "null argument");
    const size_t wb = m * (n / 2);
    rc = e->ws_raw.ensure(wb + 64);
    if (!rc) rc = e->ws_x.ensure(n * 4);
    if (!rc) rc = e->ws_y.ensure(m * 4);
    if (rc) return rc;
    uint8_t* dw = (uint8_t*)e->ws_raw.p;
    float* dlut = (float*)(dw + (wb + 15) / 16 * 16);
    if ((wb + 15) / 16 * 16 + 64 > e->ws_raw.cap) {
        rc = e->ws_raw.ensure((wb + 15) / 16 * 16 + 64);
        if (rc) return rc;
        dw = (uint8_t*)e->ws_raw.p;
        dlut = (float*)(dw + (wb + 15) / 16 * 16);
    }
    HC_CUDA(cudaMemcpyAsync(dw, w, wb, cudaMemcpyHostToDevice, e->stream));
    HC_CUDA(cudaMemcpyAsync(dlut, lut16, 64, cudaMemcpyHostToDevice, e->stream));
    HC_CUDA(cudaMemcpyAsync(e->ws_x.p, x, n * 4, cudaMemcpyHostToDevice, e->stream));
    cudaError_t ce = launch_lut_matmul_q4(dw, (int)m, (int)n, dlut, (const float*)e->ws_x.p, (float*)e->ws_y.p, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "lut_matmul_q4 launch");
    HC_CUDA(cudaMemcpyAsync(y, e->ws_y.p, m * 4, cudaMemcpyDeviceToHost, e->stream));
    HC_CUDA(cudaStreamSynchronize(e->stream));
    return HC_OK;
}

// ------------------------------------------------------------------ FFN
static int check_ffn(const hc_weights* g, const hc_weights* u, const hc_weights* d) {
    if (!g || !u || !d) return hc_set_error(HC_ERR_INVALID, "null FFN weights");
    if (g->m != u->m || g->n != u->n)
        return hc_set_error(HC_ERR_INVALID, "gate %zux%zu and up %zux%zu shapes differ", g->m, g->n, u->m, u->n);
    if (d->n != g->m)
        return hc_set_error(HC_ERR_INVALID, "down has %zu columns, gate/up produce %zu", d->n, g->m);
    if (d->m > g->n) return hc_set_error(HC_ERR_INVALID, "down rows %zu exceed the FFN input width %zu", d->m, g->n);
    if (g->device != d->device || u->device != d->device)
        return hc_set_error(HC_ERR_INVALID, "FFN weights live on different devices");
    return HC_OK;
}

// h[v][d_ff] = silu(gate xn[v]) * (up xn[v]), xn = rms_norm(x) when norm_w is given
// (over the first norm_len entries of each row) else x.
int hc_launch_gateup(hc_engine* e, const hc_weights* g, const hc_weights* u, const float* x, size_t ldx, float* h,
                     size_t nvec, const float* norm_w, size_t norm_len, float eps) {
    if (((uintptr_t)x & 15) || (ldx & 3))
        return hc_set_error(HC_ERR_INVALID, "x must be 16-byte aligned with ldx a multiple of 4");
    if (norm_w && (norm_len == 0 || norm_len > g->n))
        return hc_set_error(HC_ERR_INVALID, "norm length %zu must be in [1, %zu]", norm_len, g->n);
    if (e->use_tc && g->type == u->type && g->stride == u->stride &&
        tc_gemm_supported(g->type, (int)g->m, (int)g->n, (int)nvec)) {
        void* ws;
        int rc = hc_tc_prepare(e, g->type, g->m, g->n, nvec, 2, &ws);
        if (rc) return rc;
        cudaError_t ce = launch_tc_gemm(g->type, (const uint8_t*)g->dev, (const uint8_t*)u->dev, (long long)g->stride,
                                        (int)g->m, (int)g->n, x, (int)ldx, (int)nvec, h, (int)g->m, nullptr, 0, norm_w,
                                        (int)norm_len, eps, ws, e->d_err, e->num_sms, e->smem_optin, e->stream);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "gate/up tensor-core launch");
        return HC_OK;
    }
    if (g->type == u->type && gemv_mma_supported(g->type)) {
        GemvArgs a{};
        a.w = (const uint8_t*)g->dev;
        a.w2 = (const uint8_t*)u->dev;
        a.row_stride = (long long)g->stride;
        a.M = (int)g->m;
        a.K = (int)g->n;
        a.x = x;
        a.ldx = (int)ldx;
        a.y = h;
        a.ldy = (int)g->m;
        a.resid = nullptr;
        a.err = e->d_err;
        a.norm_w = norm_w;
        a.norm_len = (int)norm_len;
        a.norm_eps = eps;
        int rc = hc_sk_prepare(e, g->type, g->m, g->n, true, &a.sk_ws, &a.sk_cnt);
        if (rc) return rc;
        cudaError_t ce = launch_gemv_mma(g->type, a, (int)nvec, true, e->num_sms, e->smem_optin, e->stream);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "gate/up launch");
        return HC_OK;
    }
    // unfused: (norm) -> gate GEMV, up GEMV -> SwiGLU
    const size_t ff = g->m, K = g->n;
    int rc = e->ws_g.ensure(nvec * ff * 4);
    if (!rc) rc = e->ws_u.ensure(nvec * ff * 4);
    if (rc) return rc;
    const float* xin = x;
    size_t ldin = ldx;
    if (norm_w) {
        rc = e->ws_misc.ensure(nvec * K * 4);
        if (rc) return rc;
        cudaError_t ce = launch_rms_norm(x, (int)ldx, norm_w, (int)norm_len, (int)K, eps, (float*)e->ws_misc.p,
                                         (int)K, (int)nvec, e->stream);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "rms_norm launch");
        xin = (const float*)e->ws_misc.p;
        ldin = K;
    }
    rc = hc_launch_gemv(e, g, xin, ldin, (float*)e->ws_g.p, ff, nullptr, 0, nvec);
    if (!rc) rc = hc_launch_gemv(e, u, xin, ldin, (float*)e->ws_u.p, ff, nullptr, 0, nvec);
    if (rc) return rc;
    cudaError_t ce = launch_swiglu((const float*)e->ws_g.p, (const float*)e->ws_u.p, h, nvec * ff, e->stream);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "swiglu launch");
    return HC_OK;
}

int hc_launch_ffn(hc_engine* e, const hc_weights* g, const hc_weights* u, const hc_weights* d, const float* x,
                  size_t ldx, float* y, size_t ldy, const float* resid, size_t ldr, float* h_ws, size_t nvec,
                  const float* norm_w, size_t norm_len, float eps) {
    int rc = check_ffn(g, u, d);
    if (rc) return rc;
    if (!h_ws) {
        rc = e->ws_h.ensure(nvec * g->m * 4);
        if (rc) return rc;
        h_ws = (float*)e->ws_h.p;
    }
    rc = hc_launch_gateup(e, g, u, x, ldx, h_ws, nvec, norm_w, norm_len, eps);
    if (rc) return rc;
    return hc_launch_gemv(e, d, h_ws, g->m, y, ldy, resid, ldr, nvec);
}

extern "C" int hc_ffn_swiglu_dev(hc_engine* e, const hc_weights* g, const hc_weights* u, const hc_weights* d,
                                 const float* x, float* y, const float* resid, float* h_ws, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    rc = check_ffn(g, u, d);
    if (rc) return rc;
    if (!x || !y) return hc_set_error(HC_ERR_INVALID, "null argument");
    return hc_launch_ffn(e, g, u, d, x, g->n, y, d->m, resid, d->m, h_ws, nvec, nullptr, 0, 0.f);
}

extern "C" int hc_ffn_gateup_dev(hc_engine* e, const hc_weights* g, const hc_weights* u, const float* x, float* h,
                                 size_t nvec, const float* norm_w, size_t norm_len, float eps) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!g || !u || !x || !h) return hc_set_error(HC_ERR_INVALID, "null argument");
    if (g->m != u->m || g->n != u->n)
        return hc_set_error(HC_ERR_INVALID, "gate %zux%zu and up %zux%zu shapes differ", g->m, g->n, u->m, u->n);
    if (nvec == 0) return HC_OK;
    return hc_launch_gateup(e, g, u, x, g->n, h, nvec, norm_w, norm_len, eps);
}

extern "C" int hc_ffn_swiglu(hc_engine* e, const hc_weights* g, const hc_weights* u, const hc_weights* d,
                             const float* x, float* y, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    rc = check_ffn(g, u, d);
    if (rc) return rc;
    if (!x || !y) return hc_set_error(HC_ERR_INVALID, "null argument");
    if (nvec == 0) return HC_OK;
    rc = e->ws_x.ensure(nvec * g->n * 4);
    if (!rc) rc = e->ws_y.ensure(nvec * d->m * 4);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(e->ws_x.p, x, nvec * g->n * 4, cudaMemcpyHostToDevice, e->stream));
    rc = hc_launch_ffn(e, g, u, d, (const float*)e->ws_x.p, g->n, (float*)e->ws_y.p, d->m, nullptr, 0, nullptr,
                       nvec, nullptr, 0, 0.f);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(y, e->ws_y.p, nvec * d->m * 4, cudaMemcpyDeviceToHost, e->stream));
    return hc_finish_sync(e);
}

// ------------------------------------------------------------------ FFN stack (+ CUDA graph)
static uint64_t mix(uint64_t h, uint64_t v) {
    h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    return h;
}

struct StackArgs {
    const hc_weights* const* g;
    const hc_weights* const* u;
    const hc_weights* const* d;
    const float* const* norm;  // per-layer RMSNorm weights (device) or nullptr
    size_t L;
    float eps;
};

static int stack_enqueue(hc_engine* e, const StackArgs& s, float* x, size_t nvec, float* h) {
    const size_t k_in = s.g[0]->n, dm = s.d[0]->m;
    for (size_t l = 0; l < s.L; ++l) {
        // in place: each element of x is read (residual) and written by the same thread
        int rc = hc_launch_ffn(e, s.g[l], s.u[l], s.d[l], x, k_in, x, k_in, x, k_in, h, nvec,
                               s.norm ? s.norm[l] : nullptr, dm, s.eps);
        if (rc) return rc;
    }
    return HC_OK;
}

static int stack_check(const StackArgs& s) {
    if (!s.g || !s.u || !s.d || s.L == 0) return hc_set_error(HC_ERR_INVALID, "empty FFN stack");
    for (size_t l = 0; l < s.L; ++l) {
        int rc = check_ffn(s.g[l], s.u[l], s.d[l]);
        if (rc) return rc;
        if (s.g[l]->n != s.g[0]->n || s.d[l]->m != s.d[0]->m)
            return hc_set_error(HC_ERR_INVALID, "layer %zu changes the model width", l);
        if (s.norm && !s.norm[l]) return hc_set_error(HC_ERR_INVALID, "layer %zu has no norm weight", l);
    }
    return HC_OK;
}

// Device table of per-layer {gate, up, down, norm} pointers, cached per stack.
static int stack_table(hc_engine* e, const StackArgs& s, const void** out) {
    uint64_t key = 0x5354434Bull;  // "STCK"
    for (size_t l = 0; l < s.L; ++l) {
        key = mix(key, (uint64_t)(uintptr_t)s.g[l]->dev);
        key = mix(key, (uint64_t)(uintptr_t)s.u[l]->dev);
        key = mix(key, (uint64_t)(uintptr_t)s.d[l]->dev);
        key = mix(key, (uint64_t)(uintptr_t)(s.norm ? s.norm[l] : nullptr));
    }
    key = mix(key, s.L);
    auto it = e->ptr_tables.find(key);
    if (it == e->ptr_tables.end()) {
        std::vector<const void*> host(4 * s.L);
        for (size_t l = 0; l < s.L; ++l) {
            host[4 * l + 0] = s.g[l]->dev;
            host[4 * l + 1] = s.u[l]->dev;
            host[4 * l + 2] = s.d[l]->dev;
            host[4 * l + 3] = s.norm ? (const void*)s.norm[l] : nullptr;
        }
        void* d = nullptr;
        HC_CUDA(cudaMalloc(&d, host.size() * sizeof(void*)));
        cudaError_t ce = cudaMemcpy(d, host.data(), host.size() * sizeof(void*), cudaMemcpyHostToDevice);
        if (ce != cudaSuccess) {
            cudaFree(d);
            return hc_cuda_error(ce, "stack table upload");
        }
        it = e->ptr_tables.emplace(key, d).first;
    }
    *out = it->second;
    return HC_OK;
}

// Batch 1 with uniform layers: the whole stack as one persistent kernel (ffn_stack.cu).
// *done = false leaves the stack to the per-layer kernels.
static int stack_try_kernel(hc_engine* e, const StackArgs& s, float* x, size_t nvec, bool* done, bool tp = false) {
    *done = false;
    if ((!e->use_stack_kernel && !tp) || nvec != 1) return HC_OK;
    const hc_weights *g0 = s.g[0], *d0 = s.d[0];
    const int ta = g0->type, td = d0->type;
    if (!tiled_type(ta) || !tiled_type(td)) return HC_OK;
    const size_t dm = d0->m, ff = g0->m;
    // gate/up inputs: d_model, or d_model zero-padded to whole super-blocks (SmolLM's 576 ->
    // 768 for Q4_K); the kernel's prologue pads the fragment table to whole blocks with zeros
    // and touches only the first d_model entries of x
    if (g0->n != dm && !(ta != T_Q8_0 && g0->n == (dm + 255) / 256 * 256)) return HC_OK;
    for (size_t l = 0; l < s.L; ++l)
        if (s.g[l]->type != ta || s.u[l]->type != ta || s.d[l]->type != td || s.g[l]->m != ff || s.d[l]->n != ff)
            return HC_OK;
    StackLaunch L{};
    L.L = (int)s.L;
    L.dm = (int)dm;
    L.ff = (int)ff;
    L.ts_a = (long long)g0->stride;
    L.ts_b = (long long)d0->stride;
    L.x = x;
    L.eps = s.eps;
    L.err = e->d_err;
    if (tp) {
        L.tp_rank = e->peer.rank;
        L.tp_size = e->peer.world;
        L.tp_regions = e->peer.d_peer;
        L.tp_base = e->peer.tp_phases;
        L.tp_flow_base = e->peer.flow_phases;
    }
    int flow_used = 0;
    L.flow_used = &flow_used;
    size_t bytes = 0;
    cudaError_t ce = launch_ffn_stack(ta, td, L, e->num_sms, e->smem_optin, e->stream, true, &bytes);
    if (ce == cudaErrorInvalidConfiguration) {
        cudaGetLastError();
        return HC_OK;
    }
    if (ce != cudaSuccess) return hc_cuda_error(ce, "stack kernel setup");
    int rc = e->stack_bar.ensure(bytes);
    if (!rc) rc = stack_table(e, s, &L.layers);
    if (rc) return rc;
    L.scratch = e->stack_bar.p;
    ce = launch_ffn_stack(ta, td, L, e->num_sms, e->smem_optin, e->stream, false, nullptr);
    if (ce != cudaSuccess) return hc_cuda_error(ce, "stack kernel launch");
    if (tp && flow_used) e->peer.flow_phases += (uint32_t)s.L;  // its per-tile counters advanced
    *done = true;
    return HC_OK;
}

// Size every workspace the per-layer kernels of a stack use for nvec rows, before a capture
// (no allocation may happen inside one).
static int stack_prepare(hc_engine* e, const StackArgs& s, size_t nvec) {
    for (size_t l = 0; l < s.L; ++l) {
        float* ws;
        int* cnt;
        int rc;
        if (s.g[l]->type == s.u[l]->type && gemv_mma_supported(s.g[l]->type)) {
            rc = hc_sk_prepare(e, s.g[l]->type, s.g[l]->m, s.g[l]->n, true, &ws, &cnt);
        } else {
            rc = e->ws_g.ensure(nvec * s.g[l]->m * 4);
            if (!rc) rc = e->ws_u.ensure(nvec * s.g[l]->m * 4);
            if (!rc && s.norm) rc = e->ws_misc.ensure(nvec * s.g[l]->n * 4);
            if (!rc && gemv_mma_supported(s.g[l]->type))
                rc = hc_sk_prepare(e, s.g[l]->type, s.g[l]->m, s.g[l]->n, false, &ws, &cnt);
            if (!rc && gemv_mma_supported(s.u[l]->type))
                rc = hc_sk_prepare(e, s.u[l]->type, s.u[l]->m, s.u[l]->n, false, &ws, &cnt);
        }
        if (!rc && gemv_mma_supported(s.d[l]->type))
            rc = hc_sk_prepare(e, s.d[l]->type, s.d[l]->m, s.d[l]->n, false, &ws, &cnt);
        void* tws;
        if (!rc && e->use_tc && tc_gemm_supported(s.g[l]->type, (int)s.g[l]->m, (int)s.g[l]->n, (int)nvec))
            rc = hc_tc_prepare(e, s.g[l]->type, s.g[l]->m, s.g[l]->n, nvec, 2, &tws);
        if (!rc && e->use_tc && tc_gemm_supported(s.d[l]->type, (int)s.d[l]->m, (int)s.d[l]->n, (int)nvec))
            rc = hc_tc_prepare(e, s.d[l]->type, s.d[l]->m, s.d[l]->n, nvec, 1, &tws);
        if (rc) return rc;
    }
    return HC_OK;
}

// Key of a captured stack: every address and shape the graph bakes in.
static uint64_t stack_key(const hc_engine* e, const StackArgs& s, const float* x, size_t nvec, const float* h) {
    uint64_t key = mix(mix(mix(0, (uint64_t)(uintptr_t)x), nvec), s.L);
    key = mix(key, (uint64_t)(uintptr_t)h);
    key = mix(key, (uint64_t)(uintptr_t)e->ws_g.p);
    key = mix(key, (uint64_t)(uintptr_t)e->ws_u.p);
    key = mix(key, (uint64_t)(uintptr_t)e->ws_misc.p);
    uint32_t eb;
    memcpy(&eb, &s.eps, 4);
    key = mix(key, eb);
    for (size_t l = 0; l < s.L; ++l) {
        key = mix(key, (uint64_t)(uintptr_t)s.g[l]->dev);
        key = mix(key, (uint64_t)(uintptr_t)s.u[l]->dev);
        key = mix(key, (uint64_t)(uintptr_t)s.d[l]->dev);
        key = mix(key, (uint64_t)(uintptr_t)(s.norm ? s.norm[l] : nullptr));
        key = mix(key, ((uint64_t)s.g[l]->type << 32) ^ s.g[l]->m ^ (s.g[l]->n << 20) ^ ((uint64_t)s.d[l]->type << 40));
    }
    return key;
}

// Launch the graph cached under `key`, capturing enqueue() into it first if there is none.
template <class F>
static int graph_run(hc_engine* e, uint64_t key, F enqueue) {
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        // capture on the engine's private stream (the caller's may be the legacy default
        // stream, which cannot be captured); the graph is then launched on the caller's
        cudaGraph_t graph;
        cudaStream_t caller = e->stream;
        e->stream = e->own_stream;
        cudaError_t ce = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeRelaxed);
        if (ce != cudaSuccess) {
            e->stream = caller;
            return hc_cuda_error(ce, "stack capture begin");
        }
        int rc = enqueue();
        ce = cudaStreamEndCapture(e->stream, &graph);
        e->stream = caller;
        if (rc) {
            if (ce == cudaSuccess) cudaGraphDestroy(graph);
            return rc;
        }
        if (ce != cudaSuccess) return hc_cuda_error(ce, "stack capture");
        cudaGraphExec_t exec;
        ce = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "stack graph instantiate");
        it = e->graphs.emplace(key, exec).first;
    }
    HC_CUDA(cudaGraphLaunch(it->second, e->stream));
    return HC_OK;
}

// h workspace for nvec rows of the widest layer; moving it drops the captured graphs.
static int stack_h(hc_engine* e, const StackArgs& s, size_t nvec, float** h) {
    size_t ffmax = 0;
    for (size_t l = 0; l < s.L; ++l) ffmax = s.g[l]->m > ffmax ? s.g[l]->m : ffmax;
    void* old_h = e->ws_h.p;
    int rc = e->ws_h.ensure(nvec * ffmax * 4);
    if (rc) return rc;
    if (old_h && old_h != e->ws_h.p) hc_drop_graphs(e);
    *h = (float*)e->ws_h.p;
    return HC_OK;
}

static int stack_run(hc_engine* e, const StackArgs& s, float* x, size_t nvec) {
    float* h;
    int rc = stack_h(e, s, nvec, &h);
    if (rc) return rc;
    bool done = false;
    rc = stack_try_kernel(e, s, x, nvec, &done);
    if (rc || done) return rc;
    rc = stack_prepare(e, s, nvec);
    if (rc) return rc;
    if (!e->use_graphs) return stack_enqueue(e, s, x, nvec, h);
    return graph_run(e, stack_key(e, s, x, nvec, h), [&] { return stack_enqueue(e, s, x, nvec, h); });
}

// Tensor-parallel stack at batch > 1, per layer: the fused gate/up of this rank's d_ff shard
// (RMSNorm of the replicated x in its prologue), the down GEMV of the shard into a partial of
// every output row, and the all-reduce of the partials into x over the exchange regions
// (tp_reduce.cu).  x is replicated and stays bit-identical on every rank.
static int stack_tp_enqueue(hc_engine* e, const StackArgs& s, float* x, size_t nvec, float* h, float* yp) {
    const size_t dm = s.d[0]->m;
    for (size_t l = 0; l < s.L; ++l) {
        int rc = hc_launch_gateup(e, s.g[l], s.u[l], x, dm, h, nvec, s.norm ? s.norm[l] : nullptr, dm, s.eps);
        if (!rc) rc = hc_launch_gemv(e, s.d[l], h, s.g[l]->m, yp, dm, nullptr, 0, nvec);
        if (rc) return rc;
        cudaError_t ce = launch_tp_allreduce(yp, x, nvec * dm, e->peer.d_peer, e->peer.rank, e->peer.world, e->d_err,
                                             e->stream);
        if (ce != cudaSuccess) return hc_cuda_error(ce, "tensor-parallel all-reduce");
    }
    return HC_OK;
}

static int stack_tp_batched(hc_engine* e, const StackArgs& s, float* x, size_t nvec) {
    const size_t dm = s.d[0]->m;
    const PeerState& pe = e->peer;
    const size_t need = tp_exchange_bytes(pe.world, nvec * dm);
    if (pe.bytes < need)
        return hc_set_error(HC_ERR_INVALID,
                            "tensor-parallel exchange of %zu rows x %zu needs a peer region of %zu bytes (have %zu)",
                            nvec, dm, need, pe.bytes);
    if (dm % 4 || ((uintptr_t)x) % 16)
        return hc_set_error(HC_ERR_INVALID, "tensor-parallel exchange: x must be 16-byte aligned, d_model %% 4 == 0");
    float* h;
    int rc = stack_h(e, s, nvec, &h);
    if (rc) return rc;
    void* old_y = e->ws_tp.p;
    rc = e->ws_tp.ensure(nvec * dm * 4);
    if (rc) return rc;
    if (old_y && old_y != e->ws_tp.p) hc_drop_graphs(e);
    float* yp = (float*)e->ws_tp.p;
    rc = stack_prepare(e, s, nvec);
    if (rc) return rc;
    if (!e->use_graphs) return stack_tp_enqueue(e, s, x, nvec, h, yp);
    uint64_t key = mix(stack_key(e, s, x, nvec, h), 0x54504231ull);  // "TPB1"
    key = mix(mix(key, (uint64_t)(uintptr_t)yp), (uint64_t)(uintptr_t)pe.d_peer);
    return graph_run(e, key, [&] { return stack_tp_enqueue(e, s, x, nvec, h, yp); });
}

extern "C" int hc_ffn_stack_dev(hc_engine* e, const hc_weights* const* g, const hc_weights* const* u,
                                const hc_weights* const* d, const float* const* norm_w, float eps, size_t L, float* x,
                                size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    StackArgs s{g, u, d, norm_w, L, eps};
    rc = stack_check(s);
    if (rc) return rc;
    if (!x) return hc_set_error(HC_ERR_INVALID, "null x");
    if (nvec == 0) return HC_OK;
    return stack_run(e, s, x, nvec);
}

// Tensor-parallel stack: the layers are this rank's d_ff shard (gate/up rows and down
// columns of the same range); x [nvec][d_model] is replicated and ends identical on every
// rank.  Batch 1: the persistent stack kernel with the exchange inside; otherwise per-layer
// kernels and the in-kernel all-reduce of tp_reduce.cu, captured as one graph.
extern "C" int hc_ffn_stack_tp_dev(hc_engine* e, const hc_weights* const* g, const hc_weights* const* u,
                                   const hc_weights* const* d, const float* const* norm_w, float eps, size_t L,
                                   float* x, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    StackArgs s{g, u, d, norm_w, L, eps};
    rc = stack_check(s);
    if (rc) return rc;
    if (!x) return hc_set_error(HC_ERR_INVALID, "null x");
    if (!e->peer.connected) return hc_set_error(HC_ERR_INVALID, "tensor-parallel stack without a connected peer group");
    if (g[0]->n != d[0]->m)
        return hc_set_error(HC_ERR_UNSUPPORTED, "tensor-parallel stack: padded model width (%zu inputs, %zu outputs)",
                            g[0]->n, d[0]->m);
    if (nvec == 0) return HC_OK;
    if (nvec > 1) return stack_tp_batched(e, s, x, nvec);
    bool done = false;
    rc = stack_try_kernel(e, s, x, 1, &done, true);
    if (rc) return rc;
    if (!done)
        return hc_set_error(HC_ERR_UNSUPPORTED,
                            "tensor-parallel stack: formats or shard shape not covered by the persistent kernel");
    e->peer.tp_phases += (uint32_t)L;
    return HC_OK;
}

extern "C" int hc_ffn_stack_tp(hc_engine* e, const hc_weights* const* g, const hc_weights* const* u,
                               const hc_weights* const* d, const float* const* norm_w, float eps, size_t L,
                               const float* x_in, float* x_out, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    if (!g || !g[0] || !x_in || !x_out) return hc_set_error(HC_ERR_INVALID, "null argument");
    const size_t bytes = nvec * g[0]->n * 4;
    if (bytes == 0) return HC_OK;
    rc = e->ws_x.ensure(bytes);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(e->ws_x.p, x_in, bytes, cudaMemcpyHostToDevice, e->stream));
    rc = hc_ffn_stack_tp_dev(e, g, u, d, norm_w, eps, L, (float*)e->ws_x.p, nvec);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(x_out, e->ws_x.p, bytes, cudaMemcpyDeviceToHost, e->stream));
    return hc_finish_sync(e);
}

extern "C" int hc_ffn_stack(hc_engine* e, const hc_weights* const* g, const hc_weights* const* u,
                            const hc_weights* const* d, const float* const* norm_w, float eps, size_t L,
                            const float* x_in, float* x_out, size_t nvec) {
    int rc = hc_engine_activate(e);
    if (rc) return rc;
    StackArgs s{g, u, d, norm_w, L, eps};
    rc = stack_check(s);
    if (rc) return rc;
    if (!x_in || !x_out) return hc_set_error(HC_ERR_INVALID, "null argument");
    if (nvec == 0) return HC_OK;
    const size_t bytes = nvec * g[0]->n * 4;
    rc = e->ws_x.ensure(bytes);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(e->ws_x.p, x_in, bytes, cudaMemcpyHostToDevice, e->stream));
    rc = stack_run(e, s, (float*)e->ws_x.p, nvec);
    if (rc) return rc;
    HC_CUDA(cudaMemcpyAsync(x_out, e->ws_x.p, bytes, cudaMemcpyDeviceToHost, e->stream));
    return hc_finish_sync(e);
}
