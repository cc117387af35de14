/*
 * hayai_cuda.h -- C ABI of the B200 (sm_100a) quantized-FFN backend.
 *
 * This is the drop-in boundary for Hayai's FFN hot path.  Every entry point is
 * extern "C", takes plain pointers and sizes, returns an int status (HC_OK = 0)
 * and never throws or aborts across the ABI; the message of the last failure on
 * the calling thread is available from hc_last_error().
 *
 * Each declaration cites the reference interface it replaces (paths relative to
 * the aitups/hayai repository root).  The reference backend is
 * hayai-opencl's OpenClEngine (crates/hayai-opencl/src/compute.rs,
 * async_gemv.rs), dispatched from hayai-core's EngineOrchestrator
 * (crates/hayai-core/src/orchestrator.rs).
 *
 * Conventions
 *  - ggml_type uses GGUF's GgmlType ids (crates/hayai-model/src/gguf_types.rs:6-40):
 *    F32=0, F16=1, Q4_0=2, Q4_1=3, Q5_0=6, Q5_1=7, Q8_0=8, Q8_1=9, Q2_K=10, Q3_K=11, Q4_K=12,
 *    Q5_K=13, Q6_K=14, Q8_K=15, IQ2_XXS=16, IQ2_XS=17, IQ3_XXS=18, IQ4_NL=20, IQ3_S=21, IQ2_S=22,
 *    IQ4_XS=23, BF16=30 (the formats of gemv_row_bytes, compute.rs:877-907).
 *    Q4_K, Q6_K and Q8_0 run on the tensor-core kernels (tile-major upload); the others on
 *    CUDA-core kernels over the raw GGUF rows.  Any other id is HC_ERR_UNSUPPORTED.
 *  - A weight matrix is GGUF-layout: nrows = m rows of ncols = n columns, each row
 *    n/QK consecutive blocks (crates/hayai-model/src/quant.rs:28-37); y[m] = W x[n].
 *  - "host" pointers are ordinary CPU memory, borrowed for the call only (or until
 *    hc_pending_wait for the async call).  "_dev" entry points take device pointers
 *    of the engine's GPU, enqueue on the engine's stream and return without waiting.
 *  - An engine is externally synchronised (the reference keeps its orchestrator
 *    behind a Mutex, orchestrator.rs:65-68); engines on different GPUs are independent.
 */
#ifndef HAYAI_CUDA_H
#define HAYAI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define HC_OK 0
#define HC_ERR_INVALID 1     /* bad shape / size / argument (compute.rs:912-951 validation) */
#define HC_ERR_UNSUPPORTED 2 /* no kernel for this ggml type (orchestrator.rs:403-409 hard fail) */
#define HC_ERR_CUDA 3        /* CUDA runtime error */
#define HC_ERR_RANGE 4       /* an activation is outside the f16 range used by the tensor-core split */
#define HC_ERR_NCCL 5        /* collective failed */
#define HC_ERR_TIMEOUT 6     /* a bounded device wait expired */

typedef struct hc_engine hc_engine;   /* one GPU + stream: OpenClEngine (crates/hayai-opencl/src/context.rs:23) */
typedef struct hc_weights hc_weights; /* a resident weight matrix (one-time upload) */
typedef struct hc_pending hc_pending; /* in-flight GEMV: PendingGemv (crates/hayai-opencl/src/async_gemv.rs:15-57) */

/* Message of the last failure on this thread ("" if none).  Replaces
 * OpenClError::ClError(String) (crates/hayai-opencl/src/context.rs:14). */
const char* hc_last_error(void);

/* Number of CUDA devices.  Replaces discover_opencl_devices (crates/hayai-opencl/src/device.rs). */
int hc_device_count(int* out);

/* Create / destroy an engine on `device`.  Replaces OpenClEngine::init_device
 * (crates/hayai-opencl/src/context.rs:106). */
int hc_engine_init(int device, hc_engine** out);
int hc_engine_free(hc_engine* eng);

/* Enqueue on the caller's CUDA stream (cudaStream_t as void*; NULL = the legacy default
 * stream), or go back to the engine's own non-blocking stream. */
int hc_engine_set_stream(hc_engine* eng, void* stream);
int hc_engine_use_own_stream(hc_engine* eng);
int hc_engine_get_stream(hc_engine* eng, void** stream);

/* Wait for all work on the engine stream and report any device-side error. */
int hc_sync(hc_engine* eng);

/* Packed bytes per row for n columns; HC_ERR_INVALID if n is not a multiple of the
 * block.  Replaces gemv_row_bytes (crates/hayai-opencl/src/compute.rs:877-907). */
int hc_gemv_row_bytes(int ggml_type, size_t n, size_t* out);

/* ---- resident weights --------------------------------------------------------
 * One-time upload of an m x n GGUF-layout matrix into HBM, rewritten into the GPU
 * layout of its format.  Replaces the device mirror / resident preload
 * (allocate_resident_for_pool, crates/hayai-opencl/src/hetero_scratch.rs:243) and
 * the ping-pong streaming it fed.  Validation as validate_gemv_weights
 * (compute.rs:912-933). */
int hc_weights_upload(hc_engine* eng, int ggml_type, size_t m, size_t n, const void* host_bytes, size_t len,
                      hc_weights** out);
/* Same, from GGUF-layout bytes already on the engine's GPU (GgmlWeightBind::Device,
 * compute.rs:21-27). */
int hc_weights_from_device(hc_engine* eng, int ggml_type, size_t m, size_t n, const void* dev_bytes, size_t len,
                           hc_weights** out);
int hc_weights_free(hc_weights* w);
/* ggml_type, m, n and resident bytes of a weights object. */
int hc_weights_info(const hc_weights* w, int* ggml_type, size_t* m, size_t* n, size_t* bytes);

/* ---- GEMV ---------------------------------------------------------------------- */
/* y[m] = W x[n] with host weights, host input/output; blocking.  Replaces
 * OpenClEngine::ggml_gemv_dispatch (compute.rs:281-385) and the per-type wrappers
 * ggml_gemv_q4_k / q6_k / q8_0 (compute.rs:153-276). */
int hc_ggml_gemv_dispatch(hc_engine* eng, int ggml_type, size_t m, size_t n, const uint8_t* weights,
                          size_t weights_len, const float* input, float* output);

/* Resident weights, host input/output; blocking.  Replaces ggml_gemv_dispatch_bound
 * (compute.rs:388-461) and EngineOrchestrator::execute_quant_gemv (orchestrator.rs:222-234). */
int hc_ggml_gemv_bound(hc_engine* eng, const hc_weights* w, const float* input, float* output);

/* `batch` input rows [batch][n] -> outputs [batch][m]; blocking.  Replaces
 * ggml_gemv_batched_q4_k (compute.rs:179-257) and execute_quant_gemv_batched
 * (orchestrator.rs:240-269) for every type. */
int hc_ggml_gemv_batched(hc_engine* eng, const hc_weights* w, const float* inputs, float* outputs, size_t batch);

/* Asynchronous GEMV: ggml_gemv_async / ggml_gemv_async_from_device
 * (async_gemv.rs:90-130).  hc_pending_wait copies the m outputs into `output`
 * (PendingGemv::wait, async_gemv.rs:27); hc_pending_free waits first, as
 * PendingGemv::drop does (async_gemv.rs:48-57). */
int hc_ggml_gemv_async(hc_engine* eng, const hc_weights* w, const float* input, hc_pending** out);
int hc_pending_wait(hc_pending* p, float* output, size_t m);
int hc_pending_free(hc_pending* p);

/* Device pointers: y[v][ldy] = resid[v][ldr] (if non-NULL) + W x[v][ldx] for v < nvec,
 * enqueued on the engine stream.  x must be 16-byte aligned with ldx % 4 == 0. */
int hc_gemv_dev(hc_engine* eng, const hc_weights* w, const float* x, size_t ldx, float* y, size_t ldy,
                const float* resid, size_t ldr, size_t nvec);

/* hc_gemv_dev for Q4_K, Q6_K and Q8_0 weights that allocates nothing.  No counterpart in
 * the reference: it exists for callers that cannot let a library call cudaMalloc -- hosts
 * whose device memory belongs to their own pool allocator, and decode loops that cannot
 * absorb the device synchronisation a cudaMalloc/cudaFree may cause.  The scratch the
 * stream-K split needs comes from a static device array of the library (4 MiB of partial
 * sums + 16384 tile counters per GPU, held until exit); a matrix that needs more is
 * rejected with HC_ERR_INVALID (every Llama-3 8B/70B FFN matrix and a 128256 x 4096 output
 * projection fit; M above 262144 never does).  Every call looks the array's address up
 * on the current device (cudaGetSymbolAddress, which allocates nothing); on the first call
 * on a device that lookup also loads the library's device code there, so make that first
 * call before any stream capture.  All calls on a device share the array, so calls that overlap
 * on the GPU race: serialise them.  Other formats return HC_ERR_UNSUPPORTED. */
int hc_gemv_dev_noalloc(hc_engine* eng, const hc_weights* w, const float* x, size_t ldx, float* y, size_t ldy,
                        const float* resid, size_t ldr, size_t nvec);

/* Toy 16-entry LUT-Q4 matmul (two nibbles per byte, low nibble first); blocking.
 * Replaces OpenClEngine::lut_matmul_q4 (compute.rs:45-128) and
 * EngineOrchestrator::execute_lut_matmul (orchestrator.rs:198-218). */
int hc_lut_matmul_q4(hc_engine* eng, size_t m, size_t n, const uint8_t* weights_q4, const float* lut16,
                     const float* input, float* output);
int hc_lut_matmul_q4_dev(hc_engine* eng, size_t m, size_t n, const uint8_t* weights_q4, const float* lut16,
                         const float* input, float* output);

/* ---- SwiGLU FFN block -------------------------------------------------------------
 * y = W_down (silu(W_gate x) * (W_up x)), the block of run_ffn_block
 * (crates/hayai-core/src/stream_infer.rs:574-606) with the host SiLU*up combine
 * (:3836-3840) fused on the device.  gate/up are d_ff x k_in, down is n_out x d_ff.
 * Host version: blocking, no residual. */
int hc_ffn_swiglu(hc_engine* eng, const hc_weights* gate, const hc_weights* up, const hc_weights* down,
                  const float* x, float* y, size_t nvec);
/* Device version: y[v] = resid[v] (optional) + FFN(x[v]); h_ws is a device scratch of
 * nvec * d_ff floats (NULL = engine workspace).  x/y rows are k_in / n_out floats. */
int hc_ffn_swiglu_dev(hc_engine* eng, const hc_weights* gate, const hc_weights* up, const hc_weights* down,
                      const float* x, float* y, const float* resid, float* h_ws, size_t nvec);

/* The fused first half of the block alone: h[v] = silu(W_gate xn[v]) * (W_up xn[v]), one
 * kernel reading both matrices (ffn_begin_gate_up_scratch + the SiLU*up combine,
 * stream_infer.rs:3752-3840).  xn = rms_norm(x, norm_w, eps) over the first norm_len
 * entries of each row (crates/hayai-cpu/src/attention.rs:142-147) when norm_w (device,
 * norm_len floats) is non-NULL, else x.  h is [nvec][d_ff]. */
int hc_ffn_gateup_dev(hc_engine* eng, const hc_weights* gate, const hc_weights* up, const float* x, float* h,
                      size_t nvec, const float* norm_w, size_t norm_len, float eps);

/* Stack of n_layers FFN sublayers with pre-norm and residual, as in a decode step
 * (stream_infer.rs:2166-2170 rms_norm(x, ffn_norm) then :3752-3864):
 *     x <- x + FFN_l(rms_norm(x, norm_w[l], eps))        for l = 0..n_layers-1
 * norm_w is an array of n_layers device pointers (n_out floats each), or NULL for no
 * normalization.  x is [nvec][k_in] with k_in >= n_out (rows zero-padded for K-quant
 * block alignment; norm and residual cover the first n_out entries).  _dev works in place
 * on device memory (captured once into a CUDA graph and replayed); the host version
 * copies x in and the result out. */
int hc_ffn_stack_dev(hc_engine* eng, const hc_weights* const* gate, const hc_weights* const* up,
                     const hc_weights* const* down, const float* const* norm_w, float eps, size_t n_layers,
                     float* x, size_t nvec);
int hc_ffn_stack(hc_engine* eng, const hc_weights* const* gate, const hc_weights* const* up,
                 const hc_weights* const* down, const float* const* norm_w, float eps, size_t n_layers,
                 const float* x_in, float* x_out, size_t nvec);

/* ---- tensor / expert parallelism (one process per GPU) -----------------------------
 * No reference counterpart: the reference has no multi-GPU FFN.  A group of `world` ranks
 * (<= 8, one GPU each) shares exchange regions: hc_peer_open allocates this rank's region
 * (bytes >= 12 MiB; zeroed) and writes its CUDA IPC handle (hc_peer_handle_bytes bytes) to
 * handle_out; the caller gathers every rank's handle over its own process group, in rank
 * order, and passes them to hc_peer_connect; then all ranks must pass a host barrier before
 * the first parallel call.  Kernels store partial results into the peers' regions over
 * NVLink and signal each other with system-scope atomics (waits bounded by one second:
 * HC_ERR_TIMEOUT).  Parallel calls are collective: every rank makes the same calls in the
 * same order.  hc_peer_close (after a host barrier) unmaps and frees. */
int hc_peer_handle_bytes(size_t* out);
int hc_peer_open(hc_engine* eng, int rank, int world, size_t bytes, void* handle_out);
int hc_peer_connect(hc_engine* eng, const void* handles);
int hc_peer_close(hc_engine* eng);
/* This rank's exchange region (device address and size) for diagnostics: its layout holds
 * the exchange counters and epochs.  No reference counterpart. */
int hc_peer_region(hc_engine* eng, void** region, size_t* bytes);

/* Tensor-parallel FFN stack, the config-5 sharding of Llama-3-70B: rank p holds gate/up rows
 * and down columns [p*F/P, (p+1)*F/P) of every layer (F = d_ff, column shards whole
 * super-blocks).  x [nvec][d_model] is replicated; each layer's down output is all-reduced
 * over the ranks' exchange regions (stream_infer.rs:2166's residual add after the down GEMV,
 * with the sum over shards) and added in rank order, so x ends identical on every rank.
 * nvec = 1: inside the persistent stack kernel.  nvec > 1: per-layer kernels plus one
 * all-reduce kernel per layer, as one CUDA graph; the region must then hold
 * 8 MiB + 4 KiB + 8 * P * nvec * d_model bytes (hc_peer_open's `bytes`). */
int hc_ffn_stack_tp_dev(hc_engine* eng, const hc_weights* const* gate, const hc_weights* const* up,
                        const hc_weights* const* down, const float* const* norm_w, float eps, size_t n_layers,
                        float* x, size_t nvec);
int hc_ffn_stack_tp(hc_engine* eng, const hc_weights* const* gate, const hc_weights* const* up,
                    const hc_weights* const* down, const float* const* norm_w, float eps, size_t n_layers,
                    const float* x_in, float* x_out, size_t nvec);

/* ---- MoE ---------------------------------------------------------------------------
 * Routing of route_experts (crates/hayai-core/src/moe_infer.rs:868-935, with
 * top_k_indices :852-862 and MoeMeta exec_plan.rs:244-272), on the device, for
 * n_tok score rows [n_tok][n_expert].  ids are bit-exact with the reference for
 * identical scores; weights follow the reference's softmax/sigmoid in f32. */
int hc_route_experts_dev(hc_engine* eng, const float* scores, const float* bias, size_t n_tok, size_t n_expert,
                         size_t top_k, size_t n_group, size_t topk_group, int gating, int norm_topk_prob,
                         float routed_scaling_factor, int32_t* ids, float* weights);

/* Router GEMV with the reference's summation order (gemv_f32, quant.rs:358-369:
 * sequential sum += w*x, no FMA), so scores are bit-identical to the CPU path. */
int hc_router_scores_dev(hc_engine* eng, const float* router_w, size_t n_expert, size_t d_model, const float* x,
                         size_t n_tok, float* scores);

/* Expert-routed SwiGLU FFN for n_tok tokens (forward_moe's router -> top-k ->
 * per-expert FFN -> weighted sum, moe_infer.rs:221-264, :342-376, :449-455):
 * y[t] = sum_i w_i * FFN_{e_i}(x[t]) (no residual).  Experts are given as arrays of
 * n_expert weight handles.  ids_out/w_out (device, [n_tok][top_k], may be NULL)
 * receive the routing. */
int hc_moe_ffn_dev(hc_engine* eng, const float* router_w, size_t n_expert, size_t top_k, int norm_topk_prob,
                   float routed_scaling_factor, const hc_weights* const* gate, const hc_weights* const* up,
                   const hc_weights* const* down, const float* x, size_t n_tok, float* y, int32_t* ids_out,
                   float* w_out);

/* Expert-parallel MoE FFN (the Qwen3-30B-A3B sharding): this rank holds experts
 * [expert_lo, expert_lo + n_local) (gate/up/down arrays of n_local handles); router_w
 * covers all n_expert experts and x [n_tok][d_model] is replicated, so every rank routes
 * identically.  Each rank computes the (token, slot) pairs routed to its experts and stores
 * their down rows into every rank's exchange region over NVLink (the all-to-all of routed
 * outputs, fused into the expert GEMV's epilogue); after a cross-GPU signal every rank adds
 * the rows in top-k order (moe_infer.rs:449-455), so y is identical on all ranks and does
 * not depend on the rank count.  Needs a connected peer group; collective. */
int hc_moe_ffn_ep_dev(hc_engine* eng, const float* router_w, size_t n_expert, size_t top_k, int norm_topk_prob,
                      float routed_scaling_factor, const hc_weights* const* gate, const hc_weights* const* up,
                      const hc_weights* const* down, size_t expert_lo, size_t n_local, const float* x, size_t n_tok,
                      float* y, int32_t* ids_out, float* w_out);

/* A stack of MoE layers for n_tok tokens, x <- x + MoE_l(x) for l = 0..n_layers-1 (the
 * residual add of the callers of forward_moe, moe_infer.rs:222-223), in place on device
 * memory, captured once into a CUDA graph and replayed.  router_w: n_layers device pointers
 * ([n_expert][d_model] each); gate/up/down: n_layers x n_expert handles, layer-major.  The
 * _ep variant holds experts [expert_lo, expert_lo + n_local) of every layer (n_layers x
 * n_local handles) and exchanges the routed rows as hc_moe_ffn_ep_dev does; collective. */
int hc_moe_stack_dev(hc_engine* eng, size_t n_layers, const float* const* router_w, size_t n_expert, size_t top_k,
                     int norm_topk_prob, float routed_scaling_factor, const hc_weights* const* gate,
                     const hc_weights* const* up, const hc_weights* const* down, float* x, size_t n_tok);
int hc_moe_stack_ep_dev(hc_engine* eng, size_t n_layers, const float* const* router_w, size_t n_expert,
                        size_t top_k, int norm_topk_prob, float routed_scaling_factor, const hc_weights* const* gate,
                        const hc_weights* const* up, const hc_weights* const* down, size_t expert_lo, size_t n_local,
                        float* x, size_t n_tok);

/* ---- synthetic data ----------------------------------------------------------------
 * Seeded N(mean, std^2) floats on the device (splitmix64 at a position + Box-Muller in
 * double; the same stream as the test oracle's generator up to last-bit differences of
 * the device's double log/sin/cos). */
int hc_synth_normal_dev(hc_engine* eng, uint64_t seed, size_t n, float mean, float stdv, float* out);
/* Quantize n device floats into GGUF blocks on the device.  Q4_K restates the reference
 * quantizer bit-exactly (quantize_q4_k, crates/hayai-model/src/q4k.rs:85-160); Q6_K and
 * Q8_0 use this library's own quantizers (the reference has none). */
int hc_quantize_dev(hc_engine* eng, int ggml_type, const float* x, size_t n, uint8_t* out);

#ifdef __cplusplus
}
#endif

#endif /* HAYAI_CUDA_H */
