//! Raw declarations of every entry point of include/hayai_cuda.h (same order, same types).
#![allow(non_camel_case_types)]
use std::ffi::{c_char, c_int, c_void};

#[repr(C)]
pub struct hc_engine {
    _p: [u8; 0],
}
#[repr(C)]
pub struct hc_weights {
    _p: [u8; 0],
}
#[repr(C)]
pub struct hc_pending {
    _p: [u8; 0],
}

pub const HC_OK: c_int = 0;
pub const HC_ERR_INVALID: c_int = 1;
pub const HC_ERR_UNSUPPORTED: c_int = 2;
pub const HC_ERR_CUDA: c_int = 3;
pub const HC_ERR_RANGE: c_int = 4;
pub const HC_ERR_NCCL: c_int = 5;
pub const HC_ERR_TIMEOUT: c_int = 6;

#[link(name = "hayai_cuda")]
extern "C" {
    pub fn hc_last_error() -> *const c_char;
    pub fn hc_device_count(out: *mut c_int) -> c_int;
    pub fn hc_engine_init(device: c_int, out: *mut *mut hc_engine) -> c_int;
    pub fn hc_engine_free(eng: *mut hc_engine) -> c_int;
    pub fn hc_engine_set_stream(eng: *mut hc_engine, stream: *mut c_void) -> c_int;
    pub fn hc_engine_use_own_stream(eng: *mut hc_engine) -> c_int;
    pub fn hc_engine_get_stream(eng: *mut hc_engine, stream: *mut *mut c_void) -> c_int;
    pub fn hc_sync(eng: *mut hc_engine) -> c_int;
    pub fn hc_gemv_row_bytes(ggml_type: c_int, n: usize, out: *mut usize) -> c_int;
    pub fn hc_weights_upload(eng: *mut hc_engine, ggml_type: c_int, m: usize, n: usize, host_bytes: *const c_void,
                             len: usize, out: *mut *mut hc_weights) -> c_int;
    pub fn hc_weights_from_device(eng: *mut hc_engine, ggml_type: c_int, m: usize, n: usize, dev_bytes: *const c_void,
                                  len: usize, out: *mut *mut hc_weights) -> c_int;
    pub fn hc_weights_free(w: *mut hc_weights) -> c_int;
    pub fn hc_weights_info(w: *const hc_weights, ggml_type: *mut c_int, m: *mut usize, n: *mut usize,
                           bytes: *mut usize) -> c_int;
    pub fn hc_ggml_gemv_dispatch(eng: *mut hc_engine, ggml_type: c_int, m: usize, n: usize, weights: *const u8,
                                 len: usize, input: *const f32, output: *mut f32) -> c_int;
    pub fn hc_ggml_gemv_bound(eng: *mut hc_engine, w: *const hc_weights, input: *const f32, output: *mut f32) -> c_int;
    pub fn hc_ggml_gemv_batched(eng: *mut hc_engine, w: *const hc_weights, inputs: *const f32, outputs: *mut f32,
                                batch: usize) -> c_int;
    pub fn hc_ggml_gemv_async(eng: *mut hc_engine, w: *const hc_weights, input: *const f32,
                              out: *mut *mut hc_pending) -> c_int;
    pub fn hc_pending_wait(p: *mut hc_pending, output: *mut f32, m: usize) -> c_int;
    pub fn hc_pending_free(p: *mut hc_pending) -> c_int;
    pub fn hc_gemv_dev(eng: *mut hc_engine, w: *const hc_weights, x: *const f32, ldx: usize, y: *mut f32, ldy: usize,
                       resid: *const f32, ldr: usize, nvec: usize) -> c_int;
    pub fn hc_gemv_dev_noalloc(eng: *mut hc_engine, w: *const hc_weights, x: *const f32, ldx: usize, y: *mut f32,
                               ldy: usize, resid: *const f32, ldr: usize, nvec: usize) -> c_int;
    pub fn hc_lut_matmul_q4(eng: *mut hc_engine, m: usize, n: usize, weights_q4: *const u8, lut16: *const f32,
                            input: *const f32, output: *mut f32) -> c_int;
    pub fn hc_lut_matmul_q4_dev(eng: *mut hc_engine, m: usize, n: usize, weights_q4: *const u8, lut16: *const f32,
                                input: *const f32, output: *mut f32) -> c_int;
    pub fn hc_ffn_swiglu(eng: *mut hc_engine, gate: *const hc_weights, up: *const hc_weights, down: *const hc_weights,
                         x: *const f32, y: *mut f32, nvec: usize) -> c_int;
    pub fn hc_ffn_swiglu_dev(eng: *mut hc_engine, gate: *const hc_weights, up: *const hc_weights,
                             down: *const hc_weights, x: *const f32, y: *mut f32, resid: *const f32, h_ws: *mut f32,
                             nvec: usize) -> c_int;
    pub fn hc_ffn_gateup_dev(eng: *mut hc_engine, gate: *const hc_weights, up: *const hc_weights, x: *const f32,
                             h: *mut f32, nvec: usize, norm_w: *const f32, norm_len: usize, eps: f32) -> c_int;
    pub fn hc_ffn_stack_dev(eng: *mut hc_engine, gate: *const *const hc_weights, up: *const *const hc_weights,
                            down: *const *const hc_weights, norm_w: *const *const f32, eps: f32, n_layers: usize,
                            x: *mut f32, nvec: usize) -> c_int;
    pub fn hc_ffn_stack(eng: *mut hc_engine, gate: *const *const hc_weights, up: *const *const hc_weights,
                        down: *const *const hc_weights, norm_w: *const *const f32, eps: f32, n_layers: usize,
                        x_in: *const f32, x_out: *mut f32, nvec: usize) -> c_int;
    pub fn hc_peer_handle_bytes(out: *mut usize) -> c_int;
    pub fn hc_peer_open(eng: *mut hc_engine, rank: c_int, world: c_int, bytes: usize, handle_out: *mut c_void) -> c_int;
    pub fn hc_peer_connect(eng: *mut hc_engine, handles: *const c_void) -> c_int;
    pub fn hc_peer_close(eng: *mut hc_engine) -> c_int;
    pub fn hc_peer_region(eng: *mut hc_engine, region: *mut *mut c_void, bytes: *mut usize) -> c_int;
    pub fn hc_ffn_stack_tp_dev(eng: *mut hc_engine, gate: *const *const hc_weights, up: *const *const hc_weights,
                               down: *const *const hc_weights, norm_w: *const *const f32, eps: f32, n_layers: usize,
                               x: *mut f32, nvec: usize) -> c_int;
    pub fn hc_ffn_stack_tp(eng: *mut hc_engine, gate: *const *const hc_weights, up: *const *const hc_weights,
                           down: *const *const hc_weights, norm_w: *const *const f32, eps: f32, n_layers: usize,
                           x_in: *const f32, x_out: *mut f32, nvec: usize) -> c_int;
    pub fn hc_route_experts_dev(eng: *mut hc_engine, scores: *const f32, bias: *const f32, n_tok: usize,
                                n_expert: usize, top_k: usize, n_group: usize, topk_group: usize, gating: c_int,
                                norm_topk_prob: c_int, routed_scaling_factor: f32, ids: *mut i32,
                                weights: *mut f32) -> c_int;
    pub fn hc_router_scores_dev(eng: *mut hc_engine, router_w: *const f32, n_expert: usize, d_model: usize,
                                x: *const f32, n_tok: usize, scores: *mut f32) -> c_int;
    pub fn hc_moe_ffn_dev(eng: *mut hc_engine, router_w: *const f32, n_expert: usize, top_k: usize,
                          norm_topk_prob: c_int, routed_scaling_factor: f32, gate: *const *const hc_weights,
                          up: *const *const hc_weights, down: *const *const hc_weights, x: *const f32, n_tok: usize,
                          y: *mut f32, ids_out: *mut i32, w_out: *mut f32) -> c_int;
    pub fn hc_moe_ffn_ep_dev(eng: *mut hc_engine, router_w: *const f32, n_expert: usize, top_k: usize,
                             norm_topk_prob: c_int, routed_scaling_factor: f32, gate: *const *const hc_weights,
                             up: *const *const hc_weights, down: *const *const hc_weights, expert_lo: usize,
                             n_local: usize, x: *const f32, n_tok: usize, y: *mut f32, ids_out: *mut i32,
                             w_out: *mut f32) -> c_int;
    pub fn hc_moe_stack_dev(eng: *mut hc_engine, n_layers: usize, router_w: *const *const f32, n_expert: usize,
                            top_k: usize, norm_topk_prob: c_int, routed_scaling_factor: f32,
                            gate: *const *const hc_weights, up: *const *const hc_weights,
                            down: *const *const hc_weights, x: *mut f32, n_tok: usize) -> c_int;
    pub fn hc_moe_stack_ep_dev(eng: *mut hc_engine, n_layers: usize, router_w: *const *const f32, n_expert: usize,
                               top_k: usize, norm_topk_prob: c_int, routed_scaling_factor: f32,
                               gate: *const *const hc_weights, up: *const *const hc_weights,
                               down: *const *const hc_weights, expert_lo: usize, n_local: usize, x: *mut f32,
                               n_tok: usize) -> c_int;
    pub fn hc_synth_normal_dev(eng: *mut hc_engine, seed: u64, n: usize, mean: f32, stdv: f32, out: *mut f32) -> c_int;
    pub fn hc_quantize_dev(eng: *mut hc_engine, ggml_type: c_int, x: *const f32, n: usize, out: *mut u8) -> c_int;
}
