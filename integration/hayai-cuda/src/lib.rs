//! hayai-cuda: the OpenClEngine-shaped wrapper the orchestrator calls for the B200 backend.
//!
//! Mirrors the method set of `OpenClEngine` (crates/hayai-opencl/src/compute.rs:45-461,
//! async_gemv.rs:15-130) over the C ABI of libhayai_cuda.so (include/hayai_cuda.h).  Ownership
//! follows the ABI: the engine owns its stream and workspaces, `ResidentWeights` own their
//! HBM copy, host slices are borrowed for one call (or until `PendingGemv::wait`).
pub mod ffi;
pub mod orchestrator_arm;

use std::ffi::CStr;

/// A failed call: the status code (`ffi::HC_ERR_*`) and `hc_last_error()` of this thread
/// (the `OpenClError::ClError(String)` counterpart).
#[derive(Debug, Clone, PartialEq, Eq)]
pub struct CudaError {
    pub code: i32,
    pub msg: String,
}

impl std::fmt::Display for CudaError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "hayai-cuda error {}: {}", self.code, self.msg)
    }
}
impl std::error::Error for CudaError {}

pub fn last_error() -> String {
    unsafe { CStr::from_ptr(ffi::hc_last_error()).to_string_lossy().into_owned() }
}

fn check(rc: i32) -> Result<(), CudaError> {
    if rc == ffi::HC_OK {
        Ok(())
    } else {
        Err(CudaError { code: rc, msg: last_error() })
    }
}

pub fn device_count() -> usize {
    let mut n = 0;
    if unsafe { ffi::hc_device_count(&mut n) } == ffi::HC_OK { n as usize } else { 0 }
}

/// One GPU and its stream (OpenClEngine).
pub struct CudaEngine {
    raw: *mut ffi::hc_engine,
    pub device: i32,
}

// Used behind the orchestrator's Mutex, like OpenClEngine (orchestrator.rs:65-68).
unsafe impl Send for CudaEngine {}

/// A matrix uploaded once to HBM (the resident device mirror).
pub struct ResidentWeights {
    raw: *mut ffi::hc_weights,
    pub ggml_type: u32,
    pub m: usize,
    pub n: usize,
}
unsafe impl Send for ResidentWeights {}

impl Drop for ResidentWeights {
    fn drop(&mut self) {
        unsafe { ffi::hc_weights_free(self.raw) };
    }
}

/// An in-flight GEMV (PendingGemv): `wait` returns the output; dropping it waits first.
pub struct PendingGemv {
    raw: *mut ffi::hc_pending,
    m: usize,
}
unsafe impl Send for PendingGemv {}

impl PendingGemv {
    pub fn wait(mut self) -> Result<Vec<f32>, CudaError> {
        let mut out = vec![0.0f32; self.m];
        let rc = unsafe { ffi::hc_pending_wait(self.raw, out.as_mut_ptr(), self.m) };
        unsafe { ffi::hc_pending_free(self.raw) };
        self.raw = std::ptr::null_mut();
        check(rc)?;
        Ok(out)
    }
}

impl Drop for PendingGemv {
    fn drop(&mut self) {
        if !self.raw.is_null() {
            unsafe { ffi::hc_pending_free(self.raw) };  // blocks until the device is done
        }
    }
}

impl CudaEngine {
    /// OpenClEngine::init_device (context.rs:106).
    pub fn init_device(device: i32) -> Result<Self, CudaError> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::hc_engine_init(device, &mut raw) })?;
        Ok(Self { raw, device })
    }

    pub fn sync(&self) -> Result<(), CudaError> {
        check(unsafe { ffi::hc_sync(self.raw) })
    }

    /// OpenClEngine::ggml_gemv_dispatch (compute.rs:281): host weights, host x, host y;
    /// the kernel is chosen by the GgmlType id.
    pub fn ggml_gemv_dispatch(&self, ggml_type: u32, m: usize, n: usize, weights: &[u8], input: &[f32],
                              output: &mut [f32]) -> Result<(), CudaError> {
        assert_eq!(input.len(), n);
        assert_eq!(output.len(), m);
        check(unsafe {
            ffi::hc_ggml_gemv_dispatch(self.raw, ggml_type as i32, m, n, weights.as_ptr(), weights.len(),
                                       input.as_ptr(), output.as_mut_ptr())
        })
    }

    /// One-time resident upload (replaces the ping-pong / mirror DMA).
    pub fn upload(&self, ggml_type: u32, m: usize, n: usize, bytes: &[u8]) -> Result<ResidentWeights, CudaError> {
        let mut raw = std::ptr::null_mut();
        check(unsafe {
            ffi::hc_weights_upload(self.raw, ggml_type as i32, m, n, bytes.as_ptr().cast(), bytes.len(), &mut raw)
        })?;
        Ok(ResidentWeights { raw, ggml_type, m, n })
    }

    /// OpenClEngine::ggml_gemv_dispatch_bound (compute.rs:388) with resident weights.
    pub fn ggml_gemv_bound(&self, w: &ResidentWeights, input: &[f32], output: &mut [f32]) -> Result<(), CudaError> {
        assert_eq!(input.len(), w.n);
        assert_eq!(output.len(), w.m);
        check(unsafe { ffi::hc_ggml_gemv_bound(self.raw, w.raw, input.as_ptr(), output.as_mut_ptr()) })
    }

    /// ggml_gemv_batched_q4_k (compute.rs:179), for every type: inputs [batch][n] -> outputs [batch][m].
    pub fn ggml_gemv_batched(&self, w: &ResidentWeights, inputs: &[f32], outputs: &mut [f32],
                             batch: usize) -> Result<(), CudaError> {
        assert_eq!(inputs.len(), batch * w.n);
        assert_eq!(outputs.len(), batch * w.m);
        check(unsafe { ffi::hc_ggml_gemv_batched(self.raw, w.raw, inputs.as_ptr(), outputs.as_mut_ptr(), batch) })
    }

    /// ggml_gemv_async (async_gemv.rs:90-130).
    pub fn ggml_gemv_async(&self, w: &ResidentWeights, input: &[f32]) -> Result<PendingGemv, CudaError> {
        assert_eq!(input.len(), w.n);
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::hc_ggml_gemv_async(self.raw, w.raw, input.as_ptr(), &mut raw) })?;
        Ok(PendingGemv { raw, m: w.m })
    }

    /// lut_matmul_q4 (compute.rs:45-128).
    pub fn lut_matmul_q4(&self, m: usize, n: usize, weights_q4: &[u8], lut: &[f32; 16], input: &[f32],
                         output: &mut [f32]) -> Result<(), CudaError> {
        assert_eq!(weights_q4.len(), m * n / 2);
        check(unsafe {
            ffi::hc_lut_matmul_q4(self.raw, m, n, weights_q4.as_ptr(), lut.as_ptr(), input.as_ptr(),
                                  output.as_mut_ptr())
        })
    }

    /// One SwiGLU FFN block, y = W_d (silu(W_g x) * (W_u x)) (stream_infer.rs:3752-3864).
    pub fn ffn_swiglu(&self, gate: &ResidentWeights, up: &ResidentWeights, down: &ResidentWeights, x: &[f32],
                      y: &mut [f32], nvec: usize) -> Result<(), CudaError> {
        check(unsafe {
            ffi::hc_ffn_swiglu(self.raw, gate.raw, up.raw, down.raw, x.as_ptr(), y.as_mut_ptr(), nvec)
        })
    }

    /// A decode step's FFN sublayers: x <- x + FFN_l(rms_norm(x, norm_l)) for every layer.
    pub fn ffn_stack(&self, layers: &[(&ResidentWeights, &ResidentWeights, &ResidentWeights, &[f32])], eps: f32,
                     x_in: &[f32], x_out: &mut [f32], nvec: usize) -> Result<(), CudaError> {
        let g: Vec<_> = layers.iter().map(|l| l.0.raw as *const _).collect();
        let u: Vec<_> = layers.iter().map(|l| l.1.raw as *const _).collect();
        let d: Vec<_> = layers.iter().map(|l| l.2.raw as *const _).collect();
        let nw: Vec<*const f32> = layers.iter().map(|l| l.3.as_ptr()).collect();
        check(unsafe {
            ffi::hc_ffn_stack(self.raw, g.as_ptr(), u.as_ptr(), d.as_ptr(), nw.as_ptr(), eps, layers.len(),
                              x_in.as_ptr(), x_out.as_mut_ptr(), nvec)
        })
    }
}

impl Drop for CudaEngine {
    fn drop(&mut self) {
        unsafe { ffi::hc_engine_free(self.raw) };
    }
}
