//! The CUDA arm of hayai-core's GEMV dispatch: what `EngineOrchestrator::gemv_kernel` /
//! `gpu_gemv` (orchestrator.rs:72-98, 394-422) and `begin_gemv_engine` (:479-517) call when the
//! pool holds B200s.  There is no per-type kernel table on this side: the GgmlType id goes
//! through and the library picks the kernel; a type it lacks returns HC_ERR_UNSUPPORTED, the
//! same hard failure (no CPU fallback) as a missing OpenCL kernel.
use crate::{CudaEngine, CudaError, PendingGemv};
use hayai_model::{GgmlType, QuantMatrix};

/// GGUF type id of a GgmlType (gguf_types.rs:6-40).
pub fn ggml_id(t: GgmlType) -> u32 {
    match t {
        GgmlType::F32 => 0,
        GgmlType::F16 => 1,
        GgmlType::Q4_0 => 2,
        GgmlType::Q4_1 => 3,
        GgmlType::Q5_0 => 6,
        GgmlType::Q5_1 => 7,
        GgmlType::Q8_0 => 8,
        GgmlType::Q8_1 => 9,
        GgmlType::Q2_K => 10,
        GgmlType::Q3_K => 11,
        GgmlType::Q4_K => 12,
        GgmlType::Q5_K => 13,
        GgmlType::Q6_K => 14,
        GgmlType::Q8_K => 15,
        GgmlType::IQ2_XXS => 16,
        GgmlType::IQ2_XS => 17,
        GgmlType::IQ3_XXS => 18,
        GgmlType::IQ1_S => 19,
        GgmlType::IQ4_NL => 20,
        GgmlType::IQ3_S => 21,
        GgmlType::IQ2_S => 22,
        GgmlType::IQ4_XS => 23,
        GgmlType::I8 => 24,
        GgmlType::I16 => 25,
        GgmlType::I32 => 26,
        GgmlType::I64 => 27,
        GgmlType::F64 => 28,
        GgmlType::IQ1_M => 29,
        GgmlType::BF16 => 30,
        GgmlType::TQ1_0 => 34,
        GgmlType::TQ2_0 => 35,
        GgmlType::Other(v) => v,
    }
}

/// `gpu_gemv` for the CUDA pool: one synchronous GEMV of a QuantMatrix on host bytes.
pub fn cuda_gemv(eng: &CudaEngine, m: &QuantMatrix, input: &[f32], output: &mut [f32]) -> Result<(), CudaError> {
    eng.ggml_gemv_dispatch(ggml_id(m.ggml_type), m.nrows, m.ncols, m.data(), input, output)
}

/// `begin_gemv_engine` for the CUDA pool: uploads the matrix (callers that reuse a matrix keep
/// the `ResidentWeights` of `CudaEngine::upload` instead) and returns the pending GEMV.
pub fn begin_cuda_gemv(eng: &CudaEngine, m: &QuantMatrix, xn: &[f32]) -> Result<(PendingGemv, crate::ResidentWeights), CudaError> {
    let w = eng.upload(ggml_id(m.ggml_type), m.nrows, m.ncols, m.data())?;
    let p = eng.ggml_gemv_async(&w, xn)?;
    Ok((p, w))
}
