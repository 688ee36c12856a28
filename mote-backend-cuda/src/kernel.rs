//! `mote-kernel` registration: one `KernelImpl` per C entry point, keyed by
//! operator and dtype, supported on `BackendKind::Cuda` devices
//! (crates/mote-kernel/src/lib.rs:7-56; the table mirrors this
//! repository's mote_b200/kernel.py `CUDA_KERNELS`).
//!
//! Argument convention (`KernelArgs::opaque`): the C argument list in order,
//! one word each -- pointers and sizes as `usize`, `f32`/`f64` scalars as
//! their IEEE bits, `u32` selectors as their value, the stream handle last.
//! Later registrations take precedence (`KernelRegistry::resolve`), so
//! registering these after a portable implementation makes them the CUDA
//! device's choice.
//!
//! NOT COMPILED HERE (no cargo in this environment).

use mote_kernel::{KernelArgs, KernelError, KernelImpl, KernelKey, KernelRegistry};
use mote_types::{BackendKind, DType, Device};

use crate::{error, ffi};

type Call = fn(&[usize]) -> i32;

/// (operator, dtype, C symbol, argument words, call)
const KERNELS: &[(&str, DType, &str, usize, Call)] = &[
    ("quantized_linear_q4_0", DType::F16, "mote_cuda_quantized_linear_q4_0_f16", 7, call_quantized_linear_q4_0_f16),
    ("quantized_linear_q4_0_f32out", DType::F16, "mote_cuda_quantized_linear_q4_0_f16_f32out", 7, call_quantized_linear_q4_0_f16_f32out),
    ("quantized_linear_q4_0", DType::F32, "mote_cuda_quantized_linear_q4_0_f32", 7, call_quantized_linear_q4_0_f32),
    ("quantized_linear_q8_0", DType::F16, "mote_cuda_quantized_linear_q8_0_f16", 7, call_quantized_linear_q8_0_f16),
    ("quantized_linear_q8_0_f32out", DType::F16, "mote_cuda_quantized_linear_q8_0_f16_f32out", 7, call_quantized_linear_q8_0_f16_f32out),
    ("quantized_linear_q4_k", DType::F16, "mote_cuda_quantized_linear_q4_k_f16", 7, call_quantized_linear_q4_k_f16),
    ("quantized_linear_q4_k_f32out", DType::F16, "mote_cuda_quantized_linear_q4_k_f16_f32out", 7, call_quantized_linear_q4_k_f16_f32out),
    ("quantized_linear_q6_k", DType::F16, "mote_cuda_quantized_linear_q6_k_f16", 7, call_quantized_linear_q6_k_f16),
    ("gate_up_swiglu_q4_0", DType::F16, "mote_cuda_q4_0_gate_up_swiglu_f16", 8, call_q4_0_gate_up_swiglu_f16),
    ("quantized_linear_q4_0_residual", DType::F16, "mote_cuda_quantized_linear_q4_0_f16_residual", 8, call_quantized_linear_q4_0_f16_residual),
    ("quantized_linear_q4_0_ws", DType::F16, "mote_cuda_quantized_linear_q4_0_f16_ws", 9, call_quantized_linear_q4_0_f16_ws),
    ("quantized_linear_q4_0_noalloc", DType::F16, "mote_cuda_quantized_linear_q4_0_f16_noalloc", 7, call_quantized_linear_q4_0_f16_noalloc),
    ("rms_norm_linear_q4_0", DType::F16, "mote_cuda_q4_0_rms_norm_linear_f16", 9, call_q4_0_rms_norm_linear_f16),
    ("rms_norm_gate_up_swiglu_q4_0", DType::F16, "mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16", 10, call_q4_0_rms_norm_gate_up_swiglu_f16),
    ("rms_norm_qkv_rope_q4_0", DType::F16, "mote_cuda_q4_0_rms_norm_qkv_rope_f16", 13, call_q4_0_rms_norm_qkv_rope_f16),
    ("rms_norm", DType::F16, "mote_cuda_rms_norm_f16", 7, call_rms_norm_f16),
    ("fused_add_rms_norm", DType::F16, "mote_cuda_fused_add_rms_norm_f16", 8, call_fused_add_rms_norm_f16),
    ("rope", DType::F16, "mote_cuda_rope_f16", 10, call_rope_f16),
    ("rms_norm_rope", DType::F16, "mote_cuda_rms_norm_rope_f16", 17, call_rms_norm_rope_f16),
    ("swiglu", DType::F16, "mote_cuda_swiglu_f16", 5, call_swiglu_f16),
    ("embedding_gather", DType::F16, "mote_cuda_embedding_gather_f16", 8, call_embedding_gather_f16),
    ("q4_0_decode", DType::F32, "mote_cuda_q4_0_decode_f32", 5, call_q4_0_decode_f32),
    ("q4_0_encode", DType::F32, "mote_cuda_q4_0_encode_f32", 5, call_q4_0_encode_f32),
    ("rope_cos_sin", DType::F32, "mote_cuda_rope_cos_sin_f32", 7, call_rope_cos_sin_f32),
    ("kv_cache_append", DType::F16, "mote_cuda_kv_cache_append_f16", 11, call_kv_cache_append_f16),
    ("gqa_attention_decode", DType::F16, "mote_cuda_gqa_attention_decode_f16", 15, call_gqa_attention_decode_f16),
    ("gqa_attention_prefill", DType::F16, "mote_cuda_gqa_attention_prefill_f16", 13, call_gqa_attention_prefill_f16),
    ("decoder_stack_q4_0", DType::F16, "mote_cuda_q4_0_decoder_stack_f16", 12, call_q4_0_decoder_stack_f16),
];

struct CudaKernel {
    op: &'static str,
    symbol: &'static str,
    words: usize,
    call: Call,
}

impl KernelImpl for CudaKernel {
    fn name(&self) -> &'static str {
        self.symbol
    }

    fn supports(&self, device: &Device, key: &KernelKey) -> bool {
        device.backend() == BackendKind::Cuda && key.op == self.op
    }

    fn launch(&self, device: &Device, args: &KernelArgs<'_>) -> Result<(), KernelError> {
        if args.opaque.len() != self.words {
            return Err(KernelError::Launch(format!(
                "{} takes {} words, got {}",
                self.symbol,
                self.words,
                args.opaque.len()
            )));
        }
        // SAFETY: plain runtime call on the device's ordinal.
        let status = unsafe { ffi::mote_cuda_set_device(device.ordinal() as i32) };
        if status != ffi::SUCCESS {
            return Err(KernelError::Launch(error::status_string(status)));
        }
        let status = (self.call)(args.opaque);
        if status == ffi::SUCCESS {
            Ok(())
        } else {
            Err(KernelError::Launch(format!(
                "{}: status {status} ({})",
                self.symbol,
                error::status_string(status)
            )))
        }
    }
}

/// Registers every CUDA kernel of this backend.
pub fn register(registry: &mut KernelRegistry) {
    for &(op, dtype, symbol, words, call) in KERNELS {
        registry.register(
            KernelKey { op, dtype: Some(dtype), shape_class: None },
            CudaKernel { op, symbol, words, call },
        );
    }
}

fn call_quantized_linear_q4_0_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_0_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q4_0_f16_f32out(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_0_f16_f32out(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q4_0_f32(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_0_f32(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q8_0_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q8_0_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q8_0_f16_f32out(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q8_0_f16_f32out(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q4_k_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_k_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q4_k_f16_f32out(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_k_f16_f32out(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_quantized_linear_q6_k_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q6_k_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_q4_0_gate_up_swiglu_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_gate_up_swiglu_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *mut c_void, w[4] as u64, w[5] as u64, w[6] as u64, w[7] as *mut c_void) }
}
fn call_quantized_linear_q4_0_f16_residual(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_0_f16_residual(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *mut c_void, w[4] as u64, w[5] as u64, w[6] as u64, w[7] as *mut c_void) }
}
fn call_quantized_linear_q4_0_f16_ws(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_0_f16_ws(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void, w[7] as u64, w[8] as *mut c_void) }
}
fn call_quantized_linear_q4_0_f16_noalloc(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_quantized_linear_q4_0_f16_noalloc(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void) }
}
fn call_q4_0_rms_norm_linear_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_rms_norm_linear_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *mut c_void, w[4] as u64, w[5] as u64, w[6] as u64, f32::from_bits(w[7] as u32), w[8] as *mut c_void) }
}
fn call_q4_0_rms_norm_gate_up_swiglu_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *const c_void, w[4] as *mut c_void, w[5] as u64, w[6] as u64, w[7] as u64, f32::from_bits(w[8] as u32), w[9] as *mut c_void) }
}
fn call_q4_0_rms_norm_qkv_rope_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_rms_norm_qkv_rope_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *const c_void, w[4] as *const c_void, w[5] as *mut c_void, w[6] as u64, w[7] as u64, w[8] as u64, w[9] as u64, w[10] as u64, f32::from_bits(w[11] as u32), w[12] as *mut c_void) }
}
fn call_rms_norm_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_rms_norm_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, f32::from_bits(w[5] as u32), w[6] as *mut c_void) }
}
fn call_fused_add_rms_norm_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_fused_add_rms_norm_f16(w[0] as *const c_void, w[1] as *mut c_void, w[2] as *const c_void, w[3] as *mut c_void, w[4] as u64, w[5] as u64, f32::from_bits(w[6] as u32), w[7] as *mut c_void) }
}
fn call_rope_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_rope_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *mut c_void, w[4] as u64, w[5] as u64, w[6] as u64, w[7] as u64, w[8] as u32, w[9] as *mut c_void) }
}
fn call_rms_norm_rope_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_rms_norm_rope_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as *const c_void, w[4] as *mut c_void, w[5] as *const c_void, w[6] as *mut c_void, w[7] as *const c_void, w[8] as *const c_void, w[9] as u64, w[10] as u64, w[11] as u64, w[12] as u64, w[13] as u64, w[14] as u32, f32::from_bits(w[15] as u32), w[16] as *mut c_void) }
}
fn call_swiglu_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_swiglu_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as *mut c_void) }
}
fn call_embedding_gather_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_embedding_gather_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as *mut c_void, w[7] as *mut c_void) }
}
fn call_q4_0_decode_f32(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_decode_f32(w[0] as *const c_void, w[1] as *mut c_void, w[2] as u64, w[3] as u64, w[4] as *mut c_void) }
}
fn call_q4_0_encode_f32(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_encode_f32(w[0] as *const c_void, w[1] as *mut c_void, w[2] as u64, w[3] as u64, w[4] as *mut c_void) }
}
fn call_rope_cos_sin_f32(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_rope_cos_sin_f32(w[0] as *const c_void, w[1] as *mut c_void, w[2] as *mut c_void, w[3] as u64, w[4] as u64, f64::from_bits(w[5] as u64), w[6] as *mut c_void) }
}
fn call_kv_cache_append_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_kv_cache_append_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *mut c_void, w[3] as *mut c_void, w[4] as *const c_void, w[5] as u64, w[6] as u64, w[7] as u64, w[8] as u64, w[9] as *mut c_void, w[10] as *mut c_void) }
}
fn call_gqa_attention_decode_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_gqa_attention_decode_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *const c_void, w[4] as *mut c_void, w[5] as u64, w[6] as u64, w[7] as u64, w[8] as u64, w[9] as u64, w[10] as u64, f32::from_bits(w[11] as u32), w[12] as *mut c_void, w[13] as u64, w[14] as *mut c_void) }
}
fn call_gqa_attention_prefill_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_gqa_attention_prefill_f16(w[0] as *const c_void, w[1] as *const c_void, w[2] as *const c_void, w[3] as *mut c_void, w[4] as u64, w[5] as u64, w[6] as u64, w[7] as u64, w[8] as u64, w[9] as u64, w[10] as u64, f32::from_bits(w[11] as u32), w[12] as *mut c_void) }
}
fn call_q4_0_decoder_stack_f16(w: &[usize]) -> i32 {
    // SAFETY: the caller's words follow the entry point's argument list.
    unsafe { ffi::mote_cuda_q4_0_decoder_stack_f16(w[0] as *const c_void, w[1] as u32, w[2] as *const c_void, w[3] as u64, w[4] as u64, w[5] as u64, w[6] as u64, w[7] as u64, f32::from_bits(w[8] as u32), w[9] as *mut c_void, w[10] as u64, w[11] as *mut c_void) }
}
