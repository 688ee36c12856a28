//! The C ABI of `libmote_cuda` (`include/mote_cuda.h`), one declaration per
//! entry point -- the CUDA counterpart of `crates/mote-backend-hip/src/ffi.rs`.
//! Every kernel entry takes its stream last and returns 0 on success; the
//! status codes are those of the HIP shims (1 invalid value, 9 invalid
//! configuration, -1 the norm/RoPE shims' internal error) plus this
//! library's own (10000 NCCL missing, 10001 NCCL deadline, 10100 + an
//! ncclResult_t, 10200 scratch too small); `mote_cuda_status_string` names
//! them.
//!
//! NOT COMPILED IN THIS REPOSITORY'S BUILD ENVIRONMENT: it has no `cargo`.
//! The declarations follow the header's prototypes one for one (argument
//! order and types).
#![allow(dead_code)]

use std::ffi::{c_char, c_void};

pub type Status = i32;
pub const SUCCESS: Status = 0;

/// One layer of `mote_cuda_q4_0_decoder_stack_f16` (`mote_cuda_stack_layer`).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct StackLayer {
    pub w_qkv: *const c_void,
    pub w_o: *const c_void,
    pub w_gate: *const c_void,
    pub w_up: *const c_void,
    pub w_down: *const c_void,
    pub gamma1: *const c_void,
    pub gamma2: *const c_void,
    pub attn: *const c_void,
    pub cos: *const c_void,
    pub sin: *const c_void,
    pub qkv: *mut c_void,
    pub h1: *mut c_void,
    pub a: *mut c_void,
    pub out: *mut c_void,
}

unsafe extern "C" {
    pub fn mote_cuda_get_device_count(count: *mut i32) -> i32;
    pub fn mote_cuda_set_device(ordinal: i32) -> i32;
    pub fn mote_cuda_malloc(pointer: *mut *mut c_void, bytes: usize) -> i32;
    pub fn mote_cuda_free(pointer: *mut c_void) -> i32;
    pub fn mote_cuda_memcpy_host_to_device(destination: *mut c_void, source: *const c_void, bytes: usize) -> i32;
    pub fn mote_cuda_memcpy_device_to_host(destination: *mut c_void, source: *const c_void, bytes: usize) -> i32;
    pub fn mote_cuda_stream_create(stream: *mut *mut c_void) -> i32;
    pub fn mote_cuda_stream_destroy(stream: *mut c_void) -> i32;
    pub fn mote_cuda_stream_synchronize(stream: *mut c_void) -> i32;
    pub fn mote_cuda_mem_get_info(free_bytes: *mut usize, total_bytes: *mut usize) -> i32;
    pub fn mote_cuda_memcpy_host_to_device_async(destination: *mut c_void, source: *const c_void, bytes: usize, stream: *mut c_void) -> i32;
    pub fn mote_cuda_memcpy_device_to_host_async(destination: *mut c_void, source: *const c_void, bytes: usize, stream: *mut c_void) -> i32;
    pub fn mote_cuda_memset_async(destination: *mut c_void, value: i32, bytes: usize, stream: *mut c_void) -> i32;
    pub fn mote_cuda_host_alloc(pointer: *mut *mut c_void, bytes: usize) -> i32;
    pub fn mote_cuda_host_free(pointer: *mut c_void) -> i32;
    pub fn mote_cuda_event_create(event: *mut *mut c_void) -> i32;
    pub fn mote_cuda_event_destroy(event: *mut c_void) -> i32;
    pub fn mote_cuda_event_record(event: *mut c_void, stream: *mut c_void) -> i32;
    pub fn mote_cuda_event_elapsed_ms(ms: *mut f32, start: *mut c_void, end: *mut c_void) -> i32;
    pub fn mote_cuda_stream_wait_event(stream: *mut c_void, event: *mut c_void) -> i32;
    pub fn mote_cuda_device_status(status: *mut u32, clear: i32) -> i32;
    pub fn mote_cuda_status_string(status: i32) -> *const c_char;
    pub fn mote_cuda_abi_version() -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f16(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f16_f32out(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f32(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q8_0_f16(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q8_0_f16_f32out(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_k_f16(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_k_f16_f32out(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q6_k_f16(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_blaslt_create(output: *mut *mut c_void) -> i32;
    pub fn mote_cuda_blaslt_destroy(context: *mut c_void);
    pub fn mote_cuda_blaslt_last_error(context: *mut c_void) -> *const c_char;
    pub fn mote_cuda_blaslt_matmul_f16_f32(context: *mut c_void, m: u64, n: u64, k: u64, lhs: *const c_void, rhs: *const c_void, output: *mut c_void, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> i32;
    pub fn mote_cuda_kquant_dequantize_f32(format: i32, weights: *const c_void, output: *mut c_void, rows: u64, k: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f16_ws(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, workspace: *mut c_void, workspace_bytes: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f16_noalloc(input: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_linear_workspace_bytes(rows: u64, output_features: u64, input_features: u64, bytes: *mut u64) -> i32;
    pub fn mote_cuda_q4_0_gate_up_swiglu_f16(input: *const c_void, gate_weights: *const c_void, up_weights: *const c_void, output: *mut c_void, rows: u64, ffn_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f16_residual(input: *const c_void, weights: *const c_void, residual: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_rms_norm_linear_f16(input: *const c_void, gamma: *const c_void, weights: *const c_void, output: *mut c_void, rows: u64, output_features: u64, input_features: u64, epsilon: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16(input: *const c_void, gamma: *const c_void, gate_weights: *const c_void, up_weights: *const c_void, output: *mut c_void, rows: u64, ffn_features: u64, input_features: u64, epsilon: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_rms_norm_qkv_rope_f16(input: *const c_void, gamma: *const c_void, weights: *const c_void, cos: *const c_void, sin: *const c_void, output: *mut c_void, rows: u64, q_heads: u64, kv_heads: u64, head_dim: u64, input_features: u64, epsilon: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_decode_f32(weights: *const c_void, output: *mut c_void, rows: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_encode_f32(input: *const c_void, weights: *mut c_void, rows: u64, input_features: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_rms_norm_f16(input: *const c_void, weight: *const c_void, output: *mut c_void, rows: u64, hidden_size: u64, epsilon: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_fused_add_rms_norm_f16(input: *const c_void, residual: *mut c_void, weight: *const c_void, output: *mut c_void, rows: u64, hidden_size: u64, epsilon: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_rope_f16(input: *const c_void, cos: *const c_void, sin: *const c_void, output: *mut c_void, tokens: u64, heads: u64, head_dim: u64, rotary_dim: u64, layout: u32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_rms_norm_rope_f16(x: *const c_void, gamma: *const c_void, x_out: *mut c_void, q: *const c_void, q_out: *mut c_void, k: *const c_void, k_out: *mut c_void, cos: *const c_void, sin: *const c_void, tokens: u64, hidden: u64, q_heads: u64, kv_heads: u64, head_dim: u64, layout: u32, epsilon: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_swiglu_f16(gate: *const c_void, up: *const c_void, output: *mut c_void, n: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_embedding_gather_f16(table: *const c_void, ids: *const c_void, output: *mut c_void, tokens: u64, vocab: u64, hidden: u64, error_flag: *mut c_void, stream: *mut c_void) -> i32;
    pub fn mote_cuda_rope_cos_sin_f32(positions: *const c_void, cos_out: *mut c_void, sin_out: *mut c_void, tokens: u64, rotary_dim: u64, theta: f64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_q4_0_decoder_stack_workspace_bytes(hidden: u64, bytes: *mut u64) -> i32;
    pub fn mote_cuda_q4_0_decoder_stack_f16(layers: *const c_void, num_layers: u32, h_in: *const c_void, hidden: u64, ffn: u64, q_heads: u64, kv_heads: u64, head_dim: u64, epsilon: f32, workspace: *mut c_void, workspace_bytes: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_kv_cache_append_f16(k_new: *const c_void, v_new: *const c_void, k_cache: *mut c_void, v_cache: *mut c_void, slots: *const c_void, tokens: u64, kv_heads: u64, head_dim: u64, cache_rows: u64, error_flag: *mut c_void, stream: *mut c_void) -> i32;
    pub fn mote_cuda_gqa_attention_decode_workspace_bytes(batch: u64, q_heads: u64, kv_heads: u64, head_dim: u64, max_len: u64, bytes: *mut u64) -> i32;
    pub fn mote_cuda_gqa_attention_decode_f16(q: *const c_void, k_cache: *const c_void, v_cache: *const c_void, seq_lens: *const c_void, out: *mut c_void, batch: u64, q_heads: u64, kv_heads: u64, head_dim: u64, seq_capacity: u64, max_len: u64, scale: f32, workspace: *mut c_void, workspace_bytes: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_gqa_attention_prefill_f16(q: *const c_void, k_cache: *const c_void, v_cache: *const c_void, out: *mut c_void, tokens: u64, start: u64, q_heads: u64, kv_heads: u64, head_dim: u64, row0: u64, cache_rows: u64, scale: f32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_comm_unique_id(id_out: *mut c_void) -> i32;
    pub fn mote_cuda_comm_init(comm: *mut *mut c_void, nranks: i32, id: *const c_void, rank: i32) -> i32;
    pub fn mote_cuda_comm_init_timeout(comm: *mut *mut c_void, nranks: i32, id: *const c_void, rank: i32, timeout_ms: u64) -> i32;
    pub fn mote_cuda_comm_all_gather_f16(comm: *mut c_void, send: *const c_void, recv: *mut c_void, count: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_comm_destroy(comm: *mut c_void) -> i32;
    pub fn mote_cuda_comm_abort(comm: *mut c_void) -> i32;
    pub fn mote_cuda_ipc_get_handle(dev_ptr: *const c_void, handle_out: *mut c_void) -> i32;
    pub fn mote_cuda_ipc_open_handle(handle: *const c_void, dev_ptr: *mut *mut c_void) -> i32;
    pub fn mote_cuda_ipc_close_handle(dev_ptr: *mut c_void) -> i32;
    pub fn mote_cuda_all_gather_p2p_f16(send: *const c_void, recv_ptrs: *const *mut c_void, flag_ptrs: *const *mut u32, own_flags: *mut u32, count: u64, rank: u32, nranks: u32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_all_gather_p2p_f16_timeout(send: *const c_void, recv_ptrs: *const *mut c_void, flag_ptrs: *const *mut u32, own_flags: *mut u32, count: u64, rank: u32, nranks: u32, wait_ns: u64, stream: *mut c_void) -> i32;
    pub fn mote_cuda_peer_flags_reset(own_flags: *mut u32, nranks: u32, stream: *mut c_void) -> i32;
    pub fn mote_cuda_quantized_linear_q4_0_f16_allgather(input: *const c_void, weights: *const c_void, outputs: *const *mut c_void, flag_ptrs: *const *mut u32, own_flags: *mut u32, rows: u64, shard_features: u64, input_features: u64, total_features: u64, rank: u32, nranks: u32, stream: *mut c_void) -> i32;
}
