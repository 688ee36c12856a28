/*
 * mote_cuda.h -- C ABI of libmote_cuda.so, the B200 (sm_100a) CUDA data plane
 * for Mote's Q4_0 linear and per-token layer kernels.
 *
 * This is the surface the empty `mote-backend-cuda` crate of RiversJin/mote
 * (crates/mote-backend-cuda/src/lib.rs:1-3) binds.  It mirrors the extern "C"
 * surface of the HIP backend (crates/mote-backend-hip/src/ffi.rs) name for
 * name with the `mote_hip_` prefix replaced by `mote_cuda_`, with identical
 * argument order, types and status conventions:
 *
 *   - every function returns an int status, 0 on success;
 *   - runtime functions return the raw cudaError_t;
 *   - kernel launchers validate their arguments before enqueueing anything
 *     and return the same codes as the HIP shim they replace (1 = invalid
 *     value, 9 = invalid configuration, -1 = the norm/RoPE shims' private
 *     kInternalError), fully validated empty sizes return 0 without a launch,
 *     and after a launch they return cudaGetLastError();
 *   - pointers are untyped device pointers from mote_cuda_malloc (or any
 *     cudaMalloc'd memory), streams are opaque cudaStream_t handles and every
 *     kernel runs asynchronously on the stream it is given.
 *
 * Stream overlap: kernels are launched with programmatic dependent launch,
 * so a kernel may begin while earlier kernels of this library on the stream
 * are still running; each waits for its predecessor to complete before it
 * touches activations or outputs.  The Q4_0 and Q8_0 linears start streaming
 * their WEIGHTS before that wait (and mote_cuda_rms_norm_rope_f16 reads gamma and
 * the cos/sin rows before it), so such parameters must not be written by
 * this library's kernels still in flight on its stream (parameters written by
 * a copy, by mote_cuda_q4_0_encode_f32 or by any kernel not from this
 * library are ordered normally: those end the overlap).
 *
 * Data formats: f16 is IEEE binary16 (uint16 bits), Q4_0 is the ggml block
 * layout (per 32 elements: little-endian f16 scale d, then 16 bytes where
 * byte j holds element j in its low nibble and element j+16 in its high
 * nibble; value = (q - 8) * d), rows contiguous, K/32*18 bytes per row.
 */
#ifndef MOTE_CUDA_H
#define MOTE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------- */
/* Runtime shim: crates/mote-backend-hip/src/ffi.rs:42-61                   */
/* ---------------------------------------------------------------------- */

/* mote_hip_get_device_count (ffi.rs:43) */
int mote_cuda_get_device_count(int* count);
/* mote_hip_set_device (ffi.rs:44) */
int mote_cuda_set_device(int ordinal);
/* mote_hip_malloc (ffi.rs:45); allocations are 256-byte aligned */
int mote_cuda_malloc(void** pointer, size_t bytes);
/* mote_hip_free (ffi.rs:46) */
int mote_cuda_free(void* pointer);
/* mote_hip_memcpy_host_to_device (ffi.rs:47-51), synchronous */
int mote_cuda_memcpy_host_to_device(void* destination, const void* source, size_t bytes);
/* mote_hip_memcpy_device_to_host (ffi.rs:52-56), synchronous */
int mote_cuda_memcpy_device_to_host(void* destination, const void* source, size_t bytes);
/* mote_hip_stream_create (ffi.rs:57); non-blocking stream on the current device */
int mote_cuda_stream_create(void** stream);
/* mote_hip_stream_destroy (ffi.rs:58) */
int mote_cuda_stream_destroy(void* stream);
/* mote_hip_stream_synchronize (ffi.rs:59) */
int mote_cuda_stream_synchronize(void* stream);
/* mote_hip_mem_get_info (ffi.rs:60) */
int mote_cuda_mem_get_info(size_t* free_bytes, size_t* total_bytes);

/* Additions without a HIP counterpart: asynchronous copies, pinned host
 * memory, events, the device status word and error strings. */
int mote_cuda_memcpy_host_to_device_async(void* destination, const void* source, size_t bytes,
                                          void* stream);
int mote_cuda_memcpy_device_to_host_async(void* destination, const void* source, size_t bytes,
                                          void* stream);
int mote_cuda_memset_async(void* destination, int value, size_t bytes, void* stream);
int mote_cuda_host_alloc(void** pointer, size_t bytes);
int mote_cuda_host_free(void* pointer);
int mote_cuda_event_create(void** event);
int mote_cuda_event_destroy(void* event);
int mote_cuda_event_record(void* event, void* stream);
int mote_cuda_event_elapsed_ms(float* ms, void* start, void* end);
/* `stream` waits on the device for the work recorded in `event`
 * (cudaStreamWaitEvent); null handles -> 1. */
int mote_cuda_stream_wait_event(void* stream, void* event);
/* Reads (clear != 0: and clears) the current device's status word.  Bit 0:
 * a bounded device-side wait expired; bit 1: an index was out of range. */
int mote_cuda_device_status(unsigned* status, int clear);
const char* mote_cuda_status_string(int status);
int mote_cuda_abi_version(void);

/* ---------------------------------------------------------------------- */
/* Q4_0 weight-only linear                                                 */
/* ---------------------------------------------------------------------- */

/* Replaces mote_hip_quantized_linear_q4_0_f16
 * (crates/mote-backend-hip/src/quantized_linear.hip:56-91, bound at
 * crates/mote-backend-hip/src/ffi.rs:294-302).
 * output[rows, N] (f16) = input[rows, K] (f16) * weights[N, K] (Q4_0)^T with
 * f32 accumulation.  Errors: any null pointer (stream included) or K % 32 != 0
 * -> 1; rows*N beyond 32 bits -> 9; rows == 0 or N == 0 -> 0, no launch;
 * K == 0 writes zeros. */
int mote_cuda_quantized_linear_q4_0_f16(const void* input, const void* weights, void* output,
                                        uint64_t rows, uint64_t output_features,
                                        uint64_t input_features, void* stream);

/* Same contract, f16 input and f32 output (the f32 accumulator unrounded).
 * No HIP counterpart; same argument rules as the f16 entry point. */
int mote_cuda_quantized_linear_q4_0_f16_f32out(const void* input, const void* weights,
                                               void* output, uint64_t rows,
                                               uint64_t output_features, uint64_t input_features,
                                               void* stream);

/* f32 input and f32 output: the device counterpart of mote-reference's
 * quantized_linear_f32 (crates/mote-reference/src/quantized.rs:89-144) for
 * Q4_0.  Same argument rules as the f16 entry point. */
int mote_cuda_quantized_linear_q4_0_f32(const void* input, const void* weights, void* output,
                                        uint64_t rows, uint64_t output_features,
                                        uint64_t input_features, void* stream);

/* Q8_0 weights (ggml blocks of 34 bytes: little-endian f16 scale d, then 32
 * signed bytes; value = q * d), f16 input, f32 accumulation, f16 or f32
 * output: the device counterpart of mote-reference's quantized_linear_f32
 * for Q8_0 (crates/mote-reference/src/quantized.rs:89-144, decode :191-195).
 * No HIP counterpart (the HIP backend has a Q4_0 linear only); argument
 * rules as mote_cuda_quantized_linear_q4_0_f16.  More than 16 tokens run on
 * the tensor-core GEMM when N % 16 == 0, K % 256 == 0 and the pointers are
 * 16-byte aligned, else as consecutive decode launches of up to 16. */
int mote_cuda_quantized_linear_q8_0_f16(const void* input, const void* weights, void* output,
                                        uint64_t rows, uint64_t output_features,
                                        uint64_t input_features, void* stream);
int mote_cuda_quantized_linear_q8_0_f16_f32out(const void* input, const void* weights,
                                               void* output, uint64_t rows,
                                               uint64_t output_features, uint64_t input_features,
                                               void* stream);

/* K-quant weights (ggml 256-element super-blocks): Q4_K (144 bytes: f16 d,
 * f16 dmin, 12 bytes of packed 6-bit scales and mins, 128 bytes of nibbles;
 * value = d*sc*q - dmin*m) and Q6_K (210 bytes: 128 bytes of low nibbles, 64
 * of 2-bit high parts, 16 int8 scales, f16 d; value = d*sc*(q - 32)).  f16
 * input [rows, K], f32 accumulation, f16 (or, for Q4_K, f32) output [rows,
 * N].  No reference counterpart: mote-types fixes the geometry
 * (crates/mote-types/src/lib.rs:41-74) and mote-reference rejects these
 * formats (crates/mote-reference/src/quantized.rs:152-157).  K % 256 != 0 is
 * an invalid value; other rules as mote_cuda_quantized_linear_q4_0_f16.
 * Tensor-core decode kernels run up to 16 tokens per launch when the input
 * and weights are 16-byte aligned (Q6_K also needs K % 2048 == 0); more
 * than 16 tokens with N % 16 == 0 (and, for Q6_K, K % 2048 == 0) run on
 * the tcgen05 GEMM (weights rounded to f16 once); other shapes run a
 * warp-per-row kernel. */
int mote_cuda_quantized_linear_q4_k_f16(const void* input, const void* weights, void* output,
                                        uint64_t rows, uint64_t output_features,
                                        uint64_t input_features, void* stream);
int mote_cuda_quantized_linear_q4_k_f16_f32out(const void* input, const void* weights,
                                               void* output, uint64_t rows,
                                               uint64_t output_features, uint64_t input_features,
                                               void* stream);
int mote_cuda_quantized_linear_q6_k_f16(const void* input, const void* weights, void* output,
                                        uint64_t rows, uint64_t output_features,
                                        uint64_t input_features, void* stream);

/* Dense row-major matmul through cuBLASLt: the counterpart of the HIP
 * backend's hipBLASLt shim (crates/mote-backend-hip/src/hipblaslt_shim.cpp:
 * 326-408; mote_hipblaslt_create / _destroy / _last_error /
 * _matmul_f16_f32), same arguments and status rules.  create: a context in
 * *output (-1 for a null output or when cuBLASLt cannot be loaded, else the
 * library status).  last_error: the message of the context's last failed
 * call ("" after a success).  matmul: output[m, n] f32 = lhs[m, k] f16 x
 * rhs[k, n] f16, f32 accumulation, on `stream`; null pointers (stream and
 * workspace included) return -1; library failures the cuBLAS status; CUDA
 * failures -1000 - code.  The first call for a new (m, n, k) times the
 * library's candidate algorithms on the stream (it synchronizes; make it
 * before any stream capture) and caches the fastest.  m or n == 0 succeeds
 * without a launch; k == 0 writes zeros.  cuBLASLt is loaded with dlopen. */
int mote_cuda_blaslt_create(void** output);
void mote_cuda_blaslt_destroy(void* context);
const char* mote_cuda_blaslt_last_error(void* context);
int mote_cuda_blaslt_matmul_f16_f32(void* context, uint64_t m, uint64_t n, uint64_t k,
                                    const void* lhs, const void* rhs, void* output,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Decodes a [rows, k] Q4_K (format 2) or Q6_K (format 3) matrix into f32
 * values [rows, k], bit-identical to ggml's published decode (each element
 * one separately rounded f32 expression).  Format ids follow mote-types'
 * QuantFormat order (Q8_0, Q4_0, Q4_K, Q6_K).  A null pointer or stream,
 * another format or k % 256 != 0 is an invalid value; empty succeeds. */
int mote_cuda_kquant_dequantize_f32(int format, const void* weights, void* output, uint64_t rows,
                                    uint64_t k, void* stream);

/* The f16 linear with a caller workspace (256-byte aligned, zeroed once
 * before first use; its first 256 KiB hold per-tile counters that every call
 * leaves zero, the partial sums come after).  When a launch stages more
 * than 8 activation rows that leave room for only one CTA per SM (9 or more
 * tokens at K = 4096) and N has at most 4096 row tiles, K is split over 2 or
 * 4 CTAs whose partial sums
 * meet in the workspace (added in a fixed order: results do not depend on
 * timing).  On the tensor-core path (more than 16 tokens), the tiles of a
 * partial last wave are split along K instead, their f32 parts stored past
 * the counters and added in part order by a second kernel.  A null or too
 * small workspace gives the unsplit kernels (for either split).  Calls sharing a workspace must
 * not overlap.  No reference counterpart; argument rules as
 * mote_cuda_quantized_linear_q4_0_f16, plus an unaligned workspace -> 1. */
int mote_cuda_quantized_linear_q4_0_f16_ws(const void* input, const void* weights, void* output,
                                           uint64_t rows, uint64_t output_features,
                                           uint64_t input_features, void* workspace,
                                           uint64_t workspace_bytes, void* stream);
/* mote_cuda_quantized_linear_q4_0_f16_ws without a workspace argument, for
 * callers that cannot allocate or pass one (a kernel reached through
 * mote-kernel's KernelImpl::launch gets only its opaque argument words).  No
 * reference counterpart.  The split scratch is a static 8 MiB device array
 * per device, zero at load and left zero by every call; no memory is
 * allocated.  Limits:
 *  - decode shapes (at most 16 tokens per launch): a request whose K split
 *    over CTAs needs more than the scratch returns 10200 before anything is
 *    enqueued -- even where the unsplit kernel would have run;
 *  - prefill shapes (more than 16 tokens, the tensor-core GEMM): a partial
 *    last wave whose K split needs more than the scratch runs unsplit;
 *  - device ordinals of 64 and above return 1;
 *  - calls on the same device must not overlap (one scratch per device,
 *    shared by all streams);
 *  - the first call on a device from a CUDA context (again after a
 *    cudaDeviceReset) looks up the scratch address and must be made before
 *    any stream capture that includes this entry point. */
int mote_cuda_quantized_linear_q4_0_f16_noalloc(const void* input, const void* weights,
                                                void* output, uint64_t rows,
                                                uint64_t output_features, uint64_t input_features,
                                                void* stream);
/* Workspace bytes that allow the widest split for these sizes, on the
 * current device (0: none). */
int mote_cuda_q4_0_linear_workspace_bytes(uint64_t rows, uint64_t output_features,
                                          uint64_t input_features, uint64_t* bytes);

/* Fused FFN gate/up projection with SwiGLU epilogue:
 * output[rows, F] (f16) = silu(input * gate^T) * (input * up^T), with gate and
 * up both Q4_0 [F, K].  No reference counterpart (SwiGLU is named only in
 * docs/architecture.md:191); argument rules as the linear entry points. */
int mote_cuda_q4_0_gate_up_swiglu_f16(const void* input, const void* gate_weights,
                                      const void* up_weights, void* output, uint64_t rows,
                                      uint64_t ffn_features, uint64_t input_features,
                                      void* stream);

/* output[rows, N] = input * weights^T + residual (f16 in, f16 residual and
 * output, f32 accumulation, one rounding).  No reference counterpart: the
 * decoder layer's down projection with its residual add.  output may equal
 * residual.  Null residual -> 1; otherwise the linear entry points' rules. */
int mote_cuda_quantized_linear_q4_0_f16_residual(const void* input, const void* weights,
                                                 const void* residual, void* output,
                                                 uint64_t rows, uint64_t output_features,
                                                 uint64_t input_features, void* stream);

/* Decoder-layer fusions (no reference counterpart: the reference launches
 * rms_norm_f16, crates/mote-backend-hip/src/rms_norm.hip, and the linear
 * separately).  The f16 input rows are RMS-normalised with gamma [K] (f16)
 * and epsilon (finite, >= 0) inside the projection's activation staging --
 * mote-reference's rms_norm_f32 arithmetic, rounded to f16 -- then
 * projected.  Fast-path shapes only: K % 256 == 0, K > 0, 16-byte aligned
 * input, gamma and weights, else 1; rows == 0 or no outputs -> 0 without a
 * launch; rows * N beyond 32 bits -> 9. */
int mote_cuda_q4_0_rms_norm_linear_f16(const void* input, const void* gamma, const void* weights,
                                       void* output, uint64_t rows, uint64_t output_features,
                                       uint64_t input_features, float epsilon, void* stream);
/* ... then gate/up projection with the SwiGLU epilogue. */
int mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16(const void* input, const void* gamma,
                                               const void* gate_weights, const void* up_weights,
                                               void* output, uint64_t rows, uint64_t ffn_features,
                                               uint64_t input_features, float epsilon,
                                               void* stream);
/* ... then the QKV projection [rows, (q_heads + 2 kv_heads) * head_dim] with
 * RoPE (HalfSplit, rotary_dim = head_dim) applied to the q and k heads from
 * the f32 accumulators (one f16 rounding); cos/sin are f32
 * [rows, head_dim/2] as mote_cuda_rope_f16 takes them, 4-byte aligned;
 * head_dim a multiple of 16. */
int mote_cuda_q4_0_rms_norm_qkv_rope_f16(const void* input, const void* gamma, const void* weights,
                                         const void* cos, const void* sin, void* output,
                                         uint64_t rows, uint64_t q_heads, uint64_t kv_heads,
                                         uint64_t head_dim, uint64_t input_features,
                                         float epsilon, void* stream);

/* Decodes Q4_0 [rows, K] to f32, bit-identical to mote-reference's
 * dequantize_quantized_row (crates/mote-reference/src/quantized.rs:58-74). */
int mote_cuda_q4_0_decode_f32(const void* weights, void* output, uint64_t rows,
                              uint64_t input_features, void* stream);

/* Encodes f32 [rows, K] (16-byte aligned) into 2-byte aligned Q4_0 with ggml's reference
 * quantizer rule (d = signed absmax / -8, q = min(15, trunc(x/d + 8.5))).
 * No reference counterpart: the reference builds blocks by hand
 * (crates/mote-reference/tests/quantized_rows.rs:4-8). */
int mote_cuda_q4_0_encode_f32(const void* input, void* weights, uint64_t rows,
                              uint64_t input_features, void* stream);

/* ---------------------------------------------------------------------- */
/* Per-token layer kernels                                                 */
/* ---------------------------------------------------------------------- */

/* Replaces mote_hip_rms_norm_f16 (crates/mote-backend-hip/src/rms_norm.hip:68-98,
 * ffi.rs:126-134).  Row RMSNorm, f16 in/weight/out, f32 math.  Null -> -1;
 * rows or hidden 0 -> 0; rows > 2^32-1 -> -1.  input may equal output. */
int mote_cuda_rms_norm_f16(const void* input, const void* weight, void* output, uint64_t rows,
                           uint64_t hidden_size, float epsilon, void* stream);

/* Replaces mote_hip_fused_add_rms_norm_f16
 * (crates/mote-backend-hip/src/fused_add_rms_norm.hip:99-138, ffi.rs:176-185).
 * sum = input + residual (f32); output = norm(sum) * weight; residual <- f16(sum).
 * Null, non-finite or negative epsilon, or output == residual -> -1. */
int mote_cuda_fused_add_rms_norm_f16(const void* input, void* residual, const void* weight,
                                     void* output, uint64_t rows, uint64_t hidden_size,
                                     float epsilon, void* stream);

/* Replaces mote_hip_rope_f16 (crates/mote-backend-hip/src/rope.hip:99-150,
 * ffi.rs:230-241).  input/output [tokens, heads, head_dim] f16 (may alias),
 * cos/sin [tokens, rotary_dim/2] f32; layout 0 = half-split, 1 = interleaved;
 * the tail after rotary_dim is copied. */
int mote_cuda_rope_f16(const void* input, const void* cos, const void* sin, void* output,
                       uint64_t tokens, uint64_t heads, uint64_t head_dim, uint64_t rotary_dim,
                       uint32_t layout, void* stream);

/* Fused per-token layer kernel (no reference counterpart; composes the two
 * entry points above): x_out = rms_norm(x) * gamma over [tokens, hidden], and
 * q_out / k_out = RoPE of q [tokens, q_heads, head_dim] and
 * k [tokens, kv_heads, head_dim] with rotary_dim == head_dim, in one launch. */
int mote_cuda_rms_norm_rope_f16(const void* x, const void* gamma, void* x_out, const void* q,
                                void* q_out, const void* k, void* k_out, const void* cos,
                                const void* sin, uint64_t tokens, uint64_t hidden,
                                uint64_t q_heads, uint64_t kv_heads, uint64_t head_dim,
                                uint32_t layout, float epsilon, void* stream);

/* out = silu(gate) * up, f16, silu(g) = g / (1 + exp(-g)) in f32.  No
 * reference counterpart (docs/architecture.md:191 names the op). */
int mote_cuda_swiglu_f16(const void* gate, const void* up, void* output, uint64_t n,
                         void* stream);

/* out[t, :] = table[ids[t], :] (f16, bit-exact); ids are int32.  Ids outside
 * [0, vocab) produce a zero row and OR 2 into *error_flag (a device uint32 the
 * caller zeroes and reads).  No reference counterpart. */
int mote_cuda_embedding_gather_f16(const void* table, const void* ids, void* output,
                                   uint64_t tokens, uint64_t vocab, uint64_t hidden,
                                   void* error_flag, void* stream);

/* cos/sin tables [tokens, rotary_dim/2] f32 for RoPE:
 * angle = positions[t] * theta^(-2j/rotary_dim) in f64, rounded once.  The
 * reference takes these tables as inputs (crates/mote-backend-hip/src/rope.rs:66-82)
 * and has no generator. */
int mote_cuda_rope_cos_sin_f32(const void* positions, void* cos_out, void* sin_out,
                               uint64_t tokens, uint64_t rotary_dim, double theta,
                               void* stream);

/* ---- persistent decoder stack ---------------------------------------------
 * The non-attention ops of num_layers Llama-style decoder layers at one token
 * in ONE cooperative kernel launch (grid barriers in place of kernel
 * boundaries; each warp's weight stream runs ahead across them).  No reference
 * counterpart (the reference composes the operators launch by launch,
 * docs/architecture.md:180-192).  Per layer l, with h = h_in for l == 0 and
 * the previous layer's `out` after:
 *   qkv = rope(rms_norm(h, gamma1) @ w_qkv^T)     (HalfSplit, rotary = head_dim)
 *   h1  = h + attn @ w_o^T
 *   a   = silu(rms_norm(h1, gamma2) @ w_gate^T) * (rms_norm(h1, gamma2) @ w_up^T)
 *   out = h1 + a @ w_down^T
 * Weights Q4_0 [rows, in/32*18]; f16 vectors; cos/sin f32 [head_dim/2] of the
 * token's position.  `layers` is a DEVICE array of num_layers descriptors;
 * `workspace` (256-byte aligned) holds the grid-barrier words and the down
 * projection's partial sums: mote_cuda_q4_0_decoder_stack_workspace_bytes
 * bytes (its first 256 are zeroed by the call).  hidden and ffn
 * multiples of 256, head_dim a multiple of 16, q_heads a multiple of
 * kv_heads, 16-byte aligned tensors (cos/sin 4-byte); eps finite and >= 0;
 * otherwise 1.  A bounded grid-barrier wait that expires sets bit 1 of the
 * device status. */
typedef struct mote_cuda_stack_layer {
    const void* w_qkv;
    const void* w_o;
    const void* w_gate;
    const void* w_up;
    const void* w_down;
    const void* gamma1;
    const void* gamma2;
    const void* attn;
    const void* cos;
    const void* sin;
    void* qkv;
    void* h1;
    void* a;
    void* out;
} mote_cuda_stack_layer;
int mote_cuda_q4_0_decoder_stack_workspace_bytes(uint64_t hidden, uint64_t* bytes);
int mote_cuda_q4_0_decoder_stack_f16(const void* layers, uint32_t num_layers, const void* h_in,
                                     uint64_t hidden, uint64_t ffn, uint64_t q_heads,
                                     uint64_t kv_heads, uint64_t head_dim, float epsilon,
                                     void* workspace, uint64_t workspace_bytes, void* stream);

/* ---- grouped-query attention over a KV cache ----------------------------
 * No reference counterpart: the reference lists attention (GQA) with KV-cache
 * append and KV-cache operations as planned primitives (docs/roadmap.md:58-60,
 * docs/architecture.md:185-191) and ships none.  f16 tensors, head_dim
 * innermost: caches [cache_rows, kv_heads, head_dim]; a batch of sequences
 * keeps sequence b at rows b * seq_capacity + position.
 *
 * KV-cache append: k_new / v_new [tokens, kv_heads, head_dim] into cache row
 * slots[t] (int32); a slot outside [0, cache_rows) is skipped and sets
 * *error_flag (uint32, optional) to 1.  kv_heads * head_dim % 8 == 0, 16-byte
 * aligned tensors; tokens == 0 returns 0; null pointers -> 1. */
int mote_cuda_kv_cache_append_f16(const void* k_new, const void* v_new, void* k_cache,
                                  void* v_cache, const void* slots, uint64_t tokens,
                                  uint64_t kv_heads, uint64_t head_dim, uint64_t cache_rows,
                                  void* error_flag, void* stream);
/* Decode attention, one query token per sequence:
 *   out[b, h] = softmax(scale * q[b, h] . K_b[:len_b, h / (q_heads / kv_heads)]) . V_b
 * q / out [batch, q_heads, head_dim]; seq_lens int32 [batch] on the device,
 * len_b = min(seq_lens[b], max_len), max_len <= seq_capacity; a sequence of
 * length 0 gets zeros.  q_heads % kv_heads == 0, head_dim 64 or 128,
 * 16-byte aligned tensors.  Splits the
 * positions over CTAs, which merge their parts inside a thread-block cluster
 * (up to 8 parts) or in a second kernel: workspace of
 * mote_cuda_gqa_attention_decode_workspace_bytes bytes (16-byte aligned; 0
 * means none is needed; contents need no initialisation).  Other shapes or a
 * missing workspace -> 1. */
int mote_cuda_gqa_attention_decode_workspace_bytes(uint64_t batch, uint64_t q_heads,
                                                   uint64_t kv_heads, uint64_t head_dim,
                                                   uint64_t max_len, uint64_t* bytes);
int mote_cuda_gqa_attention_decode_f16(const void* q, const void* k_cache, const void* v_cache,
                                       const void* seq_lens, void* out, uint64_t batch,
                                       uint64_t q_heads, uint64_t kv_heads, uint64_t head_dim,
                                       uint64_t seq_capacity, uint64_t max_len, float scale,
                                       void* workspace, uint64_t workspace_bytes, void* stream);
/* Causal prefill attention on the tensor cores (tcgen05): `tokens` queries at
 * positions start .. start + tokens - 1 of one sequence,
 *   out[t, h] = softmax_{p <= start + t}(scale * q[t, h] . K[p, h / g]) . V[p, h / g],
 * q / out [tokens, q_heads, head_dim] f16, K/V from cache rows row0 + p for
 * p < start + tokens (this chunk's K/V already appended; row0 + start +
 * tokens <= cache_rows).  head_dim 64, q_heads % kv_heads == 0, scale > 0,
 * 16-byte aligned tensors; tokens == 0 returns 0; other shapes -> 1. */
int mote_cuda_gqa_attention_prefill_f16(const void* q, const void* k_cache, const void* v_cache,
                                        void* out, uint64_t tokens, uint64_t start,
                                        uint64_t q_heads, uint64_t kv_heads, uint64_t head_dim,
                                        uint64_t row0, uint64_t cache_rows, float scale,
                                        void* stream);

/* ---- multi-GPU exchange for column-sharded linears ----------------------
 * The reference is single-device (crates/mote-backend-hip/src/context.rs:13-80
 * holds one device and one stream); these entry points are new.  Each rank
 * computes y_g = x @ W_g^T for its contiguous slice W_g of the weight rows;
 * the all-gathers below deliver every slice to every rank, rank-major
 * ([nranks][count] f16).
 *
 * NCCL transport (libnccl.so.2 is loaded on first use; status 10000 if it is
 * absent, 10100 + ncclResult_t on an NCCL failure).  id is 128 bytes. */
int mote_cuda_comm_unique_id(void* id_out);
int mote_cuda_comm_init(void** comm, int nranks, const void* id, int rank);
/* Nonblocking init with a deadline: if not every rank has joined within
 * timeout_ms, the communicator is aborted and 10001 returned (*comm null),
 * so a rank that never arrives cannot block the host for good.  The
 * communicator stays nonblocking: its all-gathers are polled against the same
 * limit (10001 and an aborted communicator past it), and destroy releases it
 * with the NCCL abort. */
int mote_cuda_comm_init_timeout(void** comm, int nranks, const void* id, int rank,
                                uint64_t timeout_ms);
int mote_cuda_comm_all_gather_f16(void* comm, const void* send, void* recv, uint64_t count,
                                  void* stream);
int mote_cuda_comm_destroy(void* comm);
/* Aborts a communicator (no barrier with the other ranks) and frees it. */
int mote_cuda_comm_abort(void* comm);

/* Peer-store transport over NVLink.  Buffers are shared with CUDA IPC
 * handles (64 bytes): every rank exports its receive buffer and its flag
 * array (nranks + 2 uint32 words, zeroed once before first use) and opens
 * the others'.  recv_ptrs and flag_ptrs are DEVICE arrays of nranks
 * pointers (this rank's own buffers at index rank).  One launch stores this
 * rank's slice into every receive buffer at offset rank * count, advances
 * this rank's epoch (kept in its flag array, so graph replays work),
 * publishes it in every flag array and waits (bounded; on timeout bit 1 of
 * the device status is set) until every rank has published it.  A receive
 * buffer must not be overwritten while a rank still reads the previous
 * gather from it.  count is a multiple of 8, send 16-byte aligned. */
int mote_cuda_ipc_get_handle(const void* dev_ptr, void* handle_out);
int mote_cuda_ipc_open_handle(const void* handle, void** dev_ptr);
int mote_cuda_ipc_close_handle(void* dev_ptr);
int mote_cuda_all_gather_p2p_f16(const void* send, void* const* recv_ptrs,
                                 unsigned* const* flag_ptrs, unsigned* own_flags,
                                 uint64_t count, uint32_t rank, uint32_t nranks, void* stream);
/* The same all-gather with its flag wait limited to wait_ns nanoseconds
 * (the entry above waits up to 1 s); wait_ns == 0 -> 1.  On expiry bit 1 of
 * the device status is set and the kernel returns. */
int mote_cuda_all_gather_p2p_f16_timeout(const void* send, void* const* recv_ptrs,
                                         unsigned* const* flag_ptrs, unsigned* own_flags,
                                         uint64_t count, uint32_t rank, uint32_t nranks,
                                         uint64_t wait_ns, void* stream);
/* Resynchronisation after an expired wait: zeroes this rank's flag array
 * (nranks + 2 words) on `stream`.  Every rank calls it, with no exchange in
 * flight on any rank, between two host barriers; the epochs then restart
 * together. */
int mote_cuda_peer_flags_reset(unsigned* own_flags, uint32_t nranks, void* stream);

/* Column-sharded Q4_0 linear with the all-gather fused into the epilogue:
 * `weights` holds this rank's rows [rank*shard, rank*shard + shard) of the
 * full [total_features, K] matrix (rows past total_features are padding and
 * never stored); the f16 results go straight into every rank's full output
 * buffer [rows, total_features] at columns rank*shard.. (outputs: DEVICE
 * array of nranks pointers, peers mapped over CUDA IPC), then the flag
 * handshake of mote_cuda_all_gather_p2p_f16 runs at the end of the grid, so
 * when the launch completes every rank holds all columns.  More than 16
 * tokens run on the tensor-core GEMM with the same epilogue and handshake
 * (a rank whose shard has no real rows only joins the handshake).
 * shard % 16 == 0,
 * total_features % 8 == 0, K % 256 == 0 and K > 0, 16-byte aligned input,
 * weights and output buffers; every rank
 * passes the same rows (rows == 0 returns 0 without a launch on all ranks).
 * Null pointers, rank >= nranks or other shapes -> 1. */
int mote_cuda_quantized_linear_q4_0_f16_allgather(const void* input, const void* weights,
                                                  void* const* outputs, unsigned* const* flag_ptrs,
                                                  unsigned* own_flags, uint64_t rows,
                                                  uint64_t shard_features, uint64_t input_features,
                                                  uint64_t total_features, uint32_t rank,
                                                  uint32_t nranks, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOTE_CUDA_H */
