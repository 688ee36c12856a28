/*
 * mote_oracle.h -- CPU oracle for the Mote Q4_0 / per-token layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA data
 * plane is compared against; nothing in the product (mote_b200/, include/)
 * links, loads or calls it.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py use it.
 *
 * What it is: a C restatement of the pure-Rust `mote-reference` crate of
 * RiversJin/mote, which cannot be compiled here (no cargo/rustc).  Every
 * function keeps the reference's loop nesting and its f32 operation order,
 * and the library is compiled with -O2 -ffp-contract=off and no fast-math,
 * so on x86-64 (SSE f32 arithmetic) its results are bit-identical to the
 * Rust oracle.  Parity is pinned by the known-answer tests that the
 * reference's own test files hold (transcribed into tests/golden/).
 *
 * Functions that have no counterpart in mote-reference (Q4_0 encoder,
 * embedding gather, SwiGLU, RoPE cos/sin table) restate the math given in
 * the path's specification; their parity with the reference is unpinned
 * because the reference has no such operator.
 */
#ifndef MOTE_ORACLE_H
#define MOTE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Quantization formats, in the order of `mote_types::QuantFormat`
 * (crates/mote-types/src/lib.rs:39-45). */
enum oracle_quant_format {
    ORACLE_Q8_0 = 0,
    ORACLE_Q4_0 = 1,
    ORACLE_Q4_K = 2,
    ORACLE_Q6_K = 3,
};

/* RoPE pairing, `mote_types::RopeLayout` (crates/mote-types/src/lib.rs:82-89). */
enum oracle_rope_layout {
    ORACLE_ROPE_HALF_SPLIT = 0,
    ORACLE_ROPE_INTERLEAVED = 1,
};

/* Error taxonomy.  Each value names one variant of the reference's error
 * enums; `oracle_error.a/b/c` carry that variant's fields in declaration
 * order (e.g. expected, actual). */
enum oracle_status {
    ORACLE_OK = 0,
    /* QuantizedLinearError (crates/mote-reference/src/quantized.rs:7-44) */
    ORACLE_QL_UNSUPPORTED_FORMAT = 1,      /* a = format */
    ORACLE_QL_ROW_MISALIGNED = 2,          /* a = format, b = row_elements, c = block_elements */
    ORACLE_QL_DIMENSIONS_OVERFLOW = 3,     /* a = rows, b = output_features, c = input_features */
    ORACLE_QL_INPUT_LENGTH_MISMATCH = 4,   /* a = expected, b = actual */
    ORACLE_QL_WEIGHT_LENGTH_MISMATCH = 5,  /* a = expected, b = actual */
    ORACLE_QL_ROW_BYTE_LENGTH_MISMATCH = 6,/* a = expected, b = actual */
    /* ReferenceError (crates/mote-reference/src/lib.rs:19-58) */
    ORACLE_REF_ZERO_HIDDEN_SIZE = 10,
    ORACLE_REF_WEIGHT_LENGTH_MISMATCH = 11, /* a = weight_len, b = hidden_size */
    ORACLE_REF_INPUT_NOT_MULTIPLE = 12,     /* a = input_len, b = hidden_size */
    ORACLE_REF_RESIDUAL_LENGTH_MISMATCH = 13,/* a = residual_len, b = input_len */
    ORACLE_REF_INVALID_EPSILON = 14,
    /* RopeError (crates/mote-reference/src/lib.rs:77-103) */
    ORACLE_ROPE_ODD_ROTARY_DIMENSION = 20,  /* a = rotary_dim */
    ORACLE_ROPE_ROTARY_TOO_LARGE = 21,      /* a = rotary_dim, b = head_dim */
    ORACLE_ROPE_DIMENSIONS_OVERFLOW = 22,
    ORACLE_ROPE_INPUT_LENGTH_MISMATCH = 23, /* a = expected, b = actual */
    ORACLE_ROPE_COS_LENGTH_MISMATCH = 24,   /* a = expected, b = actual */
    ORACLE_ROPE_SIN_LENGTH_MISMATCH = 25,   /* a = expected, b = actual */
    /* MatmulError (crates/mote-reference/src/lib.rs:61-74) */
    ORACLE_MM_DIMENSIONS_OVERFLOW = 30,
    ORACLE_MM_LHS_LENGTH_MISMATCH = 31,     /* a = expected, b = actual */
    ORACLE_MM_RHS_LENGTH_MISMATCH = 32,     /* a = expected, b = actual */
    /* New operators (no reference counterpart). */
    ORACLE_ARGUMENT_INVALID = 40,
};

typedef struct oracle_error {
    uint64_t a, b, c;
} oracle_error;

/* ---- IEEE binary16 conversions (`half` 2.7.1 semantics: exact widening,
 * round-to-nearest-even narrowing) ---- */
float oracle_f16_to_f32(uint16_t bits);
uint16_t oracle_f32_to_f16(float value);
void oracle_f16_to_f32_array(const uint16_t* in, float* out, size_t n);
void oracle_f32_to_f16_array(const float* in, uint16_t* out, size_t n);

/* ---- mote-reference restatements ---- */

/* Geometry of a format: elements and bytes per block
 * (crates/mote-types/src/lib.rs:48-74). */
size_t oracle_block_elements(int format);
size_t oracle_block_bytes(int format);

/* dequantize_quantized_row, crates/mote-reference/src/quantized.rs:58-74.
 * `output` must hold `row_elements` floats. */
int oracle_dequantize_quantized_row(const uint8_t* bytes, size_t bytes_len, int format,
                                    size_t row_elements, float* output, oracle_error* err);

/* quantized_linear_f32, crates/mote-reference/src/quantized.rs:89-144.
 * `output` must hold rows*output_features floats. */
int oracle_quantized_linear_f32(const float* input, size_t input_len, const uint8_t* weights,
                                size_t weights_len, int format, size_t rows,
                                size_t output_features, size_t input_features, float* output,
                                oracle_error* err);

/* The same computation with the output features partitioned over `threads`
 * POSIX threads.  Every output element is produced by exactly the code path
 * of oracle_quantized_linear_f32, so the results are bit-identical; only the
 * wall time changes.  Used as the multi-core CPU baseline. */
int oracle_quantized_linear_f32_mt(const float* input, size_t input_len, const uint8_t* weights,
                                   size_t weights_len, int format, size_t rows,
                                   size_t output_features, size_t input_features, float* output,
                                   int threads, oracle_error* err);

/* matmul_f32, crates/mote-reference/src/lib.rs:116-156. */
int oracle_matmul_f32(const float* lhs, size_t lhs_len, const float* rhs, size_t rhs_len,
                      size_t m, size_t n, size_t k, float* output, oracle_error* err);

/* rope_f32, crates/mote-reference/src/lib.rs:170-244. */
int oracle_rope_f32(const float* input, size_t input_len, const float* cos, size_t cos_len,
                    const float* sin, size_t sin_len, size_t tokens, size_t heads,
                    size_t head_dim, size_t rotary_dim, int layout, float* output,
                    oracle_error* err);

/* rms_norm_f32, crates/mote-reference/src/lib.rs:262-301. */
int oracle_rms_norm_f32(const float* input, size_t input_len, const float* weight,
                        size_t weight_len, size_t hidden_size, float epsilon, float* output,
                        oracle_error* err);

/* fused_add_rms_norm_f32, crates/mote-reference/src/lib.rs:333-384.
 * `normalized` and `residual_out` each hold input_len floats. */
int oracle_fused_add_rms_norm_f32(const float* input, size_t input_len, const float* residual,
                                  size_t residual_len, const float* weight, size_t weight_len,
                                  size_t hidden_size, float epsilon, float* normalized,
                                  float* residual_out, oracle_error* err);

/* ---- New operators (math restated from the path's specification) ---- */

/* Q4_0 encoder for one row of `k` floats (k % 32 == 0) into k/32 18-byte
 * blocks.  Restates ggml's published reference quantizer for Q4_0
 * (quantize_row_q4_0_ref in ggml-quants.c; ggml is not vendored in the
 * reference): per block, the signed element of largest magnitude m gives
 * d = m / -8; the stored scale is f16(d); each element becomes
 * min(15, trunc(x * (1/d) + 8.5)), low nibble for element j, high nibble
 * for element j+16. */
int oracle_q4_0_quantize_rows(const float* input, size_t rows, size_t k, uint8_t* output);

/* out[t, :] = table[ids[t], :] for f16 rows; ids outside [0, vocab) produce
 * a zero row and set *out_of_range to 1. */
int oracle_embedding_gather_f16(const uint16_t* table, size_t vocab, size_t hidden,
                                const int32_t* ids, size_t tokens, uint16_t* output,
                                uint32_t* out_of_range);

/* out = silu(g) * u with silu(g) = g / (1 + exp(-g)), evaluated in f64 and
 * rounded once to f32. */
void oracle_swiglu_f64(const float* gate, const float* up, size_t n, float* output);

/* cos/sin tables [tokens, rotary_dim/2]: angle = positions[t] *
 * theta^(-2j/rotary_dim), evaluated in f64 and rounded once to f32. */
int oracle_rope_cos_sin_f64(const int32_t* positions, size_t tokens, size_t rotary_dim,
                            double theta, float* cos_out, float* sin_out);

/*
 * K-quant super-blocks (Q4_K, Q6_K; 256 elements).  mote-reference rejects
 * these formats (crates/mote-reference/src/quantized.rs:152-157) and only
 * fixes their geometry (crates/mote-types/src/lib.rs:41-74), so these
 * functions restate the published ggml algorithm as the gguf Python package,
 * version 0.19.0, implements it (gguf/quants.py, Q4_K.dequantize_blocks and
 * Q6_K.dequantize_blocks): every element is one f32 expression,
 *   Q4_K: (d * sc) * q - (dmin * m),  q in 0..15, sc/m 6-bit per 32 elements;
 *   Q6_K: (d * sc) * q,               q in -32..31, sc int8 per 16 elements.
 * Parity is pinned by golden vectors that gguf 0.19.0 produced
 * (tests/golden/kquant_golden.npz, made by tests/golden/make_kquant_golden.py).
 */
int oracle_kquant_dequantize_row(const uint8_t* bytes, size_t bytes_len, int format,
                                 size_t row_elements, float* output);

/* Y[rows, n] = X[rows, k] . W[n, k]^T with W decoded as above (f32 values)
 * and every dot product accumulated in f64: the tolerance reference of the
 * K-quant linear. */
int oracle_kquant_linear_f64(const float* input, const uint8_t* weights, int format, size_t rows,
                             size_t n, size_t k, double* output);

#ifdef __cplusplus
}
#endif

#endif /* MOTE_ORACLE_H */
