/*
 * mote_oracle.c -- CPU oracle (test infrastructure only; see mote_oracle.h).
 *
 * Compile with -O2 -ffp-contract=off and without -ffast-math: the reference
 * Rust oracle never contracts a*b+c into an FMA and never reassociates, and
 * neither may this restatement if it is to stay bit-identical.
 */
#include "mote_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static void set_err(oracle_error* err, uint64_t a, uint64_t b, uint64_t c) {
    if (err) {
        err->a = a;
        err->b = b;
        err->c = c;
    }
}

/* ------------------------------------------------------------------------ */
/* binary16 <-> binary32                                                     */
/* ------------------------------------------------------------------------ */

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        /* zero or subnormal: man * 2^-24 is exact in f32 */
        float v = (float)man * 0x1p-24f;
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (exp == 0x1F) {
        bits = man == 0 ? (sign | 0x7F800000u) : (sign | 0x7FC00000u | (man << 13));
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

uint16_t oracle_f32_to_f16(float value) {
    uint32_t x;
    memcpy(&x, &value, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) {
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    const int32_t e = (int32_t)exp - 112; /* f16 biased exponent */
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        /* result is subnormal (or rounds up to the smallest normal) */
        const int shift = 14 - e; /* right shift of the 24-bit significand */
        if (shift > 24) return (uint16_t)sign;
        const uint32_t full = man | 0x800000u;
        uint32_t m = full >> shift;
        const uint32_t rem = full & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t out = sign | ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (out & 1u))) out++;
    return (uint16_t)out;
}

void oracle_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = oracle_f16_to_f32(in[i]);
}

void oracle_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = oracle_f32_to_f16(in[i]);
}

/* ------------------------------------------------------------------------ */
/* Block geometry: crates/mote-types/src/lib.rs:48-74                        */
/* ------------------------------------------------------------------------ */

size_t oracle_block_elements(int format) {
    switch (format) {
        case ORACLE_Q4_0:
        case ORACLE_Q8_0: return 32;
        case ORACLE_Q4_K:
        case ORACLE_Q6_K: return 256;
        default: return 0;
    }
}

size_t oracle_block_bytes(int format) {
    switch (format) {
        case ORACLE_Q4_0: return 18;
        case ORACLE_Q8_0: return 34;
        case ORACLE_Q4_K: return 144;
        case ORACLE_Q6_K: return 210;
        default: return 0;
    }
}

/* checked_row_bytes, crates/mote-reference/src/quantized.rs:146-175 */
static int checked_row_bytes(int format, size_t row_elements, size_t rows,
                             size_t output_features, size_t* row_bytes, oracle_error* err) {
    if (format != ORACLE_Q4_0 && format != ORACLE_Q8_0) {
        set_err(err, (uint64_t)format, 0, 0);
        return ORACLE_QL_UNSUPPORTED_FORMAT;
    }
    const size_t block_elements = oracle_block_elements(format);
    if (row_elements % block_elements != 0) {
        set_err(err, (uint64_t)format, row_elements, block_elements);
        return ORACLE_QL_ROW_MISALIGNED;
    }
    if (__builtin_mul_overflow(row_elements / block_elements, oracle_block_bytes(format),
                               row_bytes)) {
        set_err(err, rows, output_features, row_elements);
        return ORACLE_QL_DIMENSIONS_OVERFLOW;
    }
    return ORACLE_OK;
}

/* decode_row_into, crates/mote-reference/src/quantized.rs:177-201 */
static void decode_row_into(const uint8_t* bytes, size_t row_bytes, int format, float* output) {
    const size_t block_elements = oracle_block_elements(format);
    const size_t block_bytes = oracle_block_bytes(format);
    const size_t blocks = row_bytes / block_bytes;
    for (size_t b = 0; b < blocks; b++) {
        const uint8_t* block = bytes + b * block_bytes;
        const float scale = oracle_f16_to_f32((uint16_t)(block[0] | (block[1] << 8)));
        const size_t start = b * block_elements;
        if (format == ORACLE_Q4_0) {
            for (size_t j = 0; j < 16; j++) {
                const uint8_t quants = block[2 + j];
                output[start + j] = (float)((int8_t)(quants & 0x0F) - 8) * scale;
                output[start + j + 16] = (float)((int8_t)(quants >> 4) - 8) * scale;
            }
        } else { /* Q8_0 */
            for (size_t j = 0; j < 32; j++) {
                output[start + j] = (float)(int8_t)block[2 + j] * scale;
            }
        }
    }
}

int oracle_dequantize_quantized_row(const uint8_t* bytes, size_t bytes_len, int format,
                                    size_t row_elements, float* output, oracle_error* err) {
    size_t row_bytes = 0;
    int status = checked_row_bytes(format, row_elements, 1, 1, &row_bytes, err);
    if (status != ORACLE_OK) return status;
    if (bytes_len != row_bytes) {
        set_err(err, row_bytes, bytes_len, 0);
        return ORACLE_QL_ROW_BYTE_LENGTH_MISMATCH;
    }
    for (size_t i = 0; i < row_elements; i++) output[i] = 0.0f;
    decode_row_into(bytes, row_bytes, format, output);
    return ORACLE_OK;
}

/* Validation half of quantized_linear_f32 (quantized.rs:89-125). */
static int validate_linear(size_t input_len, size_t weights_len, int format, size_t rows,
                           size_t output_features, size_t input_features, size_t* row_bytes,
                           size_t* output_len, oracle_error* err) {
    int status = checked_row_bytes(format, input_features, rows, output_features, row_bytes, err);
    if (status != ORACLE_OK) return status;
    size_t in_len, w_len, out_len;
    if (__builtin_mul_overflow(rows, input_features, &in_len) ||
        __builtin_mul_overflow(output_features, *row_bytes, &w_len) ||
        __builtin_mul_overflow(rows, output_features, &out_len)) {
        set_err(err, rows, output_features, input_features);
        return ORACLE_QL_DIMENSIONS_OVERFLOW;
    }
    if (input_len != in_len) {
        set_err(err, in_len, input_len, 0);
        return ORACLE_QL_INPUT_LENGTH_MISMATCH;
    }
    if (weights_len != w_len) {
        set_err(err, w_len, weights_len, 0);
        return ORACLE_QL_WEIGHT_LENGTH_MISMATCH;
    }
    *output_len = out_len;
    return ORACLE_OK;
}

/* Hot loop of quantized_linear_f32 (quantized.rs:127-142) over output
 * features [f0, f1): decode the weight row once, then one sequential f32
 * dot product per input row. */
static void linear_features(const float* input, const uint8_t* weights, int format, size_t rows,
                            size_t output_features, size_t input_features, size_t row_bytes,
                            size_t f0, size_t f1, float* decoded, float* output) {
    for (size_t of = f0; of < f1; of++) {
        decode_row_into(weights + of * row_bytes, row_bytes, format, decoded);
        for (size_t row = 0; row < rows; row++) {
            const float* in = input + row * input_features;
            float sum = 0.0f;
            for (size_t inner = 0; inner < input_features; inner++) {
                sum += in[inner] * decoded[inner];
            }
            output[row * output_features + of] = sum;
        }
    }
}

int oracle_quantized_linear_f32(const float* input, size_t input_len, const uint8_t* weights,
                                size_t weights_len, int format, size_t rows,
                                size_t output_features, size_t input_features, float* output,
                                oracle_error* err) {
    size_t row_bytes = 0, output_len = 0;
    int status = validate_linear(input_len, weights_len, format, rows, output_features,
                                 input_features, &row_bytes, &output_len, err);
    if (status != ORACLE_OK) return status;
    if (output_len == 0) return ORACLE_OK;
    float* decoded = (float*)malloc((input_features ? input_features : 1) * sizeof(float));
    if (!decoded) return ORACLE_ARGUMENT_INVALID;
    linear_features(input, weights, format, rows, output_features, input_features, row_bytes, 0,
                    output_features, decoded, output);
    free(decoded);
    return ORACLE_OK;
}

typedef struct {
    const float* input;
    const uint8_t* weights;
    int format;
    size_t rows, output_features, input_features, row_bytes, f0, f1;
    float* output;
} linear_job;

static void* linear_worker(void* arg) {
    linear_job* job = (linear_job*)arg;
    float* decoded = (float*)malloc((job->input_features ? job->input_features : 1) * sizeof(float));
    if (!decoded) return NULL;
    linear_features(job->input, job->weights, job->format, job->rows, job->output_features,
                    job->input_features, job->row_bytes, job->f0, job->f1, decoded, job->output);
    free(decoded);
    return NULL;
}

int oracle_quantized_linear_f32_mt(const float* input, size_t input_len, const uint8_t* weights,
                                   size_t weights_len, int format, size_t rows,
                                   size_t output_features, size_t input_features, float* output,
                                   int threads, oracle_error* err) {
    size_t row_bytes = 0, output_len = 0;
    int status = validate_linear(input_len, weights_len, format, rows, output_features,
                                 input_features, &row_bytes, &output_len, err);
    if (status != ORACLE_OK) return status;
    if (output_len == 0) return ORACLE_OK;
    if (threads < 1) threads = 1;
    if ((size_t)threads > output_features) threads = (int)output_features;
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    linear_job* jobs = (linear_job*)calloc((size_t)threads, sizeof(linear_job));
    if (!tids || !jobs) {
        free(tids);
        free(jobs);
        return ORACLE_ARGUMENT_INVALID;
    }
    for (int t = 0; t < threads; t++) {
        jobs[t] = (linear_job){input, weights, format, rows, output_features, input_features,
                               row_bytes, output_features * (size_t)t / (size_t)threads,
                               output_features * (size_t)(t + 1) / (size_t)threads, output};
        pthread_create(&tids[t], NULL, linear_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; t++) pthread_join(tids[t], NULL);
    free(tids);
    free(jobs);
    return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* matmul_f32, crates/mote-reference/src/lib.rs:116-156                      */
/* ------------------------------------------------------------------------ */

int oracle_matmul_f32(const float* lhs, size_t lhs_len, const float* rhs, size_t rhs_len,
                      size_t m, size_t n, size_t k, float* output, oracle_error* err) {
    size_t l_len, r_len, o_len;
    if (__builtin_mul_overflow(m, k, &l_len) || __builtin_mul_overflow(k, n, &r_len) ||
        __builtin_mul_overflow(m, n, &o_len)) {
        set_err(err, m, n, k);
        return ORACLE_MM_DIMENSIONS_OVERFLOW;
    }
    if (lhs_len != l_len) {
        set_err(err, l_len, lhs_len, 0);
        return ORACLE_MM_LHS_LENGTH_MISMATCH;
    }
    if (rhs_len != r_len) {
        set_err(err, r_len, rhs_len, 0);
        return ORACLE_MM_RHS_LENGTH_MISMATCH;
    }
    for (size_t i = 0; i < o_len; i++) output[i] = 0.0f;
    for (size_t row = 0; row < m; row++) {
        for (size_t inner = 0; inner < k; inner++) {
            const float lhs_value = lhs[row * k + inner];
            for (size_t col = 0; col < n; col++) {
                output[row * n + col] += lhs_value * rhs[inner * n + col];
            }
        }
    }
    return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* rope_f32, crates/mote-reference/src/lib.rs:170-244                        */
/* ------------------------------------------------------------------------ */

int oracle_rope_f32(const float* input, size_t input_len, const float* cos, size_t cos_len,
                    const float* sin, size_t sin_len, size_t tokens, size_t heads,
                    size_t head_dim, size_t rotary_dim, int layout, float* output,
                    oracle_error* err) {
    if (rotary_dim % 2 != 0) {
        set_err(err, rotary_dim, 0, 0);
        return ORACLE_ROPE_ODD_ROTARY_DIMENSION;
    }
    if (rotary_dim > head_dim) {
        set_err(err, rotary_dim, head_dim, 0);
        return ORACLE_ROPE_ROTARY_TOO_LARGE;
    }
    size_t rows, in_len, cache_len;
    const size_t frequency_count = rotary_dim / 2;
    if (__builtin_mul_overflow(tokens, heads, &rows) ||
        __builtin_mul_overflow(rows, head_dim, &in_len) ||
        __builtin_mul_overflow(tokens, frequency_count, &cache_len)) {
        set_err(err, tokens, heads, head_dim);
        return ORACLE_ROPE_DIMENSIONS_OVERFLOW;
    }
    if (input_len != in_len) {
        set_err(err, in_len, input_len, 0);
        return ORACLE_ROPE_INPUT_LENGTH_MISMATCH;
    }
    if (cos_len != cache_len) {
        set_err(err, cache_len, cos_len, 0);
        return ORACLE_ROPE_COS_LENGTH_MISMATCH;
    }
    if (sin_len != cache_len) {
        set_err(err, cache_len, sin_len, 0);
        return ORACLE_ROPE_SIN_LENGTH_MISMATCH;
    }
    for (size_t i = 0; i < input_len; i++) output[i] = input[i];
    for (size_t token = 0; token < tokens; token++) {
        const size_t cache_offset = token * frequency_count;
        for (size_t head = 0; head < heads; head++) {
            const size_t row_offset = (token * heads + head) * head_dim;
            for (size_t pair = 0; pair < frequency_count; pair++) {
                size_t first, second;
                if (layout == ORACLE_ROPE_HALF_SPLIT) {
                    first = pair;
                    second = pair + frequency_count;
                } else {
                    first = pair * 2;
                    second = pair * 2 + 1;
                }
                const float first_value = input[row_offset + first];
                const float second_value = input[row_offset + second];
                const float cosine = cos[cache_offset + pair];
                const float sine = sin[cache_offset + pair];
                output[row_offset + first] = first_value * cosine - second_value * sine;
                output[row_offset + second] = second_value * cosine + first_value * sine;
            }
        }
    }
    return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* rms_norm_f32 / fused_add_rms_norm_f32, crates/mote-reference/src/lib.rs   */
/* ------------------------------------------------------------------------ */

static int validate_norm(size_t input_len, size_t weight_len, size_t hidden_size,
                         float epsilon, oracle_error* err) {
    if (hidden_size == 0) return ORACLE_REF_ZERO_HIDDEN_SIZE;
    if (weight_len != hidden_size) {
        set_err(err, weight_len, hidden_size, 0);
        return ORACLE_REF_WEIGHT_LENGTH_MISMATCH;
    }
    if (input_len % hidden_size != 0) {
        set_err(err, input_len, hidden_size, 0);
        return ORACLE_REF_INPUT_NOT_MULTIPLE;
    }
    if (!isfinite(epsilon) || epsilon < 0.0f) return ORACLE_REF_INVALID_EPSILON;
    return ORACLE_OK;
}

/* lib.rs:288-299: sequential f32 sum of squares, mean, 1/sqrt, then
 * x * inv_rms * w evaluated left to right. */
static void norm_rows(const float* rows_in, size_t input_len, const float* weight,
                      size_t hidden_size, float epsilon, float* output) {
    for (size_t start = 0; start < input_len; start += hidden_size) {
        const float* row = rows_in + start;
        float sum_sq = 0.0f;
        for (size_t i = 0; i < hidden_size; i++) sum_sq += row[i] * row[i];
        const float mean_square = sum_sq / (float)hidden_size;
        const float inv_rms = 1.0f / sqrtf(mean_square + epsilon);
        for (size_t i = 0; i < hidden_size; i++) output[start + i] = row[i] * inv_rms * weight[i];
    }
}

int oracle_rms_norm_f32(const float* input, size_t input_len, const float* weight,
                        size_t weight_len, size_t hidden_size, float epsilon, float* output,
                        oracle_error* err) {
    int status = validate_norm(input_len, weight_len, hidden_size, epsilon, err);
    if (status != ORACLE_OK) return status;
    norm_rows(input, input_len, weight, hidden_size, epsilon, output);
    return ORACLE_OK;
}

int oracle_fused_add_rms_norm_f32(const float* input, size_t input_len, const float* residual,
                                  size_t residual_len, const float* weight, size_t weight_len,
                                  size_t hidden_size, float epsilon, float* normalized,
                                  float* residual_out, oracle_error* err) {
    if (hidden_size == 0) return ORACLE_REF_ZERO_HIDDEN_SIZE;
    if (weight_len != hidden_size) {
        set_err(err, weight_len, hidden_size, 0);
        return ORACLE_REF_WEIGHT_LENGTH_MISMATCH;
    }
    if (residual_len != input_len) {
        set_err(err, residual_len, input_len, 0);
        return ORACLE_REF_RESIDUAL_LENGTH_MISMATCH;
    }
    int status = validate_norm(input_len, weight_len, hidden_size, epsilon, err);
    if (status != ORACLE_OK) return status;
    for (size_t i = 0; i < input_len; i++) residual_out[i] = input[i] + residual[i];
    norm_rows(residual_out, input_len, weight, hidden_size, epsilon, normalized);
    return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* New operators                                                             */
/* ------------------------------------------------------------------------ */

int oracle_q4_0_quantize_rows(const float* input, size_t rows, size_t k, uint8_t* output) {
    if (k % 32 != 0) return ORACLE_ARGUMENT_INVALID;
    const size_t nb = k / 32;
    for (size_t r = 0; r < rows; r++) {
        const float* x = input + r * k;
        uint8_t* y = output + r * nb * 18;
        for (size_t i = 0; i < nb; i++) {
            float amax = 0.0f, max = 0.0f;
            for (size_t j = 0; j < 32; j++) {
                const float v = x[i * 32 + j];
                if (amax < fabsf(v)) {
                    amax = fabsf(v);
                    max = v;
                }
            }
            const float d = max / -8.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            const uint16_t dh = oracle_f32_to_f16(d);
            uint8_t* blk = y + i * 18;
            blk[0] = (uint8_t)(dh & 0xFF);
            blk[1] = (uint8_t)(dh >> 8);
            for (size_t j = 0; j < 16; j++) {
                const float x0 = x[i * 32 + j] * id;
                const float x1 = x[i * 32 + 16 + j] * id;
                int q0 = (int)(int8_t)(x0 + 8.5f);
                int q1 = (int)(int8_t)(x1 + 8.5f);
                if (q0 > 15) q0 = 15;
                if (q1 > 15) q1 = 15;
                blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
    return ORACLE_OK;
}

int oracle_embedding_gather_f16(const uint16_t* table, size_t vocab, size_t hidden,
                                const int32_t* ids, size_t tokens, uint16_t* output,
                                uint32_t* out_of_range) {
    uint32_t bad = 0;
    for (size_t t = 0; t < tokens; t++) {
        const int32_t id = ids[t];
        if (id < 0 || (size_t)id >= vocab) {
            memset(output + t * hidden, 0, hidden * sizeof(uint16_t));
            bad = 1;
        } else {
            memcpy(output + t * hidden, table + (size_t)id * hidden, hidden * sizeof(uint16_t));
        }
    }
    if (out_of_range) *out_of_range = bad;
    return ORACLE_OK;
}

void oracle_swiglu_f64(const float* gate, const float* up, size_t n, float* output) {
    for (size_t i = 0; i < n; i++) {
        const double g = gate[i];
        output[i] = (float)(g / (1.0 + exp(-g)) * (double)up[i]);
    }
}

int oracle_rope_cos_sin_f64(const int32_t* positions, size_t tokens, size_t rotary_dim,
                            double theta, float* cos_out, float* sin_out) {
    if (rotary_dim % 2 != 0) return ORACLE_ARGUMENT_INVALID;
    const size_t half = rotary_dim / 2;
    for (size_t t = 0; t < tokens; t++) {
        for (size_t j = 0; j < half; j++) {
            const double inv_freq = pow(theta, -(double)(2 * j) / (double)rotary_dim);
            const double angle = (double)positions[t] * inv_freq;
            cos_out[t * half + j] = (float)cos(angle);
            sin_out[t * half + j] = (float)sin(angle);
        }
    }
    return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* K-quants: ggml's published dequantization (gguf 0.19.0, gguf/quants.py)   */
/* ------------------------------------------------------------------------ */

/* The 6-bit scale and min of sub-block j (0..7) from the 12 packed bytes:
 * bytes 0-3 hold scales 0-3 (low 6 bits) and the top bits of scales 4-7,
 * bytes 4-7 mins 0-3 and the top bits of mins 4-7, bytes 8-11 the low four
 * bits of scales 4-7 (low nibble) and mins 4-7 (high nibble). */
static void q4_k_scale_min(const uint8_t* s, int j, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q4_K block (144 bytes): f16 d, f16 dmin, 12 scale bytes, 128 quant bytes.
 * Quant byte l of 32-byte group c holds element 64c + l (low nibble) and
 * element 64c + 32 + l (high nibble). */
static void decode_q4_k_block(const uint8_t* b, float* y) {
    const float d = oracle_f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const float dmin = oracle_f16_to_f32((uint16_t)(b[2] | (b[3] << 8)));
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    for (int c = 0; c < 4; c++) {
        uint8_t sc0, m0, sc1, m1;
        q4_k_scale_min(scales, 2 * c, &sc0, &m0);
        q4_k_scale_min(scales, 2 * c + 1, &sc1, &m1);
        const float d0 = d * (float)sc0, dm0 = dmin * (float)m0;
        const float d1 = d * (float)sc1, dm1 = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            y[64 * c + l] = d0 * (float)(qs[32 * c + l] & 0x0F) - dm0;
            y[64 * c + 32 + l] = d1 * (float)(qs[32 * c + l] >> 4) - dm1;
        }
    }
}

/* Q6_K block (210 bytes): 128 bytes of low nibbles, 64 bytes of 2-bit high
 * parts, 16 int8 scales (one per 16 elements), f16 d.  In half h (128
 * elements), element e takes nibble (e / 64) of low byte 64h + e % 64 and
 * bit pair (e / 32) of high byte 32h + e % 32; q = that 6-bit value - 32. */
static void decode_q6_k_block(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = oracle_f16_to_f32((uint16_t)(b[208] | (b[209] << 8)));
    for (int h = 0; h < 2; h++) {
        for (int e = 0; e < 128; e++) {
            const uint8_t lo = (uint8_t)((ql[64 * h + (e % 64)] >> (4 * (e / 64))) & 0x0F);
            const uint8_t hi = (uint8_t)((qh[32 * h + (e % 32)] >> (2 * (e / 32))) & 0x03);
            const int q = (int)(lo | (hi << 4)) - 32;
            const int idx = 128 * h + e;
            y[idx] = (d * (float)sc[idx / 16]) * (float)q;
        }
    }
}

int oracle_kquant_dequantize_row(const uint8_t* bytes, size_t bytes_len, int format,
                                 size_t row_elements, float* output) {
    if (format != ORACLE_Q4_K && format != ORACLE_Q6_K) return ORACLE_QL_UNSUPPORTED_FORMAT;
    if (row_elements % 256 != 0) return ORACLE_QL_ROW_MISALIGNED;
    const size_t bb = oracle_block_bytes(format);
    if (bytes_len != row_elements / 256 * bb) return ORACLE_QL_ROW_BYTE_LENGTH_MISMATCH;
    for (size_t blk = 0; blk < row_elements / 256; blk++) {
        if (format == ORACLE_Q4_K)
            decode_q4_k_block(bytes + blk * bb, output + blk * 256);
        else
            decode_q6_k_block(bytes + blk * bb, output + blk * 256);
    }
    return ORACLE_OK;
}

int oracle_kquant_linear_f64(const float* input, const uint8_t* weights, int format, size_t rows,
                             size_t n, size_t k, double* output) {
    if (format != ORACLE_Q4_K && format != ORACLE_Q6_K) return ORACLE_QL_UNSUPPORTED_FORMAT;
    if (k % 256 != 0) return ORACLE_QL_ROW_MISALIGNED;
    const size_t row_bytes = k / 256 * oracle_block_bytes(format);
    float* decoded = (float*)malloc((k ? k : 1) * sizeof(float));
    if (!decoded) return ORACLE_ARGUMENT_INVALID;
    for (size_t f = 0; f < n; f++) {
        oracle_kquant_dequantize_row(weights + f * row_bytes, row_bytes, format, k, decoded);
        for (size_t r = 0; r < rows; r++) {
            const float* x = input + r * k;
            double s = 0.0;
            for (size_t i = 0; i < k; i++) s += (double)x[i] * (double)decoded[i];
            output[r * n + f] = s;
        }
    }
    free(decoded);
    return ORACLE_OK;
}
