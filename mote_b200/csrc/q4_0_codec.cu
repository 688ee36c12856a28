// Q4_0 block codec (device decode / encode) and the RoPE cos/sin table.
//
// Decode is bit-exact with mote-reference's decode_row_into
// (crates/mote-reference/src/quantized.rs:177-201): value = f32(q - 8) *
// f32(d) is exact in f32.  Encode restates ggml's published Q4_0 reference
// quantizer with explicitly rounded IEEE operations, so it is bit-exact
// with the CPU restatement used by the tests.

#include "mote_common.cuh"

namespace mote {
namespace codec {

// One thread per 32-element block.
__global__ void __launch_bounds__(256) q4_0_decode_kernel(const std::uint8_t* __restrict__ w,
                                                          float* __restrict__ out,
                                                          std::uint64_t blocks) {
    for (std::uint64_t b = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         b < blocks; b += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
        const std::uint8_t* blk = w + b * 18;
        const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
        float* o = out + b * 32;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const std::uint8_t q = blk[2 + j];
            o[j] = __fmul_rn(static_cast<float>(static_cast<int>(q & 15) - 8), d);
            o[j + 16] = __fmul_rn(static_cast<float>(static_cast<int>(q >> 4) - 8), d);
        }
    }
}

// ggml quantize_row_q4_0_ref, per block: m = first element of largest
// magnitude; d = m / -8; id = d != 0 ? 1/d : 0; scale = f16(d);
// q = min(15, trunc(x * id + 8.5)).
__global__ void __launch_bounds__(256) q4_0_encode_kernel(const float* __restrict__ in,
                                                          std::uint8_t* __restrict__ w,
                                                          std::uint64_t blocks) {
    for (std::uint64_t b = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         b < blocks; b += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
        const float* x = in + b * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(x + j));
            v[j] = f.x;
            v[j + 1] = f.y;
            v[j + 2] = f.z;
            v[j + 3] = f.w;
        }
        float amax = 0.f, mx = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(v[j]);
            if (amax < a) {
                amax = a;
                mx = v[j];
            }
        }
        const float d = __fdiv_rn(mx, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        // The 18-byte block is 2-byte aligned: write it as nine 16-bit words
        // (little endian: scale first, then quant bytes 2j, 2j+1 per word).
        unsigned short* blk = reinterpret_cast<unsigned short*>(w + b * 18);
        blk[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            unsigned pair = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float x0 = __fmul_rn(v[j + h], id);
                const float x1 = __fmul_rn(v[j + h + 16], id);
                const int q0 = min(15, __float2int_rz(__fadd_rn(x0, 8.5f)));
                const int q1 = min(15, __float2int_rz(__fadd_rn(x1, 8.5f)));
                pair |= static_cast<unsigned>(q0 | (q1 << 4)) << (8 * h);
            }
            blk[1 + j / 2] = static_cast<unsigned short>(pair);
        }
    }
}

// angle = positions[t] * theta^(-2j / rotary_dim), evaluated in f64 and
// rounded once to f32 (CUDA's double-precision pow/cos/sin).
__global__ void __launch_bounds__(256) rope_cos_sin_kernel(const std::int32_t* __restrict__ pos,
                                                           float* __restrict__ cos_out,
                                                           float* __restrict__ sin_out,
                                                           std::uint64_t tokens,
                                                           std::uint64_t half, double theta,
                                                           double rotary_dim) {
    const std::uint64_t total = tokens * half;
    for (std::uint64_t i = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         i < total; i += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
        const std::uint64_t t = i / half;
        const std::uint64_t j = i - t * half;
        const double inv_freq = pow(theta, -static_cast<double>(2 * j) / rotary_dim);
        const double angle = static_cast<double>(pos[t]) * inv_freq;
        double s, c;
        sincos(angle, &s, &c);
        cos_out[i] = static_cast<float>(c);
        sin_out[i] = static_cast<float>(s);
    }
}

inline unsigned grid_for(std::uint64_t items) {
    const std::uint64_t g = (items + 255) / 256;
    return static_cast<unsigned>(g < 148ull * 32 ? (g == 0 ? 1 : g) : 148ull * 32);
}

}  // namespace codec
}  // namespace mote

using namespace mote;

// Decodes a [rows, input_features] Q4_0 matrix to f32 (bit-exact).
extern "C" int mote_cuda_q4_0_decode_f32(const void* weights, void* output, std::uint64_t rows,
                                         std::uint64_t input_features, void* stream) {
    if (weights == nullptr || output == nullptr || stream == nullptr) return kInvalidValue;
    if (input_features % 32 != 0) return kInvalidValue;
    if (rows == 0 || input_features == 0) return kSuccess;
    if (rows > (~0ull) / input_features) return kInvalidConfiguration;
    const std::uint64_t blocks = rows * (input_features / 32);
    codec::q4_0_decode_kernel<<<codec::grid_for(blocks), 256, 0,
                                static_cast<cudaStream_t>(stream)>>>(
        static_cast<const std::uint8_t*>(weights), static_cast<float*>(output), blocks);
    return static_cast<int>(cudaGetLastError());
}

// Encodes a [rows, input_features] f32 matrix into Q4_0 blocks.  The input
// must be 16-byte aligned (float4 loads) and the output 2-byte aligned (the
// Q4_0 storage alignment of crates/mote-types/src/lib.rs:68-74).
extern "C" int mote_cuda_q4_0_encode_f32(const void* input, void* weights, std::uint64_t rows,
                                         std::uint64_t input_features, void* stream) {
    if (input == nullptr || weights == nullptr || stream == nullptr) return kInvalidValue;
    if (input_features % 32 != 0) return kInvalidValue;
    if (reinterpret_cast<std::uintptr_t>(input) % 16 != 0) return kInvalidValue;
    if (reinterpret_cast<std::uintptr_t>(weights) % 2 != 0) return kInvalidValue;
    if (rows == 0 || input_features == 0) return kSuccess;
    if (rows > (~0ull) / input_features) return kInvalidConfiguration;
    const std::uint64_t blocks = rows * (input_features / 32);
    codec::q4_0_encode_kernel<<<codec::grid_for(blocks), 256, 0,
                                static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(input), static_cast<std::uint8_t*>(weights), blocks);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int mote_cuda_rope_cos_sin_f32(const void* positions, void* cos_out, void* sin_out,
                                          std::uint64_t tokens, std::uint64_t rotary_dim,
                                          double theta, void* stream) {
    if (positions == nullptr || cos_out == nullptr || sin_out == nullptr || stream == nullptr)
        return kInternalError;
    if ((rotary_dim & 1u) != 0 || !(theta > 0.0)) return kInternalError;
    if (tokens == 0 || rotary_dim == 0) return kSuccess;
    const std::uint64_t half = rotary_dim / 2;
    codec::rope_cos_sin_kernel<<<codec::grid_for(tokens * half), 256, 0,
                                 static_cast<cudaStream_t>(stream)>>>(
        static_cast<const std::int32_t*>(positions), static_cast<float*>(cos_out),
        static_cast<float*>(sin_out), tokens, half, theta, static_cast<double>(rotary_dim));
    return static_cast<int>(cudaGetLastError());
}
