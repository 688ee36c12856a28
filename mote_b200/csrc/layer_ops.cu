// Per-token layer kernels: RMSNorm, residual-add + RMSNorm, RoPE, the fused
// RMSNorm + RoPE layer kernel, SwiGLU and embedding gather.
//
// All of them are single-pass bandwidth kernels: every input byte is read
// once into registers with 16-byte vector loads where the shape allows, the
// row statistics are reduced with warp shuffles plus one shared-memory step,
// and outputs are written once.  Arithmetic follows the f32 operation order
// of mote-reference with explicitly rounded intrinsics (no FMA contraction):
//   rms_norm_f32           crates/mote-reference/src/lib.rs:262-301
//   fused_add_rms_norm_f32 crates/mote-reference/src/lib.rs:333-384
//   rope_f32               crates/mote-reference/src/lib.rs:170-244
// so RoPE is bit-identical to the oracle before the final f16 rounding and
// the norms differ only by the order of the sum of squares.

#include "mote_common.cuh"

namespace mote {
namespace layer {

constexpr int kNormThreads = 256;
constexpr int kLayoutHalfSplit = 0;
constexpr int kLayoutInterleaved = 1;

__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    const int nwarps = blockDim.x >> 5;
    float total = 0.f;
    for (int w = 0; w < nwarps; ++w) total += scratch[w];
    return total;
}

// 1 / sqrt(mean_square + eps) exactly as the oracle: correctly rounded sqrt
// and division.

union H8 {
    uint4 u;
    __half h[8];
};

// ---- RMSNorm ----------------------------------------------------------------
// Vector path: hidden % 8 == 0, 16-byte aligned rows, hidden <= 256*8*VPT.
template <int VPT>
__global__ void __launch_bounds__(kNormThreads) rms_norm_vec_kernel(
    const __half* input, const __half* __restrict__ weight, __half* output,
    std::uint64_t hidden, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float scratch[kNormThreads / 32];
    const std::uint64_t row = blockIdx.x;
    const uint4* in = reinterpret_cast<const uint4*>(input + row * hidden);
    uint4* out = reinterpret_cast<uint4*>(output + row * hidden);
    const uint4* wv = reinterpret_cast<const uint4*>(weight);
    const std::uint32_t nvec = static_cast<std::uint32_t>(hidden / 8);
    H8 x[VPT];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        if (v < nvec) {
            x[i].u = in[v];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float f = __half2float(x[i].h[j]);
                ss = __fadd_rn(ss, __fmul_rn(f, f));
            }
        }
    }
    const float inv = inv_rms(block_sum(ss, scratch), hidden, eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        if (v < nvec) {
            H8 w, o;
            w.u = __ldg(&wv[v]);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                o.h[j] = __float2half_rn(
                    norm_out(__half2float(x[i].h[j]), inv, __half2float(w.h[j])));
            out[v] = o.u;
        }
    }
}

// Scalar path for any hidden size (e.g. 513) and alignment: two strided
// passes over the row (the second pass re-reads from L1/L2).
__global__ void __launch_bounds__(kNormThreads) rms_norm_scalar_kernel(
    const __half* input, const __half* __restrict__ weight, __half* output,
    std::uint64_t hidden, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float scratch[kNormThreads / 32];
    const std::uint64_t row = blockIdx.x;
    const __half* in = input + row * hidden;
    __half* out = output + row * hidden;
    float ss = 0.f;
    for (std::uint64_t i = threadIdx.x; i < hidden; i += kNormThreads) {
        const float f = __half2float(in[i]);
        ss = __fadd_rn(ss, __fmul_rn(f, f));
    }
    const float inv = inv_rms(block_sum(ss, scratch), hidden, eps);
    for (std::uint64_t i = threadIdx.x; i < hidden; i += kNormThreads)
        out[i] = __float2half_rn(norm_out(__half2float(in[i]), inv, __half2float(weight[i])));
}

// ---- residual add + RMSNorm ------------------------------------------------
// input may alias output and/or residual; output never aliases residual
// (rejected by the shim).  All reads of a row happen before the block-wide
// reduction, all writes after it, and each element is read and written by
// the same thread, so the aliasing cases are race-free.
template <int VPT>
__global__ void __launch_bounds__(kNormThreads) fused_add_rms_norm_vec_kernel(
    const __half* input, __half* residual, const __half* __restrict__ weight, __half* output,
    std::uint64_t hidden, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float scratch[kNormThreads / 32];
    const std::uint64_t row = blockIdx.x;
    const uint4* in = reinterpret_cast<const uint4*>(input + row * hidden);
    uint4* res = reinterpret_cast<uint4*>(residual + row * hidden);
    uint4* out = reinterpret_cast<uint4*>(output + row * hidden);
    const uint4* wv = reinterpret_cast<const uint4*>(weight);
    const std::uint32_t nvec = static_cast<std::uint32_t>(hidden / 8);
    float s[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        if (v < nvec) {
            H8 a, b;
            a.u = in[v];
            b.u = res[v];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                s[i][j] = __fadd_rn(__half2float(a.h[j]), __half2float(b.h[j]));
                ss = __fadd_rn(ss, __fmul_rn(s[i][j], s[i][j]));
            }
        }
    }
    const float inv = inv_rms(block_sum(ss, scratch), hidden, eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        if (v < nvec) {
            H8 w, o, r;
            w.u = __ldg(&wv[v]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o.h[j] = __float2half_rn(norm_out(s[i][j], inv, __half2float(w.h[j])));
                r.h[j] = __float2half_rn(s[i][j]);
            }
            out[v] = o.u;
            res[v] = r.u;
        }
    }
}

__global__ void __launch_bounds__(kNormThreads) fused_add_rms_norm_scalar_kernel(
    const __half* input, __half* residual, const __half* __restrict__ weight, __half* output,
    std::uint64_t hidden, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float scratch[kNormThreads / 32];
    const std::uint64_t row = blockIdx.x;
    const __half* in = input + row * hidden;
    __half* res = residual + row * hidden;
    __half* out = output + row * hidden;
    float ss = 0.f;
    for (std::uint64_t i = threadIdx.x; i < hidden; i += kNormThreads) {
        const float s = __fadd_rn(__half2float(in[i]), __half2float(res[i]));
        ss = __fadd_rn(ss, __fmul_rn(s, s));
    }
    const float inv = inv_rms(block_sum(ss, scratch), hidden, eps);
    // Same element -> same thread in both passes; the reduction's
    // __syncthreads separates every read of pass 1 from the writes below.
    for (std::uint64_t i = threadIdx.x; i < hidden; i += kNormThreads) {
        const float s = __fadd_rn(__half2float(in[i]), __half2float(res[i]));
        out[i] = __float2half_rn(norm_out(s, inv, __half2float(weight[i])));
        res[i] = __float2half_rn(s);
    }
}

// ---- RoPE -------------------------------------------------------------------

// One thread per rotation pair or tail element of every (token, head)
// vector.  Each element is read and written by one thread only, so
// input == output is race-free.
__global__ void __launch_bounds__(256) rope_kernel(const __half* input,
                                                   const float* __restrict__ cos,
                                                   const float* __restrict__ sin, __half* output,
                                                   std::uint64_t vectors, std::uint64_t heads,
                                                   std::uint64_t head_dim,
                                                   std::uint64_t rotary_dim, int layout) {
    pdl_launch_dependents();
    pdl_wait();
    const std::uint64_t half = rotary_dim / 2;
    const std::uint64_t per_vec = half + (head_dim - rotary_dim);
    const std::uint64_t total = vectors * per_vec;
    for (std::uint64_t idx = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         idx < total; idx += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
        const std::uint64_t vec = idx / per_vec;
        const std::uint64_t item = idx - vec * per_vec;
        const __half* vi = input + vec * head_dim;
        __half* vo = output + vec * head_dim;
        if (item < half) {
            const std::uint64_t token = vec / heads;
            const std::uint64_t first = layout == kLayoutHalfSplit ? item : 2 * item;
            const std::uint64_t second = layout == kLayoutHalfSplit ? item + half : 2 * item + 1;
            const float c = cos[token * half + item];
            const float s = sin[token * half + item];
            float o1, o2;
            rotate(__half2float(vi[first]), __half2float(vi[second]), c, s, o1, o2);
            vo[first] = __float2half_rn(o1);
            vo[second] = __float2half_rn(o2);
        } else {
            const std::uint64_t e = rotary_dim + (item - half);
            vo[e] = vi[e];
        }
    }
}

// ---- fused RMSNorm + RoPE (one CTA per token) --------------------------------
// Normalizes x[token] (hidden) and rotates q[token] (q_heads x HD) and
// k[token] (kv_heads x HD) with the token's cos/sin row; rotary_dim == HD.
// gamma and the token's cos/sin row are parameters, not activations: they
// are copied to shared memory before griddepcontrol.wait, so their latency
// hides behind the previous kernel's tail (the caller must not have them
// written by this library's kernels still in flight on the stream).  Every
// load of the token (q, k and x rows, 16 bytes per thread per vector) is
// issued right after the wait, so the CTA pays one memory latency.  A
// thread owns 8 consecutive elements of a head; for the half-split layout
// the partner of element e < HD/2 is e + HD/2, held by the thread HD/16
// lanes away (q/k rows are whole heads, so partners never cross rows).
constexpr int kRopeVecPerThread = 2;   // (q_heads + kv_heads) * HD / 8 <= 512
constexpr int kNormVecPerThread = 4;   // hidden <= 8192

template <int HD>
__global__ void __launch_bounds__(kNormThreads, 4) rms_norm_rope_kernel(
    const __half* x, const __half* __restrict__ gamma, __half* x_out, const __half* q,
    __half* q_out, const __half* k, __half* k_out, const float* __restrict__ cos,
    const float* __restrict__ sin, std::uint64_t hidden, std::uint32_t q_heads,
    std::uint32_t kv_heads, float eps, int layout) {
    pdl_launch_dependents();
    __shared__ float scratch[kNormThreads / 32];
    // gamma (hidden f16; a thread copies exactly the vectors it later reads)
    // and the token's cos | sin row (HD/2 + HD/2 f32, shared by all threads)
    __shared__ __align__(16) uint4 gamma_s[kNormVecPerThread * kNormThreads];
    __shared__ __align__(16) float cs_s[HD];
    constexpr int kLanesPerHead = HD / 8;
    constexpr int kHalfLanes = kLanesPerHead / 2;
    const std::uint64_t token = blockIdx.x;
    const std::uint32_t qn = q_heads * HD / 8;
    const std::uint32_t rn = qn + kv_heads * HD / 8;
    const std::uint32_t xn = static_cast<std::uint32_t>(hidden / 8);
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        if (v < xn) cp_async_16_default(smem_u32(&gamma_s[v]), reinterpret_cast<const uint4*>(gamma) + v);
    }
    if (threadIdx.x < HD / 4) {  // HD/8 16-byte chunks of cos, then HD/8 of sin
        const std::uint32_t c = threadIdx.x;
        const float* src = c < HD / 8 ? cos + token * (HD / 2) + c * 4
                                      : sin + token * (HD / 2) + (c - HD / 8) * 4;
        cp_async_16_default(smem_u32(&cs_s[c * 4]), src);
    }
    cp_async_commit();
    pdl_wait();
    const uint4* qv = reinterpret_cast<const uint4*>(q + token * q_heads * HD);
    const uint4* kv = reinterpret_cast<const uint4*>(k + token * kv_heads * HD);
    const uint4* xv = reinterpret_cast<const uint4*>(x + token * hidden);

    H8 r[kRopeVecPerThread];
    H8 xr[kNormVecPerThread];
#pragma unroll
    for (int i = 0; i < kRopeVecPerThread; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        r[i].u = v < qn ? qv[v] : (v < rn ? kv[v - qn] : make_uint4(0, 0, 0, 0));
    }
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        xr[i].u = v < xn ? xv[v] : make_uint4(0, 0, 0, 0);
    }

    // RoPE of the q and k rows (the barrier runs while the loads are in flight).
    cp_async_wait<0>();
    __syncthreads();
    const float* cs = cs_s;
    const float* sn = cs_s + HD / 2;
#pragma unroll
    for (int i = 0; i < kRopeVecPerThread; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        const int pos = (v % kLanesPerHead) * 8;  // element offset within the head
        H8 o;
        if (layout == kLayoutHalfSplit) {
            H8 partner;
            partner.u.x = __shfl_xor_sync(0xffffffffu, r[i].u.x, kHalfLanes);
            partner.u.y = __shfl_xor_sync(0xffffffffu, r[i].u.y, kHalfLanes);
            partner.u.z = __shfl_xor_sync(0xffffffffu, r[i].u.z, kHalfLanes);
            partner.u.w = __shfl_xor_sync(0xffffffffu, r[i].u.w, kHalfLanes);
            const bool first = pos < HD / 2;
            const int j0 = first ? pos : pos - HD / 2;
            const float4 c0 = *reinterpret_cast<const float4*>(cs + j0);
            const float4 c1 = *reinterpret_cast<const float4*>(cs + j0 + 4);
            const float4 s0 = *reinterpret_cast<const float4*>(sn + j0);
            const float4 s1 = *reinterpret_cast<const float4*>(sn + j0 + 4);
            const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float o1, o2;
                if (first) {
                    rotate(__half2float(r[i].h[j]), __half2float(partner.h[j]), cc[j], ss[j], o1,
                           o2);
                    o.h[j] = __float2half_rn(o1);
                } else {
                    rotate(__half2float(partner.h[j]), __half2float(r[i].h[j]), cc[j], ss[j], o1,
                           o2);
                    o.h[j] = __float2half_rn(o2);
                }
            }
        } else {
            const float4 c0 = *reinterpret_cast<const float4*>(cs + pos / 2);
            const float4 s0 = *reinterpret_cast<const float4*>(sn + pos / 2);
            const float cc[4] = {c0.x, c0.y, c0.z, c0.w};
            const float ss[4] = {s0.x, s0.y, s0.z, s0.w};
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                float o1, o2;
                rotate(__half2float(r[i].h[j]), __half2float(r[i].h[j + 1]), cc[j / 2], ss[j / 2],
                       o1, o2);
                o.h[j] = __float2half_rn(o1);
                o.h[j + 1] = __float2half_rn(o2);
            }
        }
        if (v < qn)
            reinterpret_cast<uint4*>(q_out + token * q_heads * HD)[v] = o.u;
        else if (v < rn)
            reinterpret_cast<uint4*>(k_out + token * kv_heads * HD)[v - qn] = o.u;
    }

    // RMSNorm of x[token].
    float ssq = 0.f;
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float f = __half2float(xr[i].h[j]);
            ssq = __fadd_rn(ssq, __fmul_rn(f, f));
        }
    const float inv = inv_rms(block_sum(ssq, scratch), hidden, eps);
    uint4* out = reinterpret_cast<uint4*>(x_out + token * hidden);
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i) {
        const std::uint32_t v = threadIdx.x + i * kNormThreads;
        if (v < xn) {
            H8 w, o;
            w.u = gamma_s[v];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                o.h[j] = __float2half_rn(norm_out(__half2float(xr[i].h[j]), inv,
                                                  __half2float(w.h[j])));
            out[v] = o.u;
        }
    }
}

// ---- SwiGLU -----------------------------------------------------------------
__device__ __forceinline__ float silu_mul(float g, float u) {
    return g / (1.0f + expf(-g)) * u;
}

__global__ void __launch_bounds__(256) swiglu_vec_kernel(const __half* gate, const __half* up,
                                                        __half* out, std::uint64_t nvec) {
    pdl_launch_dependents();
    pdl_wait();
    for (std::uint64_t v = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         v < nvec; v += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
        H8 g, u, o;
        g.u = reinterpret_cast<const uint4*>(gate)[v];
        u.u = reinterpret_cast<const uint4*>(up)[v];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            o.h[j] = __float2half_rn(silu_mul(__half2float(g.h[j]), __half2float(u.h[j])));
        reinterpret_cast<uint4*>(out)[v] = o.u;
    }
}

__global__ void __launch_bounds__(256) swiglu_scalar_kernel(const __half* gate, const __half* up,
                                                           __half* out, std::uint64_t n) {
    pdl_launch_dependents();
    pdl_wait();
    for (std::uint64_t i = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         i < n; i += static_cast<std::uint64_t>(gridDim.x) * blockDim.x)
        out[i] = __float2half_rn(silu_mul(__half2float(gate[i]), __half2float(up[i])));
}

// ---- embedding gather ----------------------------------------------------------
// One CTA per token copies one table row (bit-exact).  Ids outside
// [0, vocab) write a zero row and set bit kDevIndexOutOfRange in *flag.
template <bool VEC>
__global__ void __launch_bounds__(256) embedding_gather_kernel(
    const __half* __restrict__ table, const std::int32_t* __restrict__ ids, __half* out,
    std::uint64_t vocab, std::uint64_t hidden, unsigned* flag) {
    pdl_launch_dependents();
    pdl_wait();
    const std::uint64_t token = blockIdx.x;
    const std::int32_t id = ids[token];
    const bool ok = id >= 0 && static_cast<std::uint64_t>(id) < vocab;
    if (!ok && threadIdx.x == 0) atomicOr(flag, kDevIndexOutOfRange);
    if constexpr (VEC) {
        const std::uint64_t nvec = hidden / 8;
        const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * hidden);
        uint4* dst = reinterpret_cast<uint4*>(out + token * hidden);
        for (std::uint64_t v = threadIdx.x; v < nvec; v += blockDim.x)
            dst[v] = ok ? __ldg(&src[v]) : make_uint4(0, 0, 0, 0);
    } else {
        const __half* src = table + (ok ? id : 0) * hidden;
        __half* dst = out + token * hidden;
        for (std::uint64_t i = threadIdx.x; i < hidden; i += blockDim.x)
            dst[i] = ok ? src[i] : __ushort_as_half(0);
    }
}

inline bool aligned16(const void* p) { return reinterpret_cast<std::uintptr_t>(p) % 16 == 0; }

inline unsigned grid_for(std::uint64_t items, unsigned threads) {
    const std::uint64_t g = (items + threads - 1) / threads;
    return static_cast<unsigned>(g < 148ull * 32 ? (g == 0 ? 1 : g) : 148ull * 32);
}

}  // namespace layer
}  // namespace mote

using namespace mote;
using namespace mote::layer;

// Argument checks mirror mote_hip_rms_norm_f16
// (crates/mote-backend-hip/src/rms_norm.hip:68-98).
extern "C" int mote_cuda_rms_norm_f16(const void* input, const void* weight, void* output,
                                      std::uint64_t rows, std::uint64_t hidden_size,
                                      float epsilon, void* stream) {
    if (input == nullptr || weight == nullptr || output == nullptr || stream == nullptr)
        return kInternalError;
    if (rows == 0 || hidden_size == 0) return kSuccess;
    if (rows > kMaxGridX) return kInternalError;
    auto* in = static_cast<const __half*>(input);
    auto* w = static_cast<const __half*>(weight);
    auto* out = static_cast<__half*>(output);
    auto s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(rows));
    const bool vec = hidden_size % 8 == 0 && aligned16(input) && aligned16(weight) &&
                     aligned16(output);
    const dim3 block(kNormThreads);
    if (vec && hidden_size <= 256 * 8)
        return launch_pdl(rms_norm_vec_kernel<1>, grid, block, s, in, w, out, hidden_size, epsilon);
    if (vec && hidden_size <= 256 * 8 * 2)
        return launch_pdl(rms_norm_vec_kernel<2>, grid, block, s, in, w, out, hidden_size, epsilon);
    if (vec && hidden_size <= 256 * 8 * 4)
        return launch_pdl(rms_norm_vec_kernel<4>, grid, block, s, in, w, out, hidden_size, epsilon);
    return launch_pdl(rms_norm_scalar_kernel, grid, block, s, in, w, out, hidden_size, epsilon);
}

// Argument checks mirror mote_hip_fused_add_rms_norm_f16
// (crates/mote-backend-hip/src/fused_add_rms_norm.hip:99-138).
extern "C" int mote_cuda_fused_add_rms_norm_f16(const void* input, void* residual,
                                                const void* weight, void* output,
                                                std::uint64_t rows, std::uint64_t hidden_size,
                                                float epsilon, void* stream) {
    if (input == nullptr || residual == nullptr || weight == nullptr || output == nullptr ||
        stream == nullptr)
        return kInternalError;
    if (!isfinite(epsilon) || epsilon < 0.0f) return kInternalError;
    if (output == residual) return kInternalError;
    if (rows == 0 || hidden_size == 0) return kSuccess;
    if (rows > kMaxGridX) return kInternalError;
    auto* in = static_cast<const __half*>(input);
    auto* res = static_cast<__half*>(residual);
    auto* w = static_cast<const __half*>(weight);
    auto* out = static_cast<__half*>(output);
    auto s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(rows));
    const bool vec = hidden_size % 8 == 0 && aligned16(input) && aligned16(residual) &&
                     aligned16(weight) && aligned16(output);
    const dim3 block(kNormThreads);
    if (vec && hidden_size <= 256 * 8)
        return launch_pdl(fused_add_rms_norm_vec_kernel<1>, grid, block, s, in, res, w, out,
                          hidden_size, epsilon);
    if (vec && hidden_size <= 256 * 8 * 2)
        return launch_pdl(fused_add_rms_norm_vec_kernel<2>, grid, block, s, in, res, w, out,
                          hidden_size, epsilon);
    if (vec && hidden_size <= 256 * 8 * 4)
        return launch_pdl(fused_add_rms_norm_vec_kernel<4>, grid, block, s, in, res, w, out,
                          hidden_size, epsilon);
    return launch_pdl(fused_add_rms_norm_scalar_kernel, grid, block, s, in, res, w, out,
                      hidden_size, epsilon);
}

// Argument checks mirror mote_hip_rope_f16
// (crates/mote-backend-hip/src/rope.hip:99-150).
extern "C" int mote_cuda_rope_f16(const void* input, const void* cos, const void* sin,
                                  void* output, std::uint64_t tokens, std::uint64_t heads,
                                  std::uint64_t head_dim, std::uint64_t rotary_dim,
                                  std::uint32_t layout, void* stream) {
    if (input == nullptr || output == nullptr || stream == nullptr) return kInternalError;
    if (rotary_dim > 0 && (cos == nullptr || sin == nullptr)) return kInternalError;
    if (layout != kLayoutHalfSplit && layout != kLayoutInterleaved) return kInternalError;
    if ((rotary_dim & 1u) != 0 || rotary_dim > head_dim) return kInternalError;
    if (tokens == 0 || heads == 0 || head_dim == 0) return kSuccess;
    if (tokens > kMaxGridX / heads) return kInternalError;
    const std::uint64_t vectors = tokens * heads;
    const std::uint64_t per_vec = rotary_dim / 2 + (head_dim - rotary_dim);
    return launch_pdl(rope_kernel, dim3(grid_for(vectors * per_vec, 256)), dim3(256),
                      static_cast<cudaStream_t>(stream), static_cast<const __half*>(input),
                      static_cast<const float*>(cos), static_cast<const float*>(sin),
                      static_cast<__half*>(output), vectors, heads, head_dim, rotary_dim,
                      static_cast<int>(layout));
}

// Fused per-token layer kernel: RMSNorm of x and RoPE of q and k in one
// launch.  Argument rules are the union of mote_cuda_rms_norm_f16's and
// mote_cuda_rope_f16's, with rotary_dim == head_dim.  Shapes the vector
// kernel does not cover (head_dim not 64/128, hidden not a multiple of 8 or
// above 8192, unaligned buffers) run as the three separate kernels.
extern "C" int mote_cuda_rms_norm_rope_f16(const void* x, const void* gamma, void* x_out,
                                           const void* q, void* q_out, const void* k, void* k_out,
                                           const void* cos, const void* sin,
                                           std::uint64_t tokens, std::uint64_t hidden,
                                           std::uint64_t q_heads, std::uint64_t kv_heads,
                                           std::uint64_t head_dim, std::uint32_t layout,
                                           float epsilon, void* stream) {
    if (x == nullptr || gamma == nullptr || x_out == nullptr || q == nullptr ||
        q_out == nullptr || k == nullptr || k_out == nullptr || stream == nullptr)
        return kInternalError;
    if (head_dim > 0 && (cos == nullptr || sin == nullptr)) return kInternalError;
    if (layout != kLayoutHalfSplit && layout != kLayoutInterleaved) return kInternalError;
    if ((head_dim & 1u) != 0) return kInternalError;
    if (!isfinite(epsilon) || epsilon < 0.0f) return kInternalError;
    if (tokens == 0) return kSuccess;
    if (tokens > kMaxGridX) return kInternalError;
    auto s = static_cast<cudaStream_t>(stream);
    const bool vec = hidden % 8 == 0 && hidden > 0 && hidden <= 256 * 8 * kNormVecPerThread &&
                     (head_dim == 64 || head_dim == 128) &&
                     (q_heads + kv_heads) * head_dim / 8 <= 256ull * kRopeVecPerThread &&
                     aligned16(cos) && aligned16(sin) && aligned16(x) && aligned16(gamma) &&
                     aligned16(x_out) && aligned16(q) && aligned16(q_out) && aligned16(k) &&
                     aligned16(k_out) && q_heads <= 0xffffffffull && kv_heads <= 0xffffffffull;
    if (!vec) {
        int st = mote_cuda_rms_norm_f16(x, gamma, x_out, tokens, hidden, epsilon, stream);
        if (st != 0) return st;
        st = mote_cuda_rope_f16(q, cos, sin, q_out, tokens, q_heads, head_dim, head_dim, layout,
                                stream);
        if (st != 0) return st;
        return mote_cuda_rope_f16(k, cos, sin, k_out, tokens, kv_heads, head_dim, head_dim,
                                  layout, stream);
    }
    const dim3 grid(static_cast<unsigned>(tokens));
    auto args = [&](auto kernel) {
        return launch_pdl(kernel, grid, dim3(kNormThreads), s, static_cast<const __half*>(x),
                          static_cast<const __half*>(gamma), static_cast<__half*>(x_out),
                          static_cast<const __half*>(q), static_cast<__half*>(q_out),
                          static_cast<const __half*>(k), static_cast<__half*>(k_out),
                          static_cast<const float*>(cos), static_cast<const float*>(sin), hidden,
                          static_cast<std::uint32_t>(q_heads),
                          static_cast<std::uint32_t>(kv_heads), epsilon,
                          static_cast<int>(layout));
    };
    return head_dim == 64 ? args(rms_norm_rope_kernel<64>) : args(rms_norm_rope_kernel<128>);
}

extern "C" int mote_cuda_swiglu_f16(const void* gate, const void* up, void* output,
                                    std::uint64_t n, void* stream) {
    if (gate == nullptr || up == nullptr || output == nullptr || stream == nullptr)
        return kInternalError;
    if (n == 0) return kSuccess;
    auto s = static_cast<cudaStream_t>(stream);
    if (n % 8 == 0 && aligned16(gate) && aligned16(up) && aligned16(output))
        return launch_pdl(swiglu_vec_kernel, dim3(grid_for(n / 8, 256)), dim3(256), s,
                          static_cast<const __half*>(gate), static_cast<const __half*>(up),
                          static_cast<__half*>(output), n / 8);
    return launch_pdl(swiglu_scalar_kernel, dim3(grid_for(n, 256)), dim3(256), s,
                      static_cast<const __half*>(gate), static_cast<const __half*>(up),
                      static_cast<__half*>(output), n);
}

extern "C" int mote_cuda_embedding_gather_f16(const void* table, const void* ids, void* output,
                                              std::uint64_t tokens, std::uint64_t vocab,
                                              std::uint64_t hidden, void* error_flag,
                                              void* stream) {
    if (table == nullptr || ids == nullptr || output == nullptr || error_flag == nullptr ||
        stream == nullptr)
        return kInternalError;
    if (tokens == 0 || hidden == 0) return kSuccess;
    if (tokens > kMaxGridX) return kInternalError;
    auto s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(tokens));
    const bool vec = hidden % 8 == 0 && aligned16(table) && aligned16(output);
    auto* flag = static_cast<unsigned*>(error_flag);
    auto args = [&](auto kernel) {
        return launch_pdl(kernel, grid, dim3(256), s, static_cast<const __half*>(table),
                          static_cast<const std::int32_t*>(ids), static_cast<__half*>(output),
                          vocab, hidden, flag);
    };
    return vec ? args(embedding_gather_kernel<true>) : args(embedding_gather_kernel<false>);
}
