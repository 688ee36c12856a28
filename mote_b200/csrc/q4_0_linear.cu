// Q4_0 weight-only linear for decode and small batches (M <= 64).
//
//   y[m, n] = sum_k x[m, k] * w[n, k],   w stored as ggml Q4_0 blocks:
//   18 bytes per 32 elements = f16 scale d (little endian) + 16 bytes, byte j
//   holding element j in its low nibble and element j+16 in its high nibble;
//   value = (q - 8) * d.  (crates/mote-types/src/lib.rs:48-74,
//   crates/mote-reference/src/quantized.rs:177-201.)
//
// Design (B200):
// * A CTA owns one tile of 16 weight rows and splits K over its 4 warps.
//   Each warp streams its K-slice of the 16 rows into its own 4-slot shared
//   memory ring with 1-D bulk copies (cp.async.bulk, TMA engine), one copy
//   per row per stage, completion tracked by an mbarrier per slot.  Weights
//   are read from HBM exactly once, in 144/288-byte contiguous runs.
// * The dequantization happens in registers: each lane decodes one 4-byte
//   quant word per row per block into exact f16 integers (q - 8) with a
//   PRMT + LOP3 + HSUB2 sequence (1024+q / 64+q exponent tricks), and the
//   warp issues mma.sync.m16n8k16 (f16 x f16 -> f32) with weights as the A
//   operand and up to 8 activation tokens per n8 tile as B.  The per-block
//   f16 scale is applied to the f32 block partial with FFMA, so products and
//   scaling are exact and only f32 accumulation rounds.
// * The k-slot permutation inside each 16-wide MMA is chosen so a lane's B
//   fragment is 4 consecutive activations (one 8-byte load) and its A
//   fragment comes from one 4-byte quant word.  The permutation is the same
//   for A and B, so the dot product is unchanged.
// * f32 activations are split into f16 hi + lo parts placed in adjacent MMA
//   columns, which keeps their full precision (error ~2^-22 relative).
// * Cross-warp reduction of the four K-slices goes through shared memory.
//
// K must be a multiple of 256 (so a row is a whole number of 144-byte,
// 16-byte-aligned groups of 8 blocks) and the weights 16-byte aligned; other
// shapes use the generic warp-per-row kernel at the end of this file.

#include "mote_common.cuh"

#include <atomic>

namespace mote {
namespace q4 {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTileRows = 16;
constexpr int kStages = 4;
constexpr int kUnitBlocks = 8;            // 8 blocks = 256 elements = 144 bytes
constexpr int kUnitBytes = kUnitBlocks * 18;
constexpr int kStageUnits = 2;            // up to 16 blocks per stage
constexpr int kRowStride = kStageUnits * kUnitBytes + 16;  // 304: padded, bank-conflict free
constexpr int kStageBytes = kTileRows * kRowStride;         // 4864
constexpr int kWarpRingBytes = kStages * kStageBytes;       // 19456
constexpr int kSmemBytes = kWarps * kWarpRingBytes + kWarps * kStages * 8;

enum Epilogue : int { kEpiPlain = 0, kEpiSwiGLU = 1 };

struct Params {
    const void* x;            // [M, K] f16 or f32, row stride K
    const std::uint8_t* w;    // [N, K/32*18]
    const std::uint8_t* w2;   // second matrix (up projection) for kEpiSwiGLU
    void* y;                  // [M, ldy] f16 or f32
    std::uint32_t M;
    std::uint32_t N;          // rows of w (and of w2)
    std::uint64_t K;
    std::uint64_t pitch;      // bytes per weight row
    std::uint32_t units;      // K / 256
    std::uint64_t ldy;        // output row stride (elements)
};

__device__ __forceinline__ void decode_word(std::uint32_t u, std::uint32_t& lo01,
                                            std::uint32_t& lo23, std::uint32_t& hi01,
                                            std::uint32_t& hi23) {
    const std::uint32_t v = prmt(u, 0u, 0x4140u);  // [B0, 0, B1, 0]
    const std::uint32_t w = prmt(u, 0u, 0x4342u);  // [B2, 0, B3, 0]
    // low nibbles: f16(1024 + q) - 1032 = q - 8 (exact)
    lo01 = hsub2_u32(and_or(v, 0x000F000Fu, 0x64006400u), 0x64086408u);
    lo23 = hsub2_u32(and_or(w, 0x000F000Fu, 0x64006400u), 0x64086408u);
    // high nibbles sit at mantissa bits 4..7: f16(64 + q) - 72 = q - 8 (exact)
    hi01 = hsub2_u32(and_or(v, 0x00F000F0u, 0x54005400u), 0x54805480u);
    hi23 = hsub2_u32(and_or(w, 0x00F000F0u, 0x54005400u), 0x54805480u);
}

__device__ __forceinline__ std::uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const std::uint32_t*>(&h);
}

// B fragments (b0,b1 for the low-nibble MMA; c0,c1 for the high-nibble MMA)
// for one 32-element block, for one n8 tile.
template <bool XF32>
__device__ __forceinline__ void load_b(const Params& p, int tile, int g, int t,
                                       std::uint64_t kelem, std::uint32_t (&b)[4]) {
    if constexpr (!XF32) {
        const std::uint32_t m = tile * 8 + g;
        if (m < p.M) {
            const __half* xr = static_cast<const __half*>(p.x) + m * p.K + kelem + 4 * t;
            const uint2 a = __ldg(reinterpret_cast<const uint2*>(xr));
            const uint2 c = __ldg(reinterpret_cast<const uint2*>(xr + 16));
            b[0] = a.x;
            b[1] = a.y;
            b[2] = c.x;
            b[3] = c.y;
        } else {
            b[0] = b[1] = b[2] = b[3] = 0u;
        }
    } else {
        // Column g of the tile holds token tile*4 + g/2; even columns carry
        // the f16 rounding of x, odd columns the f16 rounding of the rest.
        const std::uint32_t m = tile * 4 + (g >> 1);
        if (m < p.M) {
            const float* xr = static_cast<const float*>(p.x) + m * p.K + kelem + 4 * t;
            float4 a = __ldg(reinterpret_cast<const float4*>(xr));
            float4 c = __ldg(reinterpret_cast<const float4*>(xr + 16));
            if (g & 1) {
                a.x -= __half2float(__float2half_rn(a.x));
                a.y -= __half2float(__float2half_rn(a.y));
                a.z -= __half2float(__float2half_rn(a.z));
                a.w -= __half2float(__float2half_rn(a.w));
                c.x -= __half2float(__float2half_rn(c.x));
                c.y -= __half2float(__float2half_rn(c.y));
                c.z -= __half2float(__float2half_rn(c.z));
                c.w -= __half2float(__float2half_rn(c.w));
            }
            b[0] = pack_half2(a.x, a.y);
            b[1] = pack_half2(a.z, a.w);
            b[2] = pack_half2(c.x, c.y);
            b[3] = pack_half2(c.z, c.w);
        } else {
            b[0] = b[1] = b[2] = b[3] = 0u;
        }
    }
}

// One Q4_0 block for rows g and g+8: decoded A fragments plus scales,
// multiplied into every n8 tile.
template <int NT, bool XF32>
__device__ __forceinline__ void block_mma(const Params& p, std::uint32_t qg, std::uint32_t qg8,
                                          float dg, float dg8, std::uint64_t kelem, int g, int t,
                                          float (&acc)[NT][4]) {
    std::uint32_t al01, al23, ah01, ah23, bl01, bl23, bh01, bh23;
    decode_word(qg, al01, al23, ah01, ah23);
    decode_word(qg8, bl01, bl23, bh01, bh23);
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        std::uint32_t b[4];
        load_b<XF32>(p, nt, g, t, kelem, b);
        float tmp[4];
        mma_16816(tmp, al01, bl01, al23, bl23, b[0], b[1], zero);
        mma_16816(tmp, ah01, bh01, ah23, bh23, b[2], b[3], tmp);
        acc[nt][0] = fmaf(dg, tmp[0], acc[nt][0]);
        acc[nt][1] = fmaf(dg, tmp[1], acc[nt][1]);
        acc[nt][2] = fmaf(dg8, tmp[2], acc[nt][2]);
        acc[nt][3] = fmaf(dg8, tmp[3], acc[nt][3]);
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    return g / (1.0f + expf(-g)) * u;
}

template <int NT, bool XF32, bool OF32, int EPI>
__global__ void __launch_bounds__(kThreads) q4_0_linear_mma_kernel(const Params p) {
    extern __shared__ __align__(128) std::uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;

    std::uint8_t* ring = smem + warp * kWarpRingBytes;
    std::uint64_t* bars =
        reinterpret_cast<std::uint64_t*>(smem + kWarps * kWarpRingBytes) + warp * kStages;

    // Source rows of this tile.
    const std::uint8_t* src_row = nullptr;
    if (lane < kTileRows) {
        if constexpr (EPI == kEpiSwiGLU) {
            const std::uint32_t f = min(blockIdx.x * 8u + (lane & 7), p.N - 1);
            src_row = (lane < 8 ? p.w : p.w2) + f * p.pitch;
        } else {
            const std::uint32_t r = min(blockIdx.x * 16u + lane, p.N - 1);
            src_row = p.w + r * p.pitch;
        }
    }

    const std::uint32_t u0 = (p.units * warp) / kWarps;
    const std::uint32_t u1 = (p.units * (warp + 1)) / kWarps;
    const std::uint32_t nstages = (u1 - u0 + kStageUnits - 1) / kStageUnits;

    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
        fence_mbarrier_init();
    }
    __syncwarp();

    const std::uint64_t policy = l2_evict_first_policy();
    auto issue = [&](std::uint32_t s) {
        const std::uint32_t ua = u0 + s * kStageUnits;
        const std::uint32_t nu = min(static_cast<std::uint32_t>(kStageUnits), u1 - ua);
        const std::uint32_t bytes = nu * kUnitBytes;
        std::uint64_t* bar = &bars[s % kStages];
        if (lane == 0) mbar_arrive_expect_tx(bar, bytes * kTileRows);
        __syncwarp();
        if (lane < kTileRows) {
            bulk_copy_g2s(ring + (s % kStages) * kStageBytes + lane * kRowStride,
                          src_row + static_cast<std::uint64_t>(ua) * kUnitBytes, bytes, bar,
                          policy);
        }
    };

    for (std::uint32_t s = 0; s < min(nstages, static_cast<std::uint32_t>(kStages)); ++s) issue(s);

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

    unsigned* status = &g_device_status;
    bool ok = true;
    for (std::uint32_t s = 0; s < nstages && ok; ++s) {
        const int slot = s % kStages;
        ok = mbar_wait_bounded(&bars[slot], (s / kStages) & 1u, status);
        if (!ok) break;
        const std::uint32_t ua = u0 + s * kStageUnits;
        const std::uint32_t nu = min(static_cast<std::uint32_t>(kStageUnits), u1 - ua);
        const std::uint8_t* rg = ring + slot * kStageBytes + g * kRowStride;
        const std::uint8_t* rg8 = rg + 8 * kRowStride;
        const std::uint64_t kbase = static_cast<std::uint64_t>(ua) * (kUnitBlocks * 32);
        const std::uint32_t npairs = nu * (kUnitBlocks / 2);
#pragma unroll 2
        for (std::uint32_t pr = 0; pr < npairs; ++pr) {
            const std::uint32_t* ra = reinterpret_cast<const std::uint32_t*>(rg + pr * 36);
            const std::uint32_t* rb = reinterpret_cast<const std::uint32_t*>(rg8 + pr * 36);
            const std::uint32_t a_d0 = ra[0], a_q0 = ra[t], a_q1 = ra[t + 1], a_d1 = ra[4],
                                a_q2 = ra[5 + t];
            const std::uint32_t b_d0 = rb[0], b_q0 = rb[t], b_q1 = rb[t + 1], b_d1 = rb[4],
                                b_q2 = rb[5 + t];
            const std::uint64_t ke = kbase + pr * 64;
            // even block of the pair (4-byte aligned)
            block_mma<NT, XF32>(p, prmt(a_q0, a_q1, 0x5432u), prmt(b_q0, b_q1, 0x5432u),
                                half_bits_to_float(a_d0 & 0xFFFFu),
                                half_bits_to_float(b_d0 & 0xFFFFu), ke, g, t, acc);
            // odd block of the pair (quant words are 4-byte aligned)
            block_mma<NT, XF32>(p, a_q2, b_q2, half_bits_to_float(a_d1 >> 16),
                                half_bits_to_float(b_d1 >> 16), ke + 32, g, t, acc);
        }
        __syncwarp();
        if (s + kStages < nstages) {
            fence_proxy_async_smem();
            issue(s + kStages);
        }
    }

    // Cross-warp reduction.  The rings are dead once every warp is past its
    // loop; reuse them for the partial sums.
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((warp * NT + nt) * 4 + i) * 32 + lane] = acc[nt][i];
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float v = acc[nt][i];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) v += red[((w * NT + nt) * 4 + i) * 32 + lane];
            acc[nt][i] = v;
        }

    // Epilogue.  Lane (g, t) holds rows g, g+8 and MMA columns 2t, 2t+1.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        if constexpr (EPI == kEpiSwiGLU) {
            const std::uint32_t f = blockIdx.x * 8u + g;
            if (f >= p.N) continue;
            if constexpr (!XF32) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const std::uint32_t m = nt * 8 + 2 * t + c;
                    if (m >= p.M) continue;
                    const float h = silu_mul(acc[nt][c], acc[nt][2 + c]);
                    if constexpr (OF32)
                        static_cast<float*>(p.y)[m * p.ldy + f] = h;
                    else
                        static_cast<__half*>(p.y)[m * p.ldy + f] = __float2half_rn(h);
                }
            } else {
                const std::uint32_t m = nt * 4 + t;
                if (m >= p.M) continue;
                const float h = silu_mul(acc[nt][0] + acc[nt][1], acc[nt][2] + acc[nt][3]);
                if constexpr (OF32)
                    static_cast<float*>(p.y)[m * p.ldy + f] = h;
                else
                    static_cast<__half*>(p.y)[m * p.ldy + f] = __float2half_rn(h);
            }
        } else {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const std::uint32_t r = blockIdx.x * 16u + g + 8 * half;
                if (r >= p.N) continue;
                if constexpr (!XF32) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const std::uint32_t m = nt * 8 + 2 * t + c;
                        if (m >= p.M) continue;
                        const float v = acc[nt][2 * half + c];
                        if constexpr (OF32)
                            static_cast<float*>(p.y)[m * p.ldy + r] = v;
                        else
                            static_cast<__half*>(p.y)[m * p.ldy + r] = __float2half_rn(v);
                    }
                } else {
                    const std::uint32_t m = nt * 4 + t;
                    if (m >= p.M) continue;
                    const float v = acc[nt][2 * half] + acc[nt][2 * half + 1];
                    if constexpr (OF32)
                        static_cast<float*>(p.y)[m * p.ldy + r] = v;
                    else
                        static_cast<__half*>(p.y)[m * p.ldy + r] = __float2half_rn(v);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Generic path: any K multiple of 32, any alignment.  One warp per output
// row and group of up to 8 tokens; lanes stride over blocks, decode bytes
// with scalar loads, accumulate in f32 and reduce with shuffles.
// ---------------------------------------------------------------------------
constexpr int kGenericTokens = 8;

template <bool XF32, bool OF32, int EPI>
__global__ void __launch_bounds__(128) q4_0_linear_generic_kernel(const Params p) {
    const std::uint32_t warp_global = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const std::uint32_t m0 = blockIdx.y * kGenericTokens;
    if (warp_global >= p.N) return;
    const std::uint64_t nb = p.K / 32;
    float acc[2][kGenericTokens];
#pragma unroll
    for (int j = 0; j < kGenericTokens; ++j) acc[0][j] = acc[1][j] = 0.f;
    const int nmat = EPI == kEpiSwiGLU ? 2 : 1;
    for (int mat = 0; mat < nmat; ++mat) {
        const std::uint8_t* row = (mat == 0 ? p.w : p.w2) + warp_global * p.pitch;
        for (std::uint64_t b = lane; b < nb; b += 32) {
            const std::uint8_t* blk = row + b * 18;
            const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
            float wv[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const std::uint8_t q = blk[2 + j];
                wv[j] = static_cast<float>(static_cast<int>(q & 15) - 8) * d;
                wv[j + 16] = static_cast<float>(static_cast<int>(q >> 4) - 8) * d;
            }
#pragma unroll
            for (int mm = 0; mm < kGenericTokens; ++mm) {
                const std::uint32_t m = m0 + mm;
                if (m >= p.M) break;
                float s = 0.f;
                if constexpr (XF32) {
                    const float* xr = static_cast<const float*>(p.x) + m * p.K + b * 32;
#pragma unroll
                    for (int j = 0; j < 32; ++j) s = fmaf(xr[j], wv[j], s);
                } else {
                    const __half* xr = static_cast<const __half*>(p.x) + m * p.K + b * 32;
#pragma unroll
                    for (int j = 0; j < 32; ++j) s = fmaf(__half2float(xr[j]), wv[j], s);
                }
                acc[mat][mm] += s;
            }
        }
    }
#pragma unroll
    for (int mm = 0; mm < kGenericTokens; ++mm) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            acc[0][mm] += __shfl_xor_sync(0xffffffffu, acc[0][mm], off);
            acc[1][mm] += __shfl_xor_sync(0xffffffffu, acc[1][mm], off);
        }
    }
    if (lane != 0) return;
#pragma unroll
    for (int mm = 0; mm < kGenericTokens; ++mm) {
        const std::uint32_t m = m0 + mm;
        if (m >= p.M) break;
        float v = acc[0][mm];
        if constexpr (EPI == kEpiSwiGLU) v = silu_mul(acc[0][mm], acc[1][mm]);
        if constexpr (OF32)
            static_cast<float*>(p.y)[m * p.ldy + warp_global] = v;
        else
            static_cast<__half*>(p.y)[m * p.ldy + warp_global] = __float2half_rn(v);
    }
}

// ---------------------------------------------------------------------------
// Host dispatch
// ---------------------------------------------------------------------------
// Opts a kernel into more than 48 KB of dynamic shared memory, once per
// device (the attribute is per device; `done` is a bit mask of ordinals).
template <typename Kernel>
int ensure_smem_attribute(Kernel kernel, int bytes, std::atomic<std::uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    const std::uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return kSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    done.fetch_or(bit, std::memory_order_acq_rel);
    return kSuccess;
}

template <int NT, bool XF32, bool OF32, int EPI>
int launch_mma(const Params& p, std::uint32_t grid, cudaStream_t stream) {
    auto kernel = q4_0_linear_mma_kernel<NT, XF32, OF32, EPI>;
    static std::atomic<std::uint64_t> configured{0};
    const int st = ensure_smem_attribute(kernel, kSmemBytes, configured);
    if (st != kSuccess) return st;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

template <bool XF32, bool OF32, int EPI>
int launch_mma_nt(const Params& p, std::uint32_t grid, cudaStream_t stream) {
    const std::uint32_t per_tile = XF32 ? 4 : 8;
    const std::uint32_t tiles = (p.M + per_tile - 1) / per_tile;
    if (tiles <= 1) return launch_mma<1, XF32, OF32, EPI>(p, grid, stream);
    if (tiles <= 2) return launch_mma<2, XF32, OF32, EPI>(p, grid, stream);
    if (tiles <= 4) return launch_mma<4, XF32, OF32, EPI>(p, grid, stream);
    return launch_mma<8, XF32, OF32, EPI>(p, grid, stream);
}

// Runs the linear for M rows of x.  Token groups beyond what one launch
// covers (64 f16 tokens / 32 f32 tokens) are processed in consecutive
// launches on the same stream.
template <bool XF32, bool OF32, int EPI>
int run_linear(const void* x, const void* w, const void* w2, void* y, std::uint64_t M,
               std::uint64_t N, std::uint64_t K, std::uint64_t ldy, cudaStream_t stream) {
    if (K == 0) {
        // Every dot product is empty: the reference writes zeros
        // (crates/mote-backend-hip/tests/quantized_linear.rs:142-158).  For
        // SwiGLU silu(0) * 0 = 0 as well.
        const std::size_t esz = OF32 ? 4 : 2;
        const cudaError_t e = cudaMemset2DAsync(y, ldy * esz, 0, N * esz, M, stream);
        return static_cast<int>(e);
    }
    Params p{};
    p.x = x;
    p.w = static_cast<const std::uint8_t*>(w);
    p.w2 = static_cast<const std::uint8_t*>(w2);
    p.y = y;
    p.N = static_cast<std::uint32_t>(N);
    p.K = K;
    p.pitch = (K / 32) * 18;
    p.units = static_cast<std::uint32_t>(K / 256);
    p.ldy = ldy;
    const std::size_t xes = XF32 ? 4 : 2;
    bool fast = (K % 256 == 0) && (reinterpret_cast<std::uintptr_t>(w) % 16 == 0) &&
                (reinterpret_cast<std::uintptr_t>(x) % (XF32 ? 16 : 8) == 0);
    if (EPI == kEpiSwiGLU) fast = fast && (reinterpret_cast<std::uintptr_t>(w2) % 16 == 0);
    const std::uint64_t chunk = fast ? (XF32 ? 32 : 64) : kGenericTokens * 65535ull;
    for (std::uint64_t m0 = 0; m0 < M; m0 += chunk) {
        const std::uint64_t mc = (M - m0 < chunk) ? (M - m0) : chunk;
        p.M = static_cast<std::uint32_t>(mc);
        p.x = static_cast<const std::uint8_t*>(x) + m0 * K * xes;
        p.y = static_cast<std::uint8_t*>(y) + m0 * ldy * (OF32 ? 4 : 2);
        int st;
        if (fast) {
            const std::uint64_t rows_per_tile = EPI == kEpiSwiGLU ? 8 : 16;
            const std::uint64_t grid = (N + rows_per_tile - 1) / rows_per_tile;
            st = launch_mma_nt<XF32, OF32, EPI>(p, static_cast<std::uint32_t>(grid), stream);
        } else {
            const dim3 grid(static_cast<unsigned>((N + 3) / 4),
                            static_cast<unsigned>((mc + kGenericTokens - 1) / kGenericTokens));
            q4_0_linear_generic_kernel<XF32, OF32, EPI><<<grid, 128, 0, stream>>>(p);
            st = static_cast<int>(cudaGetLastError());
        }
        if (st != 0) return st;
    }
    return kSuccess;
}

// Argument checks of mote_hip_quantized_linear_q4_0_f16
// (crates/mote-backend-hip/src/quantized_linear.hip:64-76): null pointers
// (stream included) and K not a multiple of 32 are invalid values, empty
// outputs succeed without a launch, and rows*N must fit the reference's
// one-block-per-output 32-bit grid.
inline int check_linear_args(const void* x, const void* w, const void* y, std::uint64_t rows,
                             std::uint64_t n, std::uint64_t k, const void* stream) {
    if (x == nullptr || w == nullptr || y == nullptr || stream == nullptr) return kInvalidValue;
    if (k % 32 != 0) return kInvalidValue;
    if (rows == 0 || n == 0) return -2;  // empty: success without launch
    if (rows > 0xffffffffull || n > 0xffffffffull || rows > 0xffffffffull / n)
        return kInvalidConfiguration;
    return kSuccess;
}

}  // namespace q4
}  // namespace mote

extern "C" int mote_cuda_quantized_linear_q4_0_f16(const void* input, const void* weights,
                                                   void* output, std::uint64_t rows,
                                                   std::uint64_t output_features,
                                                   std::uint64_t input_features, void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == -2) return mote::kSuccess;
    if (c != 0) return c;
    return run_linear<false, false, kEpiPlain>(input, weights, nullptr, output, rows,
                                               output_features, input_features, output_features,
                                               static_cast<cudaStream_t>(stream));
}

extern "C" int mote_cuda_quantized_linear_q4_0_f16_f32out(const void* input, const void* weights,
                                                          void* output, std::uint64_t rows,
                                                          std::uint64_t output_features,
                                                          std::uint64_t input_features,
                                                          void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == -2) return mote::kSuccess;
    if (c != 0) return c;
    return run_linear<false, true, kEpiPlain>(input, weights, nullptr, output, rows,
                                              output_features, input_features, output_features,
                                              static_cast<cudaStream_t>(stream));
}

extern "C" int mote_cuda_quantized_linear_q4_0_f32(const void* input, const void* weights,
                                                   void* output, std::uint64_t rows,
                                                   std::uint64_t output_features,
                                                   std::uint64_t input_features, void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == -2) return mote::kSuccess;
    if (c != 0) return c;
    return run_linear<true, true, kEpiPlain>(input, weights, nullptr, output, rows,
                                             output_features, input_features, output_features,
                                             static_cast<cudaStream_t>(stream));
}

extern "C" int mote_cuda_q4_0_gate_up_swiglu_f16(const void* input, const void* gate_weights,
                                                 const void* up_weights, void* output,
                                                 std::uint64_t rows, std::uint64_t ffn_features,
                                                 std::uint64_t input_features, void* stream) {
    using namespace mote::q4;
    if (up_weights == nullptr) return mote::kInvalidValue;
    const int c = check_linear_args(input, gate_weights, output, rows, ffn_features,
                                    input_features, stream);
    if (c == -2) return mote::kSuccess;
    if (c != 0) return c;
    return run_linear<false, false, kEpiSwiGLU>(input, gate_weights, up_weights, output, rows,
                                                ffn_features, input_features, ffn_features,
                                                static_cast<cudaStream_t>(stream));
}
