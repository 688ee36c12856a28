// Q8_0 weight-only linear for decode: Y[M, N] = X[M, K] * W[N, K]^T with
// X f16, W ggml Q8_0 (per 32 elements: little-endian f16 scale d, then 32
// signed bytes; value = q * d), f32 accumulation, f16 or f32 out.  The
// device counterpart of mote-reference's quantized_linear_f32 for Q8_0
// (crates/mote-reference/src/quantized.rs:89-144, decode :191-195); the HIP
// backend has no Q8_0 linear.
//
// Same shape of kernel as the Q4_0 GEMV (q4_0_linear.cu), simpler decode:
// * persistent 8-warp CTAs walk 16-row weight tiles; the warps of a CTA form
//   8/S groups of S warps that split a tile's K (S from the same measured
//   rule as the Q4_0 kernel);
// * each warp streams its K-slice of 16 rows through a private cp.async ring
//   of 272-byte rows (8 blocks = 17 x 16 bytes; word t of row g sits in bank
//   4g + t, conflict-free);
// * lane (g, t) reads quant word t of each 16-byte half of a block for rows
//   g and g + 8 -- elements 4t..4t+3 -- and makes them the MMA k positions
//   {2t, 2t+1, 2t+8, 2t+9}; its B fragment is then the 8 consecutive bytes
//   of activations 4t..4t+3, so the activations are staged unpermuted;
// * decode is exact: (q ^ 0x80) is a byte u = q + 128, one PRMT places two
//   of them under the f16 exponent of 1024 (f16(1024 + u)), and one f16x2
//   subtraction of 1152 gives q;
// * mma.sync.m16n8k16 (f16 x f16 -> f32) per 16-k step, with the 8 columns
//   the tokens; each block's partial is scaled by its row's f32 d.
// More than 16 tokens run on the tcgen05 GEMM (q4_0_gemm_tcgen05.cu, Q8_0
// conversion) when N % 16 == 0, K % 256 == 0 and the pointers are aligned,
// else as consecutive launches of up to 16.  Shapes the fast path does not
// take (K % 256 != 0, unaligned pointers) run a plain warp-per-row kernel.

namespace mote {
namespace q8 {

using q4::kThreads;
using q4::kWarps;
constexpr int kTileRows = 16;
constexpr int kBlockBytes = 34;
constexpr int kUnitBlocks = 8;                          // 256 elements
constexpr int kUnitBytes = kUnitBlocks * kBlockBytes;   // 272 = 17 x 16
constexpr int kRowStride = kUnitBytes;                  // 68 words: 4 banks apart
constexpr int kStageBytes = kTileRows * kRowStride;     // 4352
constexpr int kChunksPerRow = kUnitBytes / 16;          // 17
constexpr int kChunks = kTileRows * kChunksPerRow;      // 272
constexpr int kChunksPerLane = (kChunks + 31) / 32;     // 9
constexpr int kMaxTokens = 16;                          // two n8 tiles

struct Params {
    const __half* x;         // [M, K]
    const std::uint8_t* w;   // [N, K/32*34]
    void* y;                 // [M, N]
    std::uint32_t M;         // tokens in this launch (<= 16 on the fast path)
    std::uint32_t N;
    std::uint64_t K;
    std::uint64_t pitch;     // bytes per weight row
    std::uint32_t units;     // K / 256
    std::uint32_t tiles;     // 16-row tiles
    std::uint32_t x_stride;  // bytes per staged activation row (2K + 32)
    std::uint32_t x_bytes;   // staged rows + the zero row, rounded up to 128
    std::uint32_t split_shift;
};

__host__ __device__ constexpr int red_bytes(int nt) { return 2 * kWarps * nt * 4 * 32 * 4; }
__host__ __device__ constexpr int smem_bytes(int x_bytes, int nt, int stages) {
    return x_bytes + kWarps * stages * kStageBytes + red_bytes(nt);
}

// Quant word u = bytes q0..q3 (signed) -> f16 pairs (q0, q1) and (q2, q3).
__device__ __forceinline__ void decode_word8(std::uint32_t u, std::uint32_t& lo,
                                             std::uint32_t& hi) {
    const std::uint32_t v = u ^ 0x80808080u;  // q + 128 per byte
    lo = hsub2_u32(prmt(v, 0x64646464u, 0x4140u), 0x64806480u);
    hi = hsub2_u32(prmt(v, 0x64646464u, 0x4342u), 0x64806480u);
}

template <int NT, bool OF32>
__device__ __forceinline__ void store_tile8(const Params& p, std::uint32_t tile, int g, int t,
                                            const float (&acc)[NT][4]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const std::uint32_t r = tile * 16u + g + 8 * half;
            if (r >= p.N) continue;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const std::uint32_t m = nt * 8 + 2 * t + c;
                if (m >= p.M) continue;
                const float v = acc[nt][2 * half + c];
                if constexpr (OF32)
                    static_cast<float*>(p.y)[static_cast<std::uint64_t>(m) * p.N + r] = v;
                else
                    static_cast<__half*>(p.y)[static_cast<std::uint64_t>(m) * p.N + r] =
                        __float2half_rn(v);
            }
        }
}

template <int NT, bool OF32, int STAGES>
__global__ void __launch_bounds__(kThreads, 2) q8_0_gemv_kernel(const Params p) {
    extern __shared__ __align__(1024) std::uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    std::uint8_t* xs = smem;
    std::uint8_t* ring = smem + p.x_bytes + warp * STAGES * kStageBytes;
    float* red = reinterpret_cast<float*>(smem + p.x_bytes + kWarps * STAGES * kStageBytes);

    // groups of `split` warps walk tiles first, first + stride, ...; warp
    // wig of a group owns units [u0, u1) of each
    const std::uint32_t sh = p.split_shift;
    const std::uint32_t split = 1u << sh;
    const std::uint32_t grp = static_cast<std::uint32_t>(warp) >> sh;
    const std::uint32_t wig = static_cast<std::uint32_t>(warp) & (split - 1);
    const std::uint32_t first = blockIdx.x + grp * gridDim.x;
    const std::uint32_t stride = gridDim.x * (kWarps >> sh);
    const std::uint32_t my_tiles = p.tiles > first ? (p.tiles - first + stride - 1) / stride : 0;
    const std::uint32_t u0 = (p.units * wig) >> sh;
    const std::uint32_t u1 = (p.units * (wig + 1)) >> sh;
    const std::uint32_t spt = u1 - u0;
    const std::uint32_t total = my_tiles * spt;
    const std::uint64_t policy = l2_evict_first_policy();

    // stage chunk c (16 bytes): row c / 17, column chunk c % 17
    std::uint32_t dst_off[kChunksPerLane];
    std::uint32_t src_off[kChunksPerLane];
    std::uint32_t chunk_row[kChunksPerLane];
#pragma unroll
    for (int j = 0; j < kChunksPerLane; ++j) {
        const int c = min(lane + 32 * j, kChunks - 1);
        chunk_row[j] = static_cast<std::uint32_t>(c / kChunksPerRow);
        dst_off[j] = chunk_row[j] * kRowStride + (c % kChunksPerRow) * 16;
        src_off[j] = (c % kChunksPerRow) * 16;
    }
    const std::uint32_t ring_s = smem_u32(ring);
    std::uint32_t iss_n = 0, iss_tl = 0, iss_u = 0, iss_slot = 0;
    const std::uint8_t* src[kChunksPerLane];
    auto seek_tile = [&](std::uint32_t tl) {
        const std::uint64_t row0 = static_cast<std::uint64_t>(first + tl * stride) * kTileRows;
#pragma unroll
        for (int j = 0; j < kChunksPerLane; ++j) {
            // rows past N (the ragged last tile) re-read the last row; their
            // results are never stored
            const std::uint64_t r = min(row0 + chunk_row[j], static_cast<std::uint64_t>(p.N - 1));
            src[j] = p.w + r * p.pitch + static_cast<std::uint64_t>(u0) * kUnitBytes + src_off[j];
        }
    };
    if (total > 0) seek_tile(0);
    auto issue = [&]() {
        if (iss_n < total) {
            const std::uint32_t slot_s = ring_s + iss_slot * kStageBytes;
#pragma unroll
            for (int j = 0; j < kChunksPerLane; ++j)
                if (lane + 32 * j < kChunks) cp_async_16(slot_s + dst_off[j], src[j], policy);
            if (++iss_u == spt) {
                iss_u = 0;
                if (iss_n + 1 < total) seek_tile(++iss_tl);
            } else {
#pragma unroll
                for (int j = 0; j < kChunksPerLane; ++j) src[j] += kUnitBytes;
            }
        }
        ++iss_n;
        iss_slot = iss_slot + 1 == STAGES ? 0 : iss_slot + 1;
        cp_async_commit();
    };
    // weights first (they do not depend on earlier kernels), then wait for
    // the activations
    for (int s = 0; s + 1 < STAGES; ++s) issue();
    pdl_launch_dependents();
    pdl_wait();

    // stage the activation rows (unpermuted) and one all-zero row
    {
        const std::uint32_t vec_per_row = static_cast<std::uint32_t>(p.K / 8);
        const std::uint32_t nvec = p.M * vec_per_row;
        for (std::uint32_t i = threadIdx.x; i < nvec; i += kThreads) {
            const std::uint32_t m = i / vec_per_row;
            const std::uint32_t v = i - m * vec_per_row;
            const uint4 val = __ldg(reinterpret_cast<const uint4*>(p.x + m * p.K) + v);
            *reinterpret_cast<uint4*>(xs + m * p.x_stride + 16 * v) = val;
        }
        for (std::uint32_t i = threadIdx.x; i < p.x_stride / 16; i += kThreads)
            *reinterpret_cast<uint4*>(xs + p.M * p.x_stride + 16 * i) = make_uint4(0u, 0u, 0u, 0u);
        __syncthreads();
    }

    // B rows of this lane: token nt*8 + g, or the zero row
    std::uint32_t xsel[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const std::uint32_t m = nt * 8 + g;
        xsel[nt] = smem_u32(xs) + (m < p.M ? m : p.M) * p.x_stride + 8 * t;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    constexpr std::uint32_t kR8 = 8 * kRowStride;
    std::uint32_t slot = 0;
    for (std::uint32_t tl = 0; tl < my_tiles; ++tl) {
        for (std::uint32_t st = 0; st < spt; ++st) {
            issue();
            cp_async_wait<STAGES - 1>();
            __syncwarp();
            const std::uint32_t ra = ring_s + slot * kStageBytes + g * kRowStride;  // row g
            const std::uint32_t qa = ra + 4 * t;
            const std::uint32_t xo = (u0 + st) * (kUnitBlocks * 64);
            q4::static_for<0, kUnitBlocks>([&](auto bb) {
                constexpr int b = decltype(bb)::value;
                constexpr int q0 = kBlockBytes * b + 2;  // block b's quants in the row
                // word t of each 16-byte half, rows g and g + 8: aligned for
                // odd b, straddling two words for even b
                std::uint32_t w[2][2];  // [half][row g, g+8]
                if constexpr (b & 1) {
                    w[0][0] = lds32i<q0>(qa);
                    w[0][1] = lds32i<kR8 + q0>(qa);
                    w[1][0] = lds32i<q0 + 16>(qa);
                    w[1][1] = lds32i<kR8 + q0 + 16>(qa);
                } else {
                    w[0][0] = prmt(lds32i<q0 - 2>(qa), lds32i<q0 + 2>(qa), 0x5432u);
                    w[0][1] = prmt(lds32i<kR8 + q0 - 2>(qa), lds32i<kR8 + q0 + 2>(qa),
                                   0x5432u);
                    w[1][0] = prmt(lds32i<q0 + 14>(qa), lds32i<q0 + 18>(qa), 0x5432u);
                    w[1][1] = prmt(lds32i<kR8 + q0 + 14>(qa), lds32i<kR8 + q0 + 18>(qa),
                                   0x5432u);
                }
                std::uint32_t a[2][4];  // [half][a0..a3]
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    decode_word8(w[h][0], a[h][0], a[h][2]);
                    decode_word8(w[h][1], a[h][1], a[h][3]);
                }
                const float dg = half_bits_to_float(lds16i<kBlockBytes * b>(ra));
                const float dh = half_bits_to_float(lds16i<kR8 + kBlockBytes * b>(ra));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
                    const uint2 x0 = lds64(xsel[nt] + xo + 64 * b);
                    const uint2 x1 = lds64(xsel[nt] + xo + 64 * b + 32);
                    mma_16816(d, a[0][0], a[0][1], a[0][2], a[0][3], x0.x, x0.y, d);
                    mma_16816(d, a[1][0], a[1][1], a[1][2], a[1][3], x1.x, x1.y, d);
                    acc[nt][0] = fmaf(dg, d[0], acc[nt][0]);
                    acc[nt][1] = fmaf(dg, d[1], acc[nt][1]);
                    acc[nt][2] = fmaf(dh, d[2], acc[nt][2]);
                    acc[nt][3] = fmaf(dh, d[3], acc[nt][3]);
                }
            });
            __syncwarp();  // the slot is refilled by the next iteration's issue
            slot = slot + 1 == STAGES ? 0 : slot + 1;
        }
        const std::uint32_t tile = first + tl * stride;
        if (split == 1) {
            store_tile8<NT, OF32>(p, tile, g, t, acc);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
            continue;
        }
        // the group's K-slices meet in its double-buffered reduction area
        float* gred = red + grp * 2 * split * (NT * 4 * 32);
        float* mine = gred + ((tl & 1u) * split + wig) * (NT * 4 * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                mine[(nt * 4 + i) * 32 + lane] = acc[nt][i];
                acc[nt][i] = 0.f;
            }
        q4::named_barrier_sync(1 + static_cast<int>(grp), static_cast<int>(split) * 32);
        if ((tl & (split - 1)) == wig) {
            float sum[NT][4];
            const float* base = gred + (tl & 1u) * split * (NT * 4 * 32);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sum[nt][i] = 0.f;
            for (std::uint32_t wi = 0; wi < split; ++wi)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        sum[nt][i] += base[wi * (NT * 4 * 32) + (nt * 4 + i) * 32 + lane];
            store_tile8<NT, OF32>(p, tile, g, t, sum);
        }
    }
}

// Any K multiple of 32, any alignment: one warp per output row and group of
// up to 8 tokens, lanes striding over blocks, f32 accumulation.
constexpr int kGenericTokens = 8;

template <bool OF32>
__global__ void __launch_bounds__(128) q8_0_linear_generic_kernel(const Params p) {
    pdl_launch_dependents();
    pdl_wait();
    const std::uint32_t row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const std::uint32_t m0 = blockIdx.y * kGenericTokens;
    if (row >= p.N) return;
    const std::uint64_t nb = p.K / 32;
    float acc[kGenericTokens];
#pragma unroll
    for (int j = 0; j < kGenericTokens; ++j) acc[j] = 0.f;
    const std::uint8_t* wrow = p.w + row * p.pitch;
    for (std::uint64_t b = lane; b < nb; b += 32) {
        const std::uint8_t* blk = wrow + b * kBlockBytes;
        const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
#pragma unroll
        for (int mm = 0; mm < kGenericTokens; ++mm) {
            const std::uint32_t m = m0 + mm;
            if (m >= p.M) break;
            const __half* xr = p.x + m * p.K + b * 32;
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                s = fmaf(__half2float(xr[j]),
                         static_cast<float>(static_cast<std::int8_t>(blk[2 + j])) * d, s);
            acc[mm] += s;
        }
    }
#pragma unroll
    for (int mm = 0; mm < kGenericTokens; ++mm)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[mm] += __shfl_xor_sync(0xffffffffu, acc[mm], off);
    if (lane != 0) return;
#pragma unroll
    for (int mm = 0; mm < kGenericTokens; ++mm) {
        const std::uint32_t m = m0 + mm;
        if (m >= p.M) break;
        if constexpr (OF32)
            static_cast<float*>(p.y)[static_cast<std::uint64_t>(m) * p.N + row] = acc[mm];
        else
            static_cast<__half*>(p.y)[static_cast<std::uint64_t>(m) * p.N + row] =
                __float2half_rn(acc[mm]);
    }
}

// ---- host ----------------------------------------------------------------------
template <int NT, bool OF32, int STAGES>
int launch_gemv8(const Params& p, int ctas_per_sm, cudaStream_t stream) {
    auto kernel = q8_0_gemv_kernel<NT, OF32, STAGES>;
    static std::atomic<std::uint64_t> configured{0};
    const int st = q4::ensure_smem_attribute(kernel, q4::kMaxSmem, configured);
    if (st != kSuccess) return st;
    const std::uint32_t groups = kWarps >> p.split_shift;
    const std::uint32_t cap = static_cast<std::uint32_t>(q4::sm_count() * ctas_per_sm);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(min((p.tiles + groups - 1) / groups, cap));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes(static_cast<int>(p.x_bytes), NT, STAGES);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <bool OF32>
int run_linear8(const void* x, const void* w, void* y, std::uint64_t M, std::uint64_t N,
                std::uint64_t K, cudaStream_t stream) {
    const std::size_t osz = OF32 ? 4 : 2;
    if (K == 0)  // every dot product is empty: zeros, as the reference
        return static_cast<int>(cudaMemsetAsync(y, 0, M * N * osz, stream));
    // prefill-shaped problems: the tcgen05 GEMM with Q8_0 conversion
    if (M > static_cast<std::uint64_t>(kMaxTokens) && gemm::supported(x, w, y, M, N, K, osz))
        return gemm::launch<OF32, gemm::kWQ8_0>(x, w, y, M, N, K, stream);
    Params p{};
    p.w = static_cast<const std::uint8_t*>(w);
    p.N = static_cast<std::uint32_t>(N);
    p.K = K;
    p.pitch = (K / 32) * kBlockBytes;
    p.units = static_cast<std::uint32_t>(K / 256);
    p.tiles = static_cast<std::uint32_t>((N + kTileRows - 1) / kTileRows);
    const bool fast = K % 256 == 0 && K <= (1ull << 24) &&
                      reinterpret_cast<std::uintptr_t>(x) % 16 == 0 &&
                      reinterpret_cast<std::uintptr_t>(w) % 16 == 0;
    // tokens per launch, ring depth and CTAs per SM: two CTAs per SM with
    // the deepest ring that fits, else one.  A Q8_0 stage is 4352 bytes, so
    // two CTAs with two stages each (one stage in flight per warp, 16 warps
    // per SM) beat one CTA with four: 97.5 vs 108.4 us for the 558 MB M=1
    // lm_head.
    std::uint32_t tokens = 0;
    int stages = 2, ctas = 1;
    if (fast) {
        p.x_stride = static_cast<std::uint32_t>(K * 2 + 32);
        for (std::uint32_t m = static_cast<std::uint32_t>(M < kMaxTokens ? M : kMaxTokens);
             m >= 1 && tokens == 0; m /= 2) {
            const std::uint32_t xb = ((m + 1) * p.x_stride + 127u) & ~127u;
            const int nt = m > 8 ? 2 : 1;
            constexpr int kOptions[5][2] = {{2, 4}, {2, 3}, {2, 2}, {1, 4}, {1, 2}};
            for (const auto& opt : kOptions) {
                const int bytes = smem_bytes(static_cast<int>(xb), nt, opt[1]);
                if (bytes <= q4::kMaxSmem &&
                    opt[0] * (bytes + q4::kSmemReservedPerCta) <= q4::kSmemPerSm) {
                    tokens = m;
                    ctas = opt[0];
                    stages = opt[1];
                    p.x_bytes = xb;
                    break;
                }
            }
        }
    }
    const std::uint64_t chunk = tokens ? tokens : kGenericTokens * 65535ull;
    if (tokens)
        p.split_shift = q4::choose_split_shift(
            p.tiles, p.units, static_cast<std::uint32_t>(q4::sm_count() * ctas), 1);
    for (std::uint64_t m0 = 0; m0 < M; m0 += chunk) {
        const std::uint64_t mc = M - m0 < chunk ? M - m0 : chunk;
        p.M = static_cast<std::uint32_t>(mc);
        p.x = static_cast<const __half*>(x) + m0 * K;
        p.y = static_cast<std::uint8_t*>(y) + m0 * N * osz;
        int st;
        if (tokens) {
            const bool two = mc > 8;
            switch (stages) {
                case 4:
                    st = two ? launch_gemv8<2, OF32, 4>(p, ctas, stream)
                             : launch_gemv8<1, OF32, 4>(p, ctas, stream);
                    break;
                case 3:
                    st = two ? launch_gemv8<2, OF32, 3>(p, ctas, stream)
                             : launch_gemv8<1, OF32, 3>(p, ctas, stream);
                    break;
                default:
                    st = two ? launch_gemv8<2, OF32, 2>(p, ctas, stream)
                             : launch_gemv8<1, OF32, 2>(p, ctas, stream);
            }
        } else {
            const dim3 grid(static_cast<unsigned>((N + 3) / 4),
                            static_cast<unsigned>((mc + kGenericTokens - 1) / kGenericTokens));
            st = launch_pdl(q8_0_linear_generic_kernel<OF32>, grid, dim3(128), stream, p);
        }
        if (st != 0) return st;
    }
    return kSuccess;
}

}  // namespace q8
}  // namespace mote

// f16 activations, f16 output.  No HIP counterpart (the HIP backend has a
// Q4_0 linear only); argument rules as mote_cuda_quantized_linear_q4_0_f16.
extern "C" int mote_cuda_quantized_linear_q8_0_f16(const void* input, const void* weights,
                                                   void* output, std::uint64_t rows,
                                                   std::uint64_t output_features,
                                                   std::uint64_t input_features, void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    return mote::q8::run_linear8<false>(input, weights, output, rows, output_features,
                                        input_features, static_cast<cudaStream_t>(stream));
}

// The same with an f32 output (the accumulator unrounded).
extern "C" int mote_cuda_quantized_linear_q8_0_f16_f32out(const void* input, const void* weights,
                                                          void* output, std::uint64_t rows,
                                                          std::uint64_t output_features,
                                                          std::uint64_t input_features,
                                                          void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    return mote::q8::run_linear8<true>(input, weights, output, rows, output_features,
                                       input_features, static_cast<cudaStream_t>(stream));
}
