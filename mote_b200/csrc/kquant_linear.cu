// K-quant (ggml Q4_K / Q6_K, 256-element super-blocks) weight-only linear
// and device decode.  mote-reference fixes the geometry of these formats
// (crates/mote-types/src/lib.rs:41-74: Q4_K 144 bytes, Q6_K 210 bytes per
// 256 elements) and rejects them in its linear (quantized.rs:152-157); the
// arithmetic follows ggml's published dequantization:
//   Q4_K  value = (d * sc) * q - (dmin * m), q in 0..15, 6-bit sc / m per 32
//         elements, packed in 12 bytes;
//   Q6_K  value = (d * sc) * q, q in -32..31, one int8 sc per 16 elements.
//
// Q4_K decode GEMV (1-16 tokens, K % 256 == 0, 16-byte aligned x and W): the
// Q8_0 kernel's structure (persistent 8-warp CTAs, split-K warp groups,
// per-warp cp.async ring of 16 rows x one 144-byte super-block), with
// * the 6-bit scale folded into the decode: a nibble q becomes f16 1024 + q
//   (low) or 64 + q (high) by a LOP3, and one f16x2 FMA, sc * that - 1024 sc
//   (or 64 sc), gives sc * q exactly (at most 945), so the 16 MMAs of a
//   super-block accumulate sum_s sc_s * q . x in one f32 accumulator;
// * the mins as one more MMA per super-block: A holds m_s (exact f16
//   integers) twice, B the per-token sums of x over each 32-element sub-block
//   split into f16 hi + lo (staged with the activations), so the MMA returns
//   sum_s m_s * xsum_s to ~2^-22;
// * y += d * acc - dmin * mins, f32.
// Quant byte l of 32-byte group c holds elements 64c + l (low nibble) and
// 64c + 32 + l (high nibble): lane (g, t) takes word t of each 16-byte half of
// a group, four consecutive elements per nibble plane.  A LOP3 on the word
// (and on the word >> 8) gives the pairs of elements (4t, 4t+2) and (4t+1,
// 4t+3), so the activations are staged with elements 1 and 2 of every group
// of four swapped and B stays one 8-byte load (the MMA k positions {2t, 2t+1,
// 2t+8, 2t+9} take elements 4t, 4t+2, 4t+1, 4t+3 of each 16-element step).
// The Q6_K GEMV (K % 2048 == 0) is described above its kernel; other shapes
// run a warp-per-row kernel with f32 accumulation.

namespace mote {
namespace kq {

using q4::kThreads;
using q4::kWarps;
constexpr int kQ4K = 2;  // format ids as oracle / mote-types order them
constexpr int kQ6K = 3;
constexpr int kTileRows = 16;
constexpr int kBlockBytes = 144;                      // Q4_K super-block
constexpr int kRowStride = kBlockBytes;               // 36 words: rows 4 banks apart
constexpr int kStageBytes = kTileRows * kRowStride;   // 2304
constexpr int kChunksPerRow = kBlockBytes / 16;       // 9
constexpr int kChunks = kTileRows * kChunksPerRow;    // 144
constexpr int kChunksPerLane = (kChunks + 31) / 32;   // 5
constexpr int kMaxTokens = 16;

__host__ __device__ constexpr int block_bytes(int fmt) { return fmt == kQ4K ? 144 : 210; }

struct Params {
    const __half* x;         // [M, K]
    const std::uint8_t* w;   // [N, K/256 * block bytes]
    void* y;                 // [M, N]
    std::uint32_t M;         // tokens in this launch
    std::uint32_t N;
    std::uint64_t K;
    std::uint64_t pitch;     // bytes per weight row
    std::uint32_t units;     // K / 256
    std::uint32_t tiles;     // 16-row tiles
    std::uint32_t x_stride;  // bytes per staged activation row (2K + 32)
    std::uint32_t x_bytes;   // staged rows + the zero row, rounded up to 128
    std::uint32_t s_stride;  // bytes per row of sub-block sums (4 * (K/32 + 4))
    std::uint32_t s_bytes;
    std::uint32_t split_shift;
};

__host__ __device__ constexpr int red_bytes(int nt) { return 2 * kWarps * nt * 4 * 32 * 4; }
__host__ __device__ constexpr int smem_bytes(int x_bytes, int s_bytes, int nt, int stages) {
    return x_bytes + s_bytes + kWarps * stages * kStageBytes + red_bytes(nt);
}

__device__ __forceinline__ std::uint32_t hfma2_u32(std::uint32_t a, std::uint32_t b,
                                                   std::uint32_t c) {
    std::uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ std::uint32_t hmul2_u32(std::uint32_t a, std::uint32_t b) {
    std::uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint4 lds128(std::uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

// The 6-bit scales (sc) and mins (m) of sub-blocks 0-3 and 4-7, one per byte,
// from the 12 packed bytes (h.y = bytes 0-3, h.z = 4-7, h.w = 8-11).
__device__ __forceinline__ void unpack_scales(const uint4& h, std::uint32_t& sc03,
                                              std::uint32_t& sc47, std::uint32_t& m03,
                                              std::uint32_t& m47) {
    sc03 = h.y & 0x3F3F3F3Fu;
    m03 = h.z & 0x3F3F3F3Fu;
    sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
}

// Byte b of `bytes` as the f16 pair (v, v), exact (v < 1024).
template <int B>
__device__ __forceinline__ std::uint32_t byte_pair(std::uint32_t bytes) {
    constexpr std::uint32_t sel = 0x4040u | B | (B << 8);
    return hsub2_u32(prmt(bytes, 0x64646464u, sel), 0x64006400u);
}
__device__ __forceinline__ std::uint32_t byte_pair_rt(std::uint32_t bytes, std::uint32_t sel) {
    return hsub2_u32(prmt(bytes, 0x64646464u, sel), 0x64006400u);
}

template <int NT, bool OF32>
__device__ __forceinline__ void store_tile(const Params& p, std::uint32_t tile, int g, int t,
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
__global__ void __launch_bounds__(kThreads, 2) q4_k_gemv_kernel(const Params p) {
    extern __shared__ __align__(1024) std::uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    std::uint8_t* xs = smem;
    std::uint8_t* ss = smem + p.x_bytes;
    std::uint8_t* ring = smem + p.x_bytes + p.s_bytes + warp * STAGES * kStageBytes;
    float* red =
        reinterpret_cast<float*>(smem + p.x_bytes + p.s_bytes + kWarps * STAGES * kStageBytes);

    // groups of `split` warps walk tiles first, first + stride, ...; warp
    // wig of a group owns super-blocks [u0, u1) of each
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

    // stage chunk c (16 bytes): row c / 9, column chunk c % 9
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
            src[j] = p.w + r * p.pitch + static_cast<std::uint64_t>(u0) * kBlockBytes + src_off[j];
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
                for (int j = 0; j < kChunksPerLane; ++j) src[j] += kBlockBytes;
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

    // stage the activation rows (elements 1 and 2 of every group of four
    // swapped), the per-32-element sums of each row as f16 (hi, lo) pairs,
    // and an all-zero row of each
    {
        const std::uint32_t vec_per_row = static_cast<std::uint32_t>(p.K / 8);  // % 32 == 0
        const std::uint32_t nvec = p.M * vec_per_row;
        for (std::uint32_t base = static_cast<std::uint32_t>(warp) * 32; base < nvec;
             base += kThreads) {
            const std::uint32_t i = base + lane;
            float s = 0.f;
            std::uint32_t m = 0, v = 0;
            if (i < nvec) {
                m = i / vec_per_row;
                v = i - m * vec_per_row;
                const uint4 val = __ldg(reinterpret_cast<const uint4*>(p.x + m * p.K) + v);
                // elements 1 and 2 of every group of four swapped
                const uint4 pv = make_uint4(prmt(val.x, val.y, 0x5410u), prmt(val.x, val.y, 0x7632u),
                                            prmt(val.z, val.w, 0x5410u), prmt(val.z, val.w, 0x7632u));
                *reinterpret_cast<uint4*>(xs + m * p.x_stride + 16 * v) = pv;
                const std::uint32_t wv[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = q4::half2_bits_to_float2(wv[k]);
                    s += f.x;
                    s += f.y;
                }
            }
            // four consecutive vectors are one 32-element sub-block
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (i < nvec && (lane & 3) == 0) {
                const __half hi = __float2half_rn(s);
                const __half lo = __float2half_rn(s - __half2float(hi));
                *reinterpret_cast<std::uint32_t*>(ss + m * p.s_stride + 4 * (v / 4)) =
                    static_cast<std::uint32_t>(__half_as_ushort(hi)) |
                    (static_cast<std::uint32_t>(__half_as_ushort(lo)) << 16);
            }
        }
        for (std::uint32_t i = threadIdx.x; i < p.x_stride / 16; i += kThreads)
            *reinterpret_cast<uint4*>(xs + p.M * p.x_stride + 16 * i) = make_uint4(0u, 0u, 0u, 0u);
        for (std::uint32_t i = threadIdx.x; i < p.s_stride / 16; i += kThreads)
            *reinterpret_cast<uint4*>(ss + p.M * p.s_stride + 16 * i) = make_uint4(0u, 0u, 0u, 0u);
        __syncthreads();
    }

    // B rows of this lane: token nt*8 + g, or the zero row
    std::uint32_t xsel[NT], ssel[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const std::uint32_t m = nt * 8 + g;
        const std::uint32_t r = m < p.M ? m : p.M;
        xsel[nt] = smem_u32(xs) + r * p.x_stride + 8 * t;
        ssel[nt] = smem_u32(ss) + r * p.s_stride + 4 * t;
    }
    const std::uint32_t msel = 0x4040u | static_cast<std::uint32_t>(t) |
                               (static_cast<std::uint32_t>(t) << 8);
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
            const std::uint32_t u = u0 + st;
            const uint4 hg = lds128(ra);
            const uint4 hh = lds128(ra + kR8);
            std::uint32_t scg[2], sch[2], mg[2], mh[2];
            unpack_scales(hg, scg[0], scg[1], mg[0], mg[1]);
            unpack_scales(hh, sch[0], sch[1], mh[0], mh[1]);

            // mins: A = (m_t, m_t | m_t+4, m_t+4) of rows g, g+8; B = the
            // token's (hi, lo) sums of sub-blocks t and t + 4
            const std::uint32_t ma0 = byte_pair_rt(mg[0], msel);
            const std::uint32_t ma1 = byte_pair_rt(mh[0], msel);
            const std::uint32_t ma2 = byte_pair_rt(mg[1], msel);
            const std::uint32_t ma3 = byte_pair_rt(mh[1], msel);
            float mins[NT][4];
            float dot[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const std::uint32_t b0 = lds32(ssel[nt] + 32 * u);
                const std::uint32_t b1 = lds32(ssel[nt] + 32 * u + 16);
                mins[nt][0] = mins[nt][1] = mins[nt][2] = mins[nt][3] = 0.f;
                mma_16816(mins[nt], ma0, ma1, ma2, ma3, b0, b1, mins[nt]);
                dot[nt][0] = dot[nt][1] = dot[nt][2] = dot[nt][3] = 0.f;
            }

            q4::static_for<0, 4>([&](auto cc) {
                constexpr int c = decltype(cc)::value;
                // sub-blocks 2c (low nibbles) and 2c + 1 (high nibbles)
                const std::uint32_t wg = c < 2 ? scg[0] : scg[1];
                const std::uint32_t wh = c < 2 ? sch[0] : sch[1];
                constexpr int bl = (2 * c) & 3;
                const std::uint32_t slg = byte_pair<bl>(wg), slh = byte_pair<bl>(wh);
                const std::uint32_t shg = byte_pair<bl + 1>(wg), shh = byte_pair<bl + 1>(wh);
                const std::uint32_t clg = hmul2_u32(slg, 0xE400E400u);  // -1024 sc
                const std::uint32_t clh = hmul2_u32(slh, 0xE400E400u);
                const std::uint32_t chg = hmul2_u32(shg, 0xD400D400u);  // -64 sc
                const std::uint32_t chh = hmul2_u32(shh, 0xD400D400u);
                // word t of each 16-byte half of group c, rows g and g + 8
                const std::uint32_t w[2][2] = {
                    {lds32i<16 + 32 * c>(qa), lds32i<kR8 + 16 + 32 * c>(qa)},
                    {lds32i<32 + 32 * c>(qa), lds32i<kR8 + 32 + 32 * c>(qa)}};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    std::uint32_t lo[4], hi[4];  // a0..a3 of the low / high plane
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const std::uint32_t wa = w[h][r];       // bytes 0, 2
                        const std::uint32_t wb = w[h][r] >> 8;  // bytes 1, 3
                        const std::uint32_t sl = r ? slh : slg, cl = r ? clh : clg;
                        const std::uint32_t su = r ? shh : shg, cu = r ? chh : chg;
                        lo[r] = hfma2_u32(and_or(wa, 0x000F000Fu, 0x64006400u), sl, cl);
                        lo[2 + r] = hfma2_u32(and_or(wb, 0x000F000Fu, 0x64006400u), sl, cl);
                        hi[r] = hfma2_u32(and_or(wa, 0x00F000F0u, 0x54005400u), su, cu);
                        hi[2 + r] = hfma2_u32(and_or(wb, 0x00F000F0u, 0x54005400u), su, cu);
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        // elements 64c + 16h + 4t.. (low) and + 32 (high)
                        const std::uint32_t xa = xsel[nt] + (256u * u + 64 * c + 16 * h) * 2;
                        const uint2 xl = lds64(xa);
                        const uint2 xh = lds64(xa + 64);
                        mma_16816(dot[nt], lo[0], lo[1], lo[2], lo[3], xl.x, xl.y, dot[nt]);
                        mma_16816(dot[nt], hi[0], hi[1], hi[2], hi[3], xh.x, xh.y, dot[nt]);
                    }
                }
            });
            const float dg = half_bits_to_float(hg.x & 0xFFFFu);
            const float dmg = half_bits_to_float(hg.x >> 16);
            const float dh = half_bits_to_float(hh.x & 0xFFFFu);
            const float dmh = half_bits_to_float(hh.x >> 16);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                // acc += d * dot - dmin * mins, as two packed f32x2 FMAs per row
                // pair (each lane rounds as fmaf, in the same order)
                q4::fma_pair(acc[nt][0], acc[nt][1], -dmg, -dmg, mins[nt][0], mins[nt][1]);
                q4::fma_pair(acc[nt][0], acc[nt][1], dg, dg, dot[nt][0], dot[nt][1]);
                q4::fma_pair(acc[nt][2], acc[nt][3], -dmh, -dmh, mins[nt][2], mins[nt][3]);
                q4::fma_pair(acc[nt][2], acc[nt][3], dh, dh, dot[nt][2], dot[nt][3]);
            }
            __syncwarp();  // the slot is refilled by the next iteration's issue
            slot = slot + 1 == STAGES ? 0 : slot + 1;
        }
        const std::uint32_t tile = first + tl * stride;
        if (split == 1) {
            store_tile<NT, OF32>(p, tile, g, t, acc);
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
            store_tile<NT, OF32>(p, tile, g, t, sum);
        }
    }
}

// ---- Q6_K decode GEMV ------------------------------------------------------------
// Q6_K super-blocks are 210 bytes, so inside a row they are only 2-byte
// aligned.  With K % 2048 == 0 a row is a whole number of 16-byte chunks and
// super-block u starts rem = (210 u) mod 16 bytes past a chunk boundary, the
// same in every row.  A stage copies the 14 chunks (224 bytes) that cover the
// block; the last block of a row has rem = 14, so its chunks end exactly at
// the row's end and no copy leaves the matrix.  Blocks with rem = 2 mod 4
// (odd u) have their quant words funnel-shifted out of two aligned words.
// Step s (16 elements, one int8 scale) of a block: lane (g, t) takes elements
// 16 s + 4t .. + 3, whose low nibbles are one word of ql and whose 2-bit high
// parts are one word of qh; q - 32 becomes an exact f16 pair with one PRMT
// and one f16x2 subtraction, each step is one MMA (C = 0), scaled by the
// row's f32 d * sc into the accumulator.  The 16 x 16 products d * sc of a
// stage are computed once per warp into a scratch whose 80-byte rows put the
// eight row groups' 16-byte reads in distinct banks.
constexpr int kQ6Bytes = 210;
constexpr int kQ6Row = 240;                           // smem row stride: rows 28 banks apart
constexpr int kQ6RowChunks = 14;
constexpr int kQ6Stage = kTileRows * kQ6Row;          // 3840
constexpr int kQ6Chunks = kTileRows * kQ6RowChunks;   // 224
constexpr int kQ6ChunksPerLane = kQ6Chunks / 32;      // 7
constexpr int kQ6ScaleStride = 20;                    // floats per row: rows 20 banks apart
constexpr int kQ6ScaleBytes = kTileRows * kQ6ScaleStride * 4;  // d * sc of one stage, per warp

__host__ __device__ constexpr int q6_smem_bytes(int x_bytes, int nt, int stages) {
    return x_bytes + kWarps * stages * kQ6Stage + kWarps * kQ6ScaleBytes + red_bytes(nt);
}

__device__ __forceinline__ int lds8s(std::uint32_t addr) {
    int v;
    asm volatile("ld.shared.s8 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts128f(std::uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}
__device__ __forceinline__ float4 lds128f(std::uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}
// The 4 bytes at addr: addr is word-aligned, or (MIS) 2 bytes past a word.
template <bool MIS>
__device__ __forceinline__ std::uint32_t ldw(std::uint32_t addr) {
    if constexpr (MIS)
        return prmt(lds32(addr - 2), lds32(addr + 2), 0x5432u);
    else
        return lds32(addr);
}

template <int NT, bool OF32, int STAGES>
__global__ void __launch_bounds__(kThreads, 2) q6_k_gemv_kernel(const Params p) {
    extern __shared__ __align__(1024) std::uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    std::uint8_t* xs = smem;
    std::uint8_t* ring = smem + p.x_bytes + warp * STAGES * kQ6Stage;
    const std::uint32_t dsc_s =
        smem_u32(smem + p.x_bytes + kWarps * STAGES * kQ6Stage + warp * kQ6ScaleBytes);
    float* red = reinterpret_cast<float*>(smem + p.x_bytes + kWarps * STAGES * kQ6Stage +
                                          kWarps * kQ6ScaleBytes);

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

    // chunk c = lane + 32 j: row c / 14, column chunk c % 14
    std::uint32_t dst_off[kQ6ChunksPerLane];
    std::uint32_t chunk_row[kQ6ChunksPerLane];
#pragma unroll
    for (int j = 0; j < kQ6ChunksPerLane; ++j) {
        const int c = lane + 32 * j;
        chunk_row[j] = static_cast<std::uint32_t>(c / kQ6RowChunks);
        dst_off[j] = chunk_row[j] * kQ6Row + (c % kQ6RowChunks) * 16;
    }
    const std::uint32_t ring_s = smem_u32(ring);
    std::uint32_t iss_n = 0, iss_tl = 0, iss_u = 0, iss_slot = 0;
    const std::uint8_t* src[kQ6ChunksPerLane];  // row start + column chunk
    auto seek_tile = [&](std::uint32_t tl) {
        const std::uint64_t row0 = static_cast<std::uint64_t>(first + tl * stride) * kTileRows;
#pragma unroll
        for (int j = 0; j < kQ6ChunksPerLane; ++j) {
            const std::uint64_t r = min(row0 + chunk_row[j], static_cast<std::uint64_t>(p.N - 1));
            src[j] = p.w + r * p.pitch + ((lane + 32 * j) % kQ6RowChunks) * 16;
        }
    };
    if (total > 0) seek_tile(0);
    auto issue = [&]() {
        if (iss_n < total) {
            const std::uint32_t slot_s = ring_s + iss_slot * kQ6Stage;
            const std::uint32_t boff = ((u0 + iss_u) * kQ6Bytes) & ~15u;
#pragma unroll
            for (int j = 0; j < kQ6ChunksPerLane; ++j)
                cp_async_16(slot_s + dst_off[j], src[j] + boff, policy);
            if (++iss_u == spt) {
                iss_u = 0;
                if (iss_n + 1 < total) seek_tile(++iss_tl);
            }
        }
        ++iss_n;
        iss_slot = iss_slot + 1 == STAGES ? 0 : iss_slot + 1;
        cp_async_commit();
    };
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

    std::uint32_t xsel[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const std::uint32_t m = nt * 8 + g;
        xsel[nt] = smem_u32(xs) + (m < p.M ? m : p.M) * p.x_stride + 8 * t;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    constexpr std::uint32_t kR8 = 8 * kQ6Row;
    std::uint32_t slot = 0;

    // one super-block of the stage in `slot_s`, block base 2 bytes past a
    // word when MIS
    auto block = [&](auto mis, std::uint32_t slot_s, std::uint32_t u, std::uint32_t rem) {
        constexpr bool MIS = decltype(mis)::value;
        // d * sc of the stage: lane L takes row L / 2, scale groups 8 (L % 2) ..
        {
            const std::uint32_t r = static_cast<std::uint32_t>(lane) >> 1;
            const std::uint32_t s0 = 8u * (lane & 1);
            const std::uint32_t rb = slot_s + r * kQ6Row + rem;
            const float d = half_bits_to_float(lds16(rb + 208));
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = d * static_cast<float>(lds8s(rb + 192 + s0 + i));
            sts128f(dsc_s + (r * kQ6ScaleStride + s0) * 4, v[0], v[1], v[2], v[3]);
            sts128f(dsc_s + (r * kQ6ScaleStride + s0 + 4) * 4, v[4], v[5], v[6], v[7]);
        }
        __syncwarp();
        const std::uint32_t qa = slot_s + g * kQ6Row + rem + 4 * t;  // row g, word t
        q4::static_for<0, 2>([&](auto hh) {
            constexpr int h = decltype(hh)::value;
            std::uint32_t L[4][2], H[2][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                L[i][0] = ldw<MIS>(qa + 64 * h + 16 * i);
                L[i][1] = ldw<MIS>(qa + kR8 + 64 * h + 16 * i);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                H[i][0] = ldw<MIS>(qa + 128 + 32 * h + 16 * i);
                H[i][1] = ldw<MIS>(qa + kR8 + 128 + 32 * h + 16 * i);
            }
            q4::static_for<0, 2>([&](auto qq) {
                constexpr int quad = decltype(qq)::value;  // steps 4 quad .. + 3 of this half
                const float4 sg = lds128f(dsc_s + (g * kQ6ScaleStride + 8 * h + 4 * quad) * 4);
                const float4 sh8 =
                    lds128f(dsc_s + ((g + 8) * kQ6ScaleStride + 8 * h + 4 * quad) * 4);
                const float dsg[4] = {sg.x, sg.y, sg.z, sg.w};
                const float dsh[4] = {sh8.x, sh8.y, sh8.z, sh8.w};
                q4::static_for<0, 4>([&](auto ss) {
                    constexpr int s8 = 4 * quad + decltype(ss)::value;  // step within the half
                    constexpr int n = s8 / 4, qi = s8 % 4, j = s8 / 2, hi = s8 % 2;
                    std::uint32_t p01[2], p23[2];
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const std::uint32_t a = n ? (L[qi][r] >> 4) : L[qi][r];
                        const std::uint32_t b = H[hi][r];
                        const std::uint32_t bs = j == 0 ? (b << 4) : j == 1 ? (b << 2)
                                               : j == 2 ? b : (b >> 2);
                        const std::uint32_t q = and_or(a, 0x0F0F0F0Fu, bs & 0x30303030u);
                        p01[r] = hsub2_u32(prmt(q, 0x64646464u, 0x4140u), 0x64206420u);
                        p23[r] = hsub2_u32(prmt(q, 0x64646464u, 0x4342u), 0x64206420u);
                    }
                    constexpr int s = 8 * h + s8;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const uint2 xb = lds64(xsel[nt] + (256u * u + 16 * s) * 2);
                        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
                        mma_16816(tmp, p01[0], p01[1], p23[0], p23[1], xb.x, xb.y, tmp);
                        const int k4 = decltype(ss)::value;
                        // packed f32x2 FMAs (each lane rounds as fmaf)
                        q4::fma_pair(acc[nt][0], acc[nt][1], dsg[k4], dsg[k4], tmp[0], tmp[1]);
                        q4::fma_pair(acc[nt][2], acc[nt][3], dsh[k4], dsh[k4], tmp[2], tmp[3]);
                    }
                });
            });
        });
        __syncwarp();  // the scratch and the slot are rewritten next
    };

    for (std::uint32_t tl = 0; tl < my_tiles; ++tl) {
        for (std::uint32_t st = 0; st < spt; ++st) {
            issue();
            cp_async_wait<STAGES - 1>();
            __syncwarp();
            const std::uint32_t u = u0 + st;
            const std::uint32_t rem = (u * kQ6Bytes) & 15u;
            const std::uint32_t slot_s = ring_s + slot * kQ6Stage;
            if (rem & 2u)
                block(std::true_type{}, slot_s, u, rem);
            else
                block(std::false_type{}, slot_s, u, rem);
            slot = slot + 1 == STAGES ? 0 : slot + 1;
        }
        const std::uint32_t tile = first + tl * stride;
        if (split == 1) {
            store_tile<NT, OF32>(p, tile, g, t, acc);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
            continue;
        }
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
            store_tile<NT, OF32>(p, tile, g, t, sum);
        }
    }
}

// ---- element decode shared by the generic linear and the dequantizer --------
// Sub-block j (32 elements, 0..7) of a super-block, f32, each element one
// separately rounded expression (no contraction), as the published decode.
template <int FMT>
__device__ __forceinline__ void decode_sub(const std::uint8_t* b, int j, float (&v)[32]) {
    if constexpr (FMT == kQ4K) {
        const float d = half_bits_to_float(b[0] | (b[1] << 8));
        const float dmin = half_bits_to_float(b[2] | (b[3] << 8));
        const std::uint8_t* s = b + 4;
        std::uint32_t sc, m;
        if (j < 4) {
            sc = s[j] & 63u;
            m = s[j + 4] & 63u;
        } else {
            sc = (s[j + 4] & 0x0Fu) | ((s[j - 4] >> 6) << 4);
            m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const float ds = __fmul_rn(d, static_cast<float>(sc));
        const float dm = __fmul_rn(dmin, static_cast<float>(m));
        const std::uint8_t* q = b + 16 + 32 * (j / 2);
        const int shift = 4 * (j & 1);
#pragma unroll
        for (int l = 0; l < 32; ++l)
            v[l] = __fsub_rn(__fmul_rn(ds, static_cast<float>((q[l] >> shift) & 0x0F)), dm);
    } else {
        const float d = half_bits_to_float(b[208] | (b[209] << 8));
        const int h = j / 4;        // 128-element half
        const int e0 = 32 * (j % 4);  // first element within the half
        const std::uint8_t* ql = b + 64 * h + (e0 % 64);
        const std::uint8_t* qh = b + 128 + 32 * h;
        const int lshift = 4 * (e0 / 64), hshift = 2 * (j % 4);
        const std::int8_t* sc = reinterpret_cast<const std::int8_t*>(b + 192);
        const float s0 = __fmul_rn(d, static_cast<float>(sc[(128 * h + e0) / 16]));
        const float s1 = __fmul_rn(d, static_cast<float>(sc[(128 * h + e0) / 16 + 1]));
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const int q = static_cast<int>(((ql[l] >> lshift) & 0x0F) |
                                           (((qh[l] >> hshift) & 0x03) << 4)) - 32;
            v[l] = __fmul_rn(l < 16 ? s0 : s1, static_cast<float>(q));
        }
    }
}

// Any K multiple of 256, any alignment: one warp per output row and group of
// up to 8 tokens, lanes striding over 32-element sub-blocks, f32 accumulation.
constexpr int kGenericTokens = 8;

template <int FMT, bool OF32>
__global__ void __launch_bounds__(128) kquant_linear_generic_kernel(const Params p) {
    pdl_launch_dependents();
    pdl_wait();
    const std::uint32_t row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const std::uint32_t m0 = blockIdx.y * kGenericTokens;
    if (row >= p.N) return;
    const std::uint64_t subs = p.K / 32;
    float acc[kGenericTokens];
#pragma unroll
    for (int j = 0; j < kGenericTokens; ++j) acc[j] = 0.f;
    const std::uint8_t* wrow = p.w + row * p.pitch;
    for (std::uint64_t s = lane; s < subs; s += 32) {
        float v[32];
        decode_sub<FMT>(wrow + (s / 8) * block_bytes(FMT), static_cast<int>(s % 8), v);
#pragma unroll
        for (int mm = 0; mm < kGenericTokens; ++mm) {
            const std::uint32_t m = m0 + mm;
            if (m >= p.M) break;
            const __half* xr = p.x + m * p.K + s * 32;
            float a = 0.f;
#pragma unroll
            for (int l = 0; l < 32; ++l) a = fmaf(__half2float(xr[l]), v[l], a);
            acc[mm] += a;
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

// [rows, K] block-encoded -> f32 values, one thread per 32-element sub-block.
template <int FMT>
__global__ void __launch_bounds__(256) kquant_dequantize_kernel(const std::uint8_t* w,
                                                                float* out, std::uint64_t rows,
                                                                std::uint64_t k) {
    pdl_launch_dependents();
    pdl_wait();
    const std::uint64_t subs_per_row = k / 32;
    const std::uint64_t total = rows * subs_per_row;
    const std::uint64_t pitch = k / 256 * block_bytes(FMT);
    for (std::uint64_t i = blockIdx.x * 256ull + threadIdx.x; i < total;
         i += static_cast<std::uint64_t>(gridDim.x) * 256) {
        const std::uint64_t r = i / subs_per_row;
        const std::uint64_t s = i - r * subs_per_row;
        float v[32];
        decode_sub<FMT>(w + r * pitch + (s / 8) * block_bytes(FMT), static_cast<int>(s % 8), v);
        float* o = out + r * k + s * 32;
#pragma unroll
        for (int l = 0; l < 32; ++l) o[l] = v[l];
    }
}

// ---- host ----------------------------------------------------------------------
template <int FMT, int NT, bool OF32, int STAGES>
int launch_gemv(const Params& p, int ctas_per_sm, cudaStream_t stream) {
    auto kernel = FMT == kQ4K ? q4_k_gemv_kernel<NT, OF32, STAGES> : q6_k_gemv_kernel<NT, OF32, STAGES>;
    static std::atomic<std::uint64_t> configured{0};
    const int st = q4::ensure_smem_attribute(kernel, q4::kMaxSmem, configured);
    if (st != kSuccess) return st;
    const std::uint32_t groups = kWarps >> p.split_shift;
    const std::uint32_t cap = static_cast<std::uint32_t>(q4::sm_count() * ctas_per_sm);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(min((p.tiles + groups - 1) / groups, cap));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes =
        FMT == kQ4K ? smem_bytes(static_cast<int>(p.x_bytes), static_cast<int>(p.s_bytes), NT, STAGES)
                    : q6_smem_bytes(static_cast<int>(p.x_bytes), NT, STAGES);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <int FMT, bool OF32>
int launch_gemv_config(const Params& p, int stages, int ctas, bool two, cudaStream_t stream) {
    switch (stages) {
        case 4:
            return two ? launch_gemv<FMT, 2, OF32, 4>(p, ctas, stream)
                       : launch_gemv<FMT, 1, OF32, 4>(p, ctas, stream);
        case 3:
            return two ? launch_gemv<FMT, 2, OF32, 3>(p, ctas, stream)
                       : launch_gemv<FMT, 1, OF32, 3>(p, ctas, stream);
        default:
            return two ? launch_gemv<FMT, 2, OF32, 2>(p, ctas, stream)
                       : launch_gemv<FMT, 1, OF32, 2>(p, ctas, stream);
    }
}

template <int FMT, bool OF32>
int run_linear(const void* x, const void* w, void* y, std::uint64_t M, std::uint64_t N,
               std::uint64_t K, cudaStream_t stream) {
    const std::size_t osz = OF32 ? 4 : 2;
    // prefill-shaped problems: the tcgen05 GEMM with the format's converter
    // (Q6_K windows need rows of whole 16-byte chunks: K % 2048 == 0)
    if (M > static_cast<std::uint64_t>(kMaxTokens) && (FMT == kQ4K || K % 2048 == 0) &&
        gemm::supported(x, w, y, M, N, K, osz))
        return gemm::launch<OF32, FMT == kQ4K ? gemm::kWQ4_K : gemm::kWQ6_K>(x, w, y, M, N, K,
                                                                          stream);
    Params p{};
    p.w = static_cast<const std::uint8_t*>(w);
    p.N = static_cast<std::uint32_t>(N);
    p.K = K;
    p.pitch = (K / 256) * block_bytes(FMT);
    p.units = static_cast<std::uint32_t>(K / 256);
    p.tiles = static_cast<std::uint32_t>((N + kTileRows - 1) / kTileRows);
    // Q6_K rows are whole 16-byte chunks only when K % 2048 == 0
    const bool fast = (FMT == kQ4K || K % 2048 == 0) && K <= (1ull << 20) &&
                      reinterpret_cast<std::uintptr_t>(x) % 16 == 0 &&
                      reinterpret_cast<std::uintptr_t>(w) % 16 == 0;
    // tokens per launch, ring depth and CTAs per SM: two CTAs per SM with
    // the deepest ring that fits, else one
    std::uint32_t tokens = 0;
    int stages = 2, ctas = 1;
    if (fast) {
        p.x_stride = static_cast<std::uint32_t>(K * 2 + 32);
        p.s_stride = static_cast<std::uint32_t>((K / 32 + 4) * 4);
        for (std::uint32_t m = static_cast<std::uint32_t>(M < kMaxTokens ? M : kMaxTokens);
             m >= 1 && tokens == 0; m /= 2) {
            const std::uint32_t xb = ((m + 1) * p.x_stride + 127u) & ~127u;
            const std::uint32_t sb = ((m + 1) * p.s_stride + 127u) & ~127u;
            const int nt = m > 8 ? 2 : 1;
            constexpr int kOptions[5][2] = {{2, 4}, {2, 3}, {2, 2}, {1, 4}, {1, 2}};
            for (const auto& opt : kOptions) {
                const int bytes = FMT == kQ4K
                                      ? smem_bytes(static_cast<int>(xb), static_cast<int>(sb), nt, opt[1])
                                      : q6_smem_bytes(static_cast<int>(xb), nt, opt[1]);
                if (bytes <= q4::kMaxSmem &&
                    opt[0] * (bytes + q4::kSmemReservedPerCta) <= q4::kSmemPerSm) {
                    tokens = m;
                    ctas = opt[0];
                    stages = opt[1];
                    p.x_bytes = xb;
                    p.s_bytes = FMT == kQ4K ? sb : 0u;
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
            st = launch_gemv_config<FMT, OF32>(p, stages, ctas, mc > 8, stream);
        } else {
            const dim3 grid(static_cast<unsigned>((N + 3) / 4),
                            static_cast<unsigned>((mc + kGenericTokens - 1) / kGenericTokens));
            st = launch_pdl(kquant_linear_generic_kernel<FMT, OF32>, grid, dim3(128), stream, p);
        }
        if (st != 0) return st;
    }
    return kSuccess;
}

// Argument rules of the Q4_0 linear (null pointers and the null stream are
// invalid values, empty outputs succeed without a launch, rows*N must fit
// 32 bits), plus K a multiple of the 256-element super-block (the
// reference's RowMisaligned, quantized.rs:159-165).
inline int check_args(const void* input, const void* weights, void* output, std::uint64_t rows,
                      std::uint64_t n, std::uint64_t k, void* stream) {
    const int c = q4::check_linear_args(input, weights, output, rows, n, k, stream);
    if (c != 0 && c != q4::kEmpty) return c;
    if (k % 256 != 0) return kInvalidValue;
    return c;
}

template <int FMT, bool OF32>
int linear_entry(const void* input, const void* weights, void* output, std::uint64_t rows,
                 std::uint64_t n, std::uint64_t k, void* stream) {
    const int c = check_args(input, weights, output, rows, n, k, stream);
    if (c == q4::kEmpty) return kSuccess;
    if (c != 0) return c;
    if (k == 0) return static_cast<int>(cudaMemsetAsync(output, 0, rows * n * (OF32 ? 4 : 2),
                                                        static_cast<cudaStream_t>(stream)));
    return run_linear<FMT, OF32>(input, weights, output, rows, n, k,
                                 static_cast<cudaStream_t>(stream));
}

}  // namespace kq
}  // namespace mote

// Q4_K weights (ggml 144-byte super-blocks), f16 activations [rows, K], f16
// output [rows, N], f32 accumulation.  No reference counterpart: mote-types
// defines the Q4_K geometry (crates/mote-types/src/lib.rs:41-74) and
// mote-reference rejects it (quantized.rs:152-157).  K % 256 != 0 is an
// invalid value; other rules as mote_cuda_quantized_linear_q4_0_f16.
extern "C" int mote_cuda_quantized_linear_q4_k_f16(const void* input, const void* weights,
                                                   void* output, std::uint64_t rows,
                                                   std::uint64_t output_features,
                                                   std::uint64_t input_features, void* stream) {
    return mote::kq::linear_entry<mote::kq::kQ4K, false>(input, weights, output, rows,
                                                          output_features, input_features, stream);
}

// The same with an f32 output (the accumulator unrounded).
extern "C" int mote_cuda_quantized_linear_q4_k_f16_f32out(const void* input, const void* weights,
                                                          void* output, std::uint64_t rows,
                                                          std::uint64_t output_features,
                                                          std::uint64_t input_features,
                                                          void* stream) {
    return mote::kq::linear_entry<mote::kq::kQ4K, true>(input, weights, output, rows,
                                                         output_features, input_features, stream);
}

// Q6_K weights (210-byte super-blocks), f16 activations, f16 output.
extern "C" int mote_cuda_quantized_linear_q6_k_f16(const void* input, const void* weights,
                                                   void* output, std::uint64_t rows,
                                                   std::uint64_t output_features,
                                                   std::uint64_t input_features, void* stream) {
    return mote::kq::linear_entry<mote::kq::kQ6K, false>(input, weights, output, rows,
                                                          output_features, input_features, stream);
}

// Decodes a [rows, k] Q4_K (format 2) or Q6_K (format 3) matrix into f32
// values, bit-identical to the published decode.  k % 256 != 0, another
// format, or a null pointer / stream is an invalid value; empty succeeds.
extern "C" int mote_cuda_kquant_dequantize_f32(int format, const void* weights, void* output,
                                               std::uint64_t rows, std::uint64_t k,
                                               void* stream) {
    using namespace mote;
    if (weights == nullptr || output == nullptr || stream == nullptr) return kInvalidValue;
    if ((format != kq::kQ4K && format != kq::kQ6K) || k % 256 != 0) return kInvalidValue;
    if (rows == 0 || k == 0) return kSuccess;
    const std::uint64_t subs = rows * (k / 32);
    const unsigned grid = static_cast<unsigned>(subs / 256 + 1 < 65535ull * 16 ? subs / 256 + 1
                                                                               : 65535ull * 16);
    auto s = static_cast<cudaStream_t>(stream);
    auto w = static_cast<const std::uint8_t*>(weights);
    auto o = static_cast<float*>(output);
    if (format == kq::kQ4K)
        return launch_pdl(kq::kquant_dequantize_kernel<kq::kQ4K>, dim3(grid), dim3(256), s, w, o,
                          rows, k);
    return launch_pdl(kq::kquant_dequantize_kernel<kq::kQ6K>, dim3(grid), dim3(256), s, w, o, rows,
                      k);
}
