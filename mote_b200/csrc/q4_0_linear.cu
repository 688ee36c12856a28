// Q4_0 weight-only linear for decode and small batches.
//
//   y[m, n] = sum_k x[m, k] * w[n, k],   w stored as ggml Q4_0 blocks:
//   18 bytes per 32 elements = f16 scale d (little endian) + 16 bytes, byte j
//   holding element j in its low nibble and element j+16 in its high nibble;
//   value = (q - 8) * d.  (crates/mote-types/src/lib.rs:48-74,
//   crates/mote-reference/src/quantized.rs:177-201.)
//
// Design (B200, HBM-bound):
// * Persistent kernel: 8-warp CTAs (two per SM when shared memory allows)
//   walk over tiles of 16 weight rows.  Every warp owns a fixed K-slice of
//   every tile and streams its slice of the 16 rows through a private
//   shared-memory ring: each lane issues 16-byte cp.async copies (L2
//   evict-first), one commit group per 144-byte-per-row stage.  The ring
//   runs continuously across tiles, so the copy pipeline never drains;
//   weights are read from HBM exactly once.
// * The activations (up to 16 rows, f16) are staged into shared memory once
//   per CTA, with padded rows that make the fragment loads bank-conflict
//   free, plus one all-zero row.
// * Dequantization happens in registers: each lane decodes one 4-byte quant
//   word per row per block into exact f16 integers (q - 8) with LOP3 + HSUB2
//   (the 1024+q / 64+q exponent tricks), and the warp issues
//   mma.sync.m16n8k16 (f16 x f16 -> f32) with the weights as the A operand.
//   The f16 block scale multiplies the f32 block partial (FFMA): products
//   and scaling are exact, only the f32 accumulation rounds.
// * Column packing: with 8 or fewer activation rows the eight B columns
//   carry 8/MC consecutive blocks x MC rows (MC = 1, 2, 4 or 8), the other
//   lanes reading the zero row, so one MMA chain covers 8/MC blocks with
//   every column holding a single block's exact partial.  The scale FFMAs,
//   scale loads and accumulator resets then run once per chain instead of
//   once per block; a lane shuffle folds the columns back per row at the
//   end of a tile.
// * The k-slot permutation inside each 16-wide MMA makes a lane's B
//   fragment 4 consecutive activations (one 8-byte load) and its A fragment
//   one 4-byte quant word; A and B share the permutation, so the dot product
//   is unchanged.
// * f32 activations are split into f16 hi + lo rows (adjacent MMA columns),
//   keeping their full precision (error ~2^-22 relative).
// * The eight K-slice partials of a tile meet in a double-buffered shared
//   reduction area behind one named barrier; the warps take turns writing
//   finished tiles, so the others keep streaming.
// * Programmatic dependent launch: the ring prologue (weights only) runs
//   before griddepcontrol.wait, overlapping the previous kernel's tail.
//
// Fast-path requirements: K a multiple of 256 (whole 144-byte, 16-byte
// aligned groups of 8 blocks per row), 16-byte aligned weights and
// activations.  Other shapes use the generic warp-per-row kernel.

#include "mote_common.cuh"

#include <cuda.h>

#include <atomic>
#include <mutex>
#include <type_traits>

namespace mote {
namespace q4 {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileRows = 16;
constexpr int kUnitBlocks = 8;            // 8 blocks = 256 elements = 144 bytes
constexpr int kUnitBytes = kUnitBlocks * 18;
constexpr int kStageUnits = 1;            // 8 blocks per stage
// Dense 144-byte rows: 36 words = 4 (mod 32) banks apart, so the 8 rows a
// warp reads at once (word t of row g: bank 4g + t) hit 32 distinct banks.
constexpr int kRowStride = kStageUnits * kUnitBytes;        // 144
constexpr int kStageBytes = kTileRows * kRowStride;         // 2304
constexpr int kMaxSmem = 232448;                            // 227 KB per-CTA opt-in limit
constexpr int kSmemPerSm = 233472;                          // 228 KB per SM
constexpr int kSmemReservedPerCta = 1024;                   // system use per resident CTA
constexpr int kMaxXRows = 16;                               // two n8 tiles

// kEpiPeers: the plain f16 result of this rank's row shard is stored into
// every rank's full output buffer (over NVLink for the peers) and the grid
// ends with a flag handshake, so every rank holds all shards when the
// kernel completes.
// kEpiNorm*: the staged activation rows are first RMS-normalised (with
// gamma, in mote-reference's operation order) -- the norm that precedes a
// projection in a decoder layer, fused into its prologue.  kEpiNormRope
// also rotates the q and k rows of a QKV projection (RoPE, HalfSplit) in
// the epilogue, before the single f16 rounding.
enum Epilogue : int {
    kEpiPlain = 0,
    kEpiSwiGLU = 1,
    kEpiResidual = 2,
    kEpiPeers = 3,
    kEpiNormPlain = 4,
    kEpiNormSwiGLU = 5,
    kEpiNormRope = 6
};

__host__ __device__ constexpr bool epi_norm(int e) { return e >= kEpiNormPlain; }
__host__ __device__ constexpr bool epi_swiglu(int e) {
    return e == kEpiSwiGLU || e == kEpiNormSwiGLU;
}
__host__ __device__ constexpr bool epi_rope(int e) { return e == kEpiNormRope; }

struct Params {
    const void* x;            // [M, K] f16 or f32, row stride K
    const std::uint8_t* w;    // [N, K/32*18]
    const std::uint8_t* w2;   // second matrix (up projection) for kEpiSwiGLU
    const __half* res;        // residual added by kEpiResidual, same layout as y
    void* y;                  // [M, ldy] f16 or f32
    std::uint32_t M;          // tokens in this launch
    std::uint32_t N;          // rows of w (and of w2)
    std::uint64_t K;
    std::uint64_t pitch;      // bytes per weight row
    std::uint32_t units;      // K / 256
    std::uint32_t tiles;      // row tiles
    std::uint64_t ldy;        // output row stride (elements)
    std::uint32_t x_rows;     // activation rows in shared memory (M, or 2M for f32)
    std::uint32_t x_stride;   // bytes per shared activation row (2K + 32)
    std::uint32_t x_bytes;    // (x_zero_row + 1) * x_stride rounded up to 128
    std::uint32_t x_zero_row; // index of the all-zero row after the staged rows
    std::uint32_t split_shift; // log2 of the warps sharing a tile's K (0..3)
    // kEpiPeers: output buffers [M, ldy] of every rank (device array), this
    // rank's first column, and the flag arrays of the handshake.
    __half* const* peer_y;
    unsigned* const* peer_flags;
    unsigned* own_flags;
    std::uint64_t col0;
    std::uint32_t rank;
    std::uint32_t nranks;
    // kEpiNorm*: RMSNorm of the staged rows
    const __half* gamma;
    float eps;
    // kEpiNormRope: the first rope_rows output rows are rope_rows / head_dim
    // heads rotated with cos/sin [M, head_dim/2] (f32); tiles below
    // rope_tiles pair rows d and d + head_dim/2 of a head
    const float* rope_cos;
    const float* rope_sin;
    std::uint32_t rope_rows;
    std::uint32_t rope_tiles;
    std::uint32_t head_dim;
    // K split across CTAs: CTA b works on part b % parts of K (its own
    // units and activation columns); the parts of a tile meet in the
    // workspace -- partial sums part_buf[part][tile][NT*128] and arrival
    // counters part_cnt[tile] (zero between calls: the last part to arrive
    // adds the partials in part order, stores and resets its counter)
    std::uint32_t parts;
    float* part_buf;
    unsigned* part_cnt;
};

__host__ __device__ constexpr int red_bytes(int nt) { return 2 * kWarps * nt * 4 * 32 * 4; }

// kEpiPeers also stages each stored tile (16 rows x up to 16 tokens of
// f16) per warp, to send it to the peers in 16-byte vectors.
constexpr int kPeerStageBytes = 16 * 16 * 2;

__host__ __device__ constexpr int smem_bytes(int x_bytes, int nt, int stages, bool peers = false) {
    return x_bytes + kWarps * stages * kStageBytes + red_bytes(nt) +
           (peers ? kWarps * kPeerStageBytes : 0);
}

// Quant word u = bytes B0..B3 = qs[4t .. 4t+3] of a block.  Its low
// nibbles are elements 4t..4t+3, its high nibbles 16+4t..16+4t+3.  The two
// f16 halves of a register take the nibbles of bytes (B0, B2) or (B1, B3):
//   lo02 = (q[4t],    q[4t+2])       lo13 = (q[4t+1],    q[4t+3])
//   hi02 = (q[16+4t], q[16+4t+2])    hi13 = (q[16+4t+1], q[16+4t+3])
// and the activations are staged in the matching order (elements 1 and 2
// of every group of 4 swapped), so no byte shuffles are needed here.
__device__ __forceinline__ void decode_word(std::uint32_t u, std::uint32_t& lo02,
                                            std::uint32_t& lo13, std::uint32_t& hi02,
                                            std::uint32_t& hi13) {
    const std::uint32_t v = u >> 8;
    // low nibbles: f16(1024 + q) - 1032 = q - 8 (exact)
    lo02 = hsub2_u32(and_or(u, 0x000F000Fu, 0x64006400u), 0x64086408u);
    lo13 = hsub2_u32(and_or(v, 0x000F000Fu, 0x64006400u), 0x64086408u);
    // high nibbles sit at mantissa bits 4..7: f16(64 + q) - 72 = q - 8 (exact)
    hi02 = hsub2_u32(and_or(u, 0x00F000F0u, 0x54005400u), 0x54805480u);
    hi13 = hsub2_u32(and_or(v, 0x00F000F0u, 0x54005400u), 0x54805480u);
}

// (a0, a1) += (s0 * x0, s1 * x1) with one packed f32x2 FMA.
__device__ __forceinline__ void fma_pair(float& a0, float& a1, float s0, float s1, float x0,
                                         float x1) {
    asm("{\n\t.reg .b64 a, s, x;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 s, {%2, %3};\n\t"
        "mov.b64 x, {%4, %5};\n\tfma.rn.f32x2 a, s, x, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(s0), "f"(s1), "f"(x0), "f"(x1));
}

__device__ __forceinline__ std::uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const std::uint32_t*>(&h);
}

__device__ __forceinline__ float2 half2_bits_to_float2(std::uint32_t v) {
    __half2 h;
    memcpy(&h, &v, sizeof(h));
    return __half22float2(h);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    return g / (1.0f + expf(-g)) * u;
}

// Output row held by A row i (0..15) of a kEpiNormRope tile.  A rope tile
// (tile < rope_tiles) covers 8 consecutive rows d of the first half of a
// head (A rows 0-7) and their partners d + head_dim/2 (A rows 8-15), so
// lane (g, t) holds both elements of a rotation pair; the later tiles are
// plain runs of 16 rows (the v heads).
__device__ __forceinline__ std::uint32_t rope_tile_row(const Params& p, std::uint32_t tile,
                                                       int i) {
    std::uint32_t r;
    if (tile < p.rope_tiles) {
        const std::uint32_t per_head = p.head_dim / 16;
        const std::uint32_t h = tile / per_head;
        const std::uint32_t j0 = (tile - h * per_head) * 8;
        r = h * p.head_dim + j0 + (i & 7) + (i < 8 ? 0u : p.head_dim / 2);
    } else {
        r = p.rope_rows + (tile - p.rope_tiles) * 16u + i;
    }
    return min(r, p.N - 1);
}

// Source row i (0..15) of a tile.  Plain tiles are 16 consecutive rows;
// SwiGLU tiles pair gate rows f..f+7 (A rows 0-7) with up rows f..f+7
// (A rows 8-15) so lane (g, t) ends up holding gate and up of the same
// feature.  Rows past N are clamped (loaded, never stored).
template <int EPI>
__device__ __forceinline__ const std::uint8_t* tile_row(const Params& p, std::uint32_t tile,
                                                        int i) {
    if constexpr (epi_swiglu(EPI)) {
        const std::uint32_t f = min(tile * 8u + (i & 7), p.N - 1);
        return (i < 8 ? p.w : p.w2) + f * p.pitch;
    } else if constexpr (epi_rope(EPI)) {
        return p.w + rope_tile_row(p, tile, i) * p.pitch;
    } else {
        const std::uint32_t r = min(tile * 16u + i, p.N - 1);
        return p.w + r * p.pitch;
    }
}

template <int NT, bool XF32, bool OF32, int EPI>
__device__ __forceinline__ void store_tile(const Params& p, std::uint32_t tile, int g, int t,
                                           const float (&acc)[NT][4], __half* stage = nullptr) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        if constexpr (epi_rope(EPI)) {
            if (tile < p.rope_tiles) {
                // rows (d, d + head_dim/2) of one head: rotate, round once
                const std::uint32_t per_head = p.head_dim / 16;
                const std::uint32_t h = tile / per_head;
                const std::uint32_t j = (tile - h * per_head) * 8 + g;
                const std::uint32_t r1 = h * p.head_dim + j;
                const std::uint32_t r2 = r1 + p.head_dim / 2;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const std::uint32_t m = nt * 8 + 2 * t + c;
                    if (m >= p.M) continue;
                    const float cs = p.rope_cos[m * (p.head_dim / 2) + j];
                    const float sn = p.rope_sin[m * (p.head_dim / 2) + j];
                    float o1, o2;
                    rotate(acc[nt][c], acc[nt][2 + c], cs, sn, o1, o2);
                    static_cast<__half*>(p.y)[m * p.ldy + r1] = __float2half_rn(o1);
                    static_cast<__half*>(p.y)[m * p.ldy + r2] = __float2half_rn(o2);
                }
            } else {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const std::uint32_t r = p.rope_rows + (tile - p.rope_tiles) * 16u + g + 8 * half;
                    if (r >= p.N) continue;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const std::uint32_t m = nt * 8 + 2 * t + c;
                        if (m >= p.M) continue;
                        static_cast<__half*>(p.y)[m * p.ldy + r] =
                            __float2half_rn(acc[nt][2 * half + c]);
                    }
                }
            }
            continue;
        }
        if constexpr (epi_swiglu(EPI)) {
            const std::uint32_t f = tile * 8u + g;
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
                const std::uint32_t r = tile * 16u + g + 8 * half;
                if (r >= p.N) continue;
                if constexpr (!XF32) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const std::uint32_t m = nt * 8 + 2 * t + c;
                        if (m >= p.M) continue;
                        float v = acc[nt][2 * half + c];
                        if constexpr (EPI == kEpiResidual) v += __half2float(p.res[m * p.ldy + r]);
                        if constexpr (EPI == kEpiPeers) {
                            stage[m * 16 + g + 8 * half] = __float2half_rn(v);
                            continue;
                        }
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
    if constexpr (EPI == kEpiPeers) {
        // Staged tile [token][16 rows] -> two 16-byte vectors per token, to
        // every rank's buffer (columns col0 + 16 * tile ..); a ragged last
        // tile falls back to 2-byte stores of its real rows.
        __syncwarp();
        const int lane = 4 * g + t;
        const std::uint32_t m = static_cast<std::uint32_t>(lane) >> 1;
        const std::uint32_t r0 = tile * 16u + 8u * (lane & 1);
        if (m < p.M && r0 < p.N) {
            const std::uint64_t at = m * p.ldy + p.col0 + r0;
            const __half* src = stage + m * 16 + 8 * (lane & 1);
            if (r0 + 8 <= p.N) {
                const uint4 v = *reinterpret_cast<const uint4*>(src);
                for (std::uint32_t q = 0; q < p.nranks; ++q)
                    *reinterpret_cast<uint4*>(p.peer_y[q] + at) = v;
            } else {
                for (std::uint32_t q = 0; q < p.nranks; ++q)
                    for (std::uint32_t i = 0; r0 + i < p.N; ++i) p.peer_y[q][at + i] = src[i];
            }
        }
        __syncwarp();
    }
}

// Compile-time loop: f(std::integral_constant<int, I>) for I in [B, E).
template <int B, int E, typename F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (B < E) {
        f(std::integral_constant<int, B>{});
        static_for<B + 1, E>(f);
    }
}

// End of a kEpiPeers grid: the CTA's stores are published with one
// cumulative system-scope fence after a CTA barrier; the last CTA to arrive
// advances this rank's epoch (kept in its flag array, so graph replays
// work), publishes it to every rank and waits -- bounded -- until every rank
// has published it.  Flag array: [q] epoch of rank q, [n] arrival counter,
// [n + 1] own epoch.
__device__ __forceinline__ void peer_handshake(const Params& p) {
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const unsigned arrived = atomicAdd(&p.own_flags[p.nranks], 1u);
    if (arrived != gridDim.x - 1) return;
    p.own_flags[p.nranks] = 0u;
    const unsigned epoch = p.own_flags[p.nranks + 1] + 1u;
    p.own_flags[p.nranks + 1] = epoch;
    // One system fence, then strong relaxed flag stores (a release pattern):
    // the stores to all ranks are in flight together instead of each
    // st.release fencing behind the previous one.
    __threadfence_system();
    for (std::uint32_t q = 0; q < p.nranks; ++q)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p.peer_flags[q] + p.rank),
                     "r"(epoch)
                     : "memory");
    const long long start = clock64();
    for (std::uint32_t q = 0; q < p.nranks; ++q) {
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.own_flags + q)
                         : "memory");
            if (static_cast<int>(v - epoch) >= 0) break;
            if (clock64() - start > kWaitCycles) {
                atomicOr(&g_device_status, kDevWaitTimeout);
                return;
            }
        }
    }
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int NT, int MC, bool XF32, bool OF32, int EPI, int STAGES>
__global__ void __launch_bounds__(kThreads, 2) q4_0_gemv_kernel(const Params p) {
    extern __shared__ __align__(1024) std::uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;

    std::uint8_t* xs = smem;
    std::uint8_t* ring = smem + p.x_bytes + warp * STAGES * kStageBytes;
    float* red = reinterpret_cast<float*>(smem + p.x_bytes + kWarps * STAGES * kStageBytes);
    __half* stage = reinterpret_cast<__half*>(smem + p.x_bytes + kWarps * STAGES * kStageBytes +
                                              red_bytes(NT) + warp * kPeerStageBytes);

    // Split-K: the CTA's warps form kWarps / split groups of `split` warps;
    // a group walks its own tiles (first, first + stride, ...; groups are
    // interleaved across CTAs so small problems spread over every SM) and
    // warp wig of the group owns units [u0, u1) of every one of them.
    // Parts: CTA b takes part b % parts of K (units [pu0, pu1)); the grid
    // is a multiple of parts.
    const std::uint32_t parts = p.parts;
    const std::uint32_t part = blockIdx.x % parts;
    const std::uint32_t cta_in_part = blockIdx.x / parts;
    const std::uint32_t ctas_per_part = gridDim.x / parts;
    const std::uint32_t pu0 = (p.units * part) / parts;
    const std::uint32_t pun = (p.units * (part + 1)) / parts - pu0;
    const std::uint32_t sh = p.split_shift;
    const std::uint32_t split = 1u << sh;
    const std::uint32_t grp = static_cast<std::uint32_t>(warp) >> sh;
    const std::uint32_t wig = static_cast<std::uint32_t>(warp) & (split - 1);
    const std::uint32_t first = cta_in_part + grp * ctas_per_part;
    const std::uint32_t stride = ctas_per_part * (kWarps >> sh);
    const std::uint32_t my_tiles = p.tiles > first ? (p.tiles - first + stride - 1) / stride : 0;
    const std::uint32_t u0 = pu0 + ((pun * wig) >> sh);
    const std::uint32_t u1 = pu0 + ((pun * (wig + 1)) >> sh);
    const std::uint32_t spt = u1 - u0;  // stages (units) per tile
    const std::uint32_t total = my_tiles * spt;
    const std::uint64_t policy = l2_evict_first_policy();

    // A stage is 16 rows x 144 bytes = 144 chunks of 16 bytes; lane l copies
    // chunks l, l+32, ... (row c/9, chunk c%9) with cp.async, one commit
    // group per stage.  Rows of the current tile are cached per lane.
    constexpr int kChunks = kTileRows * (kUnitBytes / 16);              // 144
    constexpr int kChunksPerLane = (kChunks + 31) / 32;                 // 5
    std::uint32_t dst_off[kChunksPerLane];
    std::uint32_t src_off[kChunksPerLane];
    int chunk_row[kChunksPerLane];
#pragma unroll
    for (int j = 0; j < kChunksPerLane; ++j) {
        const int c = min(lane + 32 * j, kChunks - 1);
        chunk_row[j] = c / 9;
        dst_off[j] = chunk_row[j] * kRowStride + (c % 9) * 16;
        src_off[j] = (c % 9) * 16;
    }
    const std::uint32_t ring_s = smem_u32(ring);
    // Issue cursor: the next stage to fetch is unit u0 + iss_u of this CTA's
    // tile number iss_tl; src[j] already points at its chunk j.
    std::uint32_t iss_n = 0, iss_tl = 0, iss_u = 0, iss_slot = 0;
    const std::uint8_t* src[kChunksPerLane];
    auto seek_tile = [&](std::uint32_t tl) {
        const std::uint32_t tile = first + tl * stride;
#pragma unroll
        for (int j = 0; j < kChunksPerLane; ++j)
            src[j] = tile_row<EPI>(p, tile, chunk_row[j]) + static_cast<std::uint64_t>(u0) * kUnitBytes +
                     src_off[j];
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
    // Programmatic dependent launch: this grid may start while earlier
    // kernels of this library are still running on the stream (each lets
    // its successor start at once).  The weights are not written by them --
    // the documented precondition -- so the ring starts streaming them
    // immediately; activations, outputs and everything else are touched only
    // after griddepcontrol.wait, which returns once the previous grid has
    // completed.
    for (int s = 0; s + 1 < STAGES; ++s) issue();
    pdl_launch_dependents();
    pdl_wait();

    // Stage the activations: row r of the shared copy holds activation row r
    // (f16) -- or, for f32 input, rows 2m / 2m+1 hold f16(x[m]) and
    // f16(x[m] - f16(x[m])) -- with elements 1 and 2 of every group of 4
    // swapped to match decode_word's pairing.
    {
        // only this part's columns: elements [256 * pu0, 256 * (pu0 + pun))
        const std::uint64_t kx0 = static_cast<std::uint64_t>(pu0) * 256;
        const std::uint32_t groups = pun * 64;
        const std::uint32_t total_groups = p.M * groups;

        if (!XF32 && p.M >= 3) {
            // Three or more rows: 16-byte chunks, row by row (no division),
            // every thread's chunks of up to four rows loaded before use.
            const std::uint32_t cpr = pun * 32;  // 16-byte chunks per row
            for (std::uint32_t m0 = 0; m0 < p.M; m0 += 4) {
                const std::uint32_t rows = min(4u, p.M - m0);
                for (std::uint32_t c = threadIdx.x; c < cpr; c += kThreads) {
                    uint4 v[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (j < rows)
                            v[j] = __ldg(reinterpret_cast<const uint4*>(
                                static_cast<const __half*>(p.x) + (m0 + j) * p.K + kx0 + 8 * c));
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (j < rows) {
                            uint4 o;
                            o.x = prmt(v[j].x, v[j].y, 0x5410u);
                            o.y = prmt(v[j].x, v[j].y, 0x7632u);
                            o.z = prmt(v[j].z, v[j].w, 0x5410u);
                            o.w = prmt(v[j].z, v[j].w, 0x7632u);
                            *reinterpret_cast<uint4*>(xs + (m0 + j) * p.x_stride + 16 * c) = o;
                        }
                }
            }
        } else
        for (std::uint32_t i = threadIdx.x; i < total_groups; i += kThreads) {
            const std::uint32_t m = i / groups;
            const std::uint32_t gi = i - m * groups;
            if constexpr (!XF32) {
                const uint2 v = __ldg(reinterpret_cast<const uint2*>(
                    static_cast<const __half*>(p.x) + m * p.K + kx0 + 4 * gi));
                uint2 o;
                o.x = prmt(v.x, v.y, 0x5410u);  // (x0, x2)
                o.y = prmt(v.x, v.y, 0x7632u);  // (x1, x3)
                *reinterpret_cast<uint2*>(xs + m * p.x_stride + 8 * gi) = o;
            } else {
                const float4 v = __ldg(reinterpret_cast<const float4*>(
                    static_cast<const float*>(p.x) + m * p.K + kx0 + 4 * gi));
                const float h0 = __half2float(__float2half_rn(v.x));
                const float h1 = __half2float(__float2half_rn(v.y));
                const float h2 = __half2float(__float2half_rn(v.z));
                const float h3 = __half2float(__float2half_rn(v.w));
                const uint2 hi = make_uint2(pack_half2(h0, h2), pack_half2(h1, h3));
                const uint2 lo = make_uint2(pack_half2(v.x - h0, v.z - h2),
                                            pack_half2(v.y - h1, v.w - h3));
                *reinterpret_cast<uint2*>(xs + (2 * m) * p.x_stride + 8 * gi) = hi;
                *reinterpret_cast<uint2*>(xs + (2 * m + 1) * p.x_stride + 8 * gi) = lo;
            }
        }
        // the zero row read by lanes whose B column has no token
        for (std::uint32_t i = threadIdx.x; i < p.x_stride / 16; i += kThreads)
            *reinterpret_cast<uint4*>(xs + p.x_zero_row * p.x_stride + 16 * i) =
                make_uint4(0u, 0u, 0u, 0u);
        __syncthreads();
    }
    if constexpr (epi_norm(EPI)) {
        static_assert(!XF32, "the fused norm takes f16 activations");
        // RMSNorm of the staged rows, in place: every CTA normalises the rows
        // it uses.  Per-row sums of squares (f32, correctly rounded steps),
        // a block reduction, inv = 1/sqrt(mean + eps), then x * inv * gamma
        // rounded once to f16 -- mote-reference's rms_norm_f32 arithmetic
        // (crates/mote-reference/src/lib.rs:289-299), in the staged order
        // (gamma permuted like the activations).
        // scratch in the (not yet used) reduction area: partial sums per
        // warp and row, then the per-row 1/rms
        float (*norm_part)[kMaxXRows] = reinterpret_cast<float (*)[kMaxXRows]>(red);
        float* norm_inv = red + kWarps * kMaxXRows;
        static_assert((kWarps + 1) * kMaxXRows * 4 <= red_bytes(1), "norm scratch");
        const std::uint32_t chunks = static_cast<std::uint32_t>(p.K / 8);
        float ss[kMaxXRows];
#pragma unroll
        for (int m = 0; m < kMaxXRows; ++m) ss[m] = 0.f;
        for (std::uint32_t i = threadIdx.x; i < chunks; i += kThreads) {
#pragma unroll
            for (int m = 0; m < kMaxXRows; ++m) {
                if (static_cast<std::uint32_t>(m) < p.M) {
                    const uint4 v = *reinterpret_cast<const uint4*>(xs + m * p.x_stride + 16 * i);
                    const std::uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 f = half2_bits_to_float2(words[q]);
                        ss[m] = __fadd_rn(ss[m], __fmul_rn(f.x, f.x));
                        ss[m] = __fadd_rn(ss[m], __fmul_rn(f.y, f.y));
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < kMaxXRows; ++m) {
            float v = ss[m];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) norm_part[warp][m] = v;
        }
        __syncthreads();
        if (threadIdx.x < p.M) {
            float total = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) total += norm_part[w][threadIdx.x];
            norm_inv[threadIdx.x] = inv_rms(total, p.K, p.eps);
        }
        __syncthreads();
        for (std::uint32_t i = threadIdx.x; i < chunks; i += kThreads) {
            const uint4 gr = __ldg(reinterpret_cast<const uint4*>(p.gamma) + i);
            const std::uint32_t gw[4] = {prmt(gr.x, gr.y, 0x5410u), prmt(gr.x, gr.y, 0x7632u),
                                         prmt(gr.z, gr.w, 0x5410u), prmt(gr.z, gr.w, 0x7632u)};
            for (std::uint32_t m = 0; m < p.M; ++m) {
                uint4* at = reinterpret_cast<uint4*>(xs + m * p.x_stride + 16 * i);
                const uint4 v = *at;
                const std::uint32_t words[4] = {v.x, v.y, v.z, v.w};
                std::uint32_t out[4];
                const float inv = norm_inv[m];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = half2_bits_to_float2(words[q]);
                    const float2 w = half2_bits_to_float2(gw[q]);
                    out[q] = pack_half2(norm_out(f.x, inv, w.x), norm_out(f.y, inv, w.y));
                }
                *at = make_uint4(out[0], out[1], out[2], out[3]);
            }
        }
        __syncthreads();
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    // Column packing.  B column n = g of this lane is activation row
    // (nt*8 + g) when MC = 8; with MC < 8 staged rows, the 8 columns are
    // BC = 8/MC consecutive blocks x MC rows (n = j*MC + m): for block j of a
    // chain only the lanes with g/MC == j see real activations, the others
    // read the zero row, so one MMA chain accumulates BC blocks into
    // disjoint columns and each column still holds one block's exact partial.
    // xsel[nt][j] is this lane's shared address for chain position j.
    constexpr int BC = 8 / MC;
    static_assert(MC == 8 || NT == 1, "column packing needs a single n8 tile");
    std::uint32_t xsel[NT][BC];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < BC; ++j) {
            const std::uint32_t row = nt * 8 + g % MC;
            const bool real = (g / MC == j) && row < p.x_rows;
            xsel[nt][j] = smem_u32(xs) + (real ? row : p.x_zero_row) * p.x_stride + 8 * t;
        }
    // Blocks whose scales this lane applies: columns 2t and 2t+1 belong to
    // chain positions (2t)/MC and (2t+1)/MC.
    const std::uint32_t doff0 = 18u * static_cast<std::uint32_t>((2 * t) / MC);
    const std::uint32_t doff1 = 18u * static_cast<std::uint32_t>((2 * t + 1) / MC);
    const std::uint32_t ring_addr = smem_u32(ring) + g * kRowStride;

    std::uint32_t slot = 0;
    for (std::uint32_t tl = 0; tl < my_tiles; ++tl) {
        for (std::uint32_t st = 0; st < spt; ++st) {
            // Keep STAGES-1 stages in flight: refill the slot freed by the
            // previous stage, then wait for this one (own groups only; the
            // warp's lanes together fetched the stage).
            issue();
            cp_async_wait<STAGES - 1>();
            __syncwarp();
            {
                // Row g of the stage at ra, row g+8 at ra + 8 rows; qa points
                // at this lane's quant words (4t bytes further).
                const std::uint32_t ra = ring_addr + slot * kStageBytes;
                const std::uint32_t qa = ra + 4 * t;
                constexpr std::uint32_t kR8 = 8 * kRowStride;
                const std::uint32_t xo = (u0 - pu0 + st) * (kUnitBlocks * 64);
                std::uint32_t xs_j[NT][BC];  // this lane's B rows for this unit
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int j = 0; j < BC; ++j) xs_j[nt][j] = xsel[nt][j] + xo;
                const std::uint32_t da0 = ra + doff0;
                const std::uint32_t da1 = ra + doff1;
                // Long chains (8/MC >= 4 blocks) keep the low- and high-nibble
                // MMAs in two accumulators so consecutive MMAs are independent.
                constexpr int NCH = BC >= 4 ? 2 : 1;
                static_for<0, kUnitBlocks / BC>([&](auto cc) {
                    constexpr int c = decltype(cc)::value;
                    float dacc[NCH][NT][4];
#pragma unroll
                    for (int h = 0; h < NCH; ++h)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            dacc[h][nt][0] = dacc[h][nt][1] = dacc[h][nt][2] = dacc[h][nt][3] = 0.f;

                    static_for<0, BC>([&](auto jj) {
                        constexpr int j = decltype(jj)::value;
                        constexpr int b = c * BC + j;
                        // Quant word t of block b (qs at byte 18b + 2): aligned
                        // for odd b, straddling two words for even b.
                        std::uint32_t wa, wb;
                        if constexpr (b & 1) {
                            wa = lds32i<18 * b + 2>(qa);
                            wb = lds32i<kR8 + 18 * b + 2>(qa);
                        } else {
                            wa = prmt(lds32i<18 * b>(qa), lds32i<18 * b + 4>(qa), 0x5432u);
                            wb = prmt(lds32i<kR8 + 18 * b>(qa), lds32i<kR8 + 18 * b + 4>(qa),
                                      0x5432u);
                        }
                        std::uint32_t al02, al13, ah02, ah13, bl02, bl13, bh02, bh13;
                        decode_word(wa, al02, al13, ah02, ah13);
                        decode_word(wb, bl02, bl13, bh02, bh13);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const uint2 xl = lds64i<b * 64>(xs_j[nt][j]);
                            const uint2 xh = lds64i<b * 64 + 32>(xs_j[nt][j]);
                            mma_16816(dacc[0][nt], al02, bl02, al13, bl13, xl.x, xl.y,
                                      dacc[0][nt]);
                            mma_16816(dacc[NCH - 1][nt], ah02, bh02, ah13, bh13, xh.x, xh.y,
                                      dacc[NCH - 1][nt]);
                        }
                    });
                    // Scale each column's block partial by its block's d.
                    constexpr int cb = 18 * (c * BC);
                    const float dg0 = half_bits_to_float(lds16i<cb>(da0));
                    const float dh0 = half_bits_to_float(lds16i<cb + kR8>(da0));
                    float dg1 = dg0, dh1 = dh0;
                    if constexpr (MC == 1) {
                        dg1 = half_bits_to_float(lds16i<cb>(da1));
                        dh1 = half_bits_to_float(lds16i<cb + kR8>(da1));
                    }
#pragma unroll
                    for (int h = 0; h < NCH; ++h)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            if constexpr (NT == 2) {
                                // packed f32x2 (each lane rounds as fmaf): measured
                                // faster with two n8 tiles of tokens only
                                fma_pair(acc[nt][0], acc[nt][1], dg0, dg1, dacc[h][nt][0],
                                         dacc[h][nt][1]);
                                fma_pair(acc[nt][2], acc[nt][3], dh0, dh1, dacc[h][nt][2],
                                         dacc[h][nt][3]);
                            } else {
                                acc[nt][0] = fmaf(dg0, dacc[h][nt][0], acc[nt][0]);
                                acc[nt][1] = fmaf(dg1, dacc[h][nt][1], acc[nt][1]);
                                acc[nt][2] = fmaf(dh0, dacc[h][nt][2], acc[nt][2]);
                                acc[nt][3] = fmaf(dh1, dacc[h][nt][3], acc[nt][3]);
                            }
                        }
                });
            }
            __syncwarp();  // the slot is refilled by the next iteration's issue
            slot = slot + 1 == STAGES ? 0 : slot + 1;
        }
        // Fold packed columns back to one value per activation row, in the
        // unpacked layout (lane t holds rows 2t, 2t+1): rows of a column
        // group live in lanes with equal (2t) % MC.
        if constexpr (MC < 8) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if constexpr (MC == 1) {
                    if (i & 1) continue;
                    acc[0][i] += acc[0][i + 1];
                    acc[0][i + 1] = 0.f;
                }
                if constexpr (MC <= 2) acc[0][i] += __shfl_xor_sync(0xffffffffu, acc[0][i], 1);
                acc[0][i] += __shfl_xor_sync(0xffffffffu, acc[0][i], 2);
            }
        }
        const std::uint32_t tile = first + tl * stride;
        // The part's sums for a tile (warp-uniform call): stored directly
        // with one part; otherwise parked in the workspace, and the last
        // part to arrive adds all parts in part order and stores.
        auto finish = [&](const float (&v)[NT][4]) {
            if (parts == 1) {
                store_tile<NT, XF32, OF32, EPI>(p, tile, g, t, v, stage);
                return;
            }
            float* slot = p.part_buf + (static_cast<std::uint64_t>(part) * p.tiles + tile) * (NT * 128);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) slot[(nt * 4 + i) * 32 + lane] = v[nt][i];
            __threadfence();
            __syncwarp();
            unsigned before = 0;
            if (lane == 0) before = atomicAdd(&p.part_cnt[tile], 1u);
            before = __shfl_sync(0xffffffffu, before, 0);
            if (before != parts - 1) return;
            __threadfence();
            float total[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) total[nt][i] = 0.f;
            for (std::uint32_t q = 0; q < parts; ++q) {
                const float* src = p.part_buf + (static_cast<std::uint64_t>(q) * p.tiles + tile) * (NT * 128);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) total[nt][i] += __ldcg(src + (nt * 4 + i) * 32 + lane);
            }
            if (lane == 0) p.part_cnt[tile] = 0u;  // ready for the next call
            store_tile<NT, XF32, OF32, EPI>(p, tile, g, t, total, stage);
        };
        if (split == 1) {  // the warp covered all of its part of K
            finish(acc);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
            continue;
        }
        // Meet the group's other K-slices in its double-buffered reduction
        // area: the writer of buffer b for tile tl+2 passes tile tl+1's
        // barrier only after the reducer of tile tl has read buffer b.
        float* gred = red + grp * 2 * split * (NT * 4 * 32);
        float* mine = gred + ((tl & 1u) * split + wig) * (NT * 4 * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                mine[(nt * 4 + i) * 32 + lane] = acc[nt][i];
                acc[nt][i] = 0.f;
            }
        named_barrier_sync(1 + static_cast<int>(grp), static_cast<int>(split) * 32);
        if ((tl & (split - 1)) == wig) {
            float sum[NT][4];
            const float* base = gred + (tl & 1u) * split * (NT * 4 * 32);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sum[nt][i] = 0.f;
            for (std::uint32_t w = 0; w < split; ++w)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        sum[nt][i] += base[w * (NT * 4 * 32) + (nt * 4 + i) * 32 + lane];
            finish(sum);
        }
    }
    if constexpr (EPI == kEpiPeers) peer_handshake(p);
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
    const int nmat = epi_swiglu(EPI) ? 2 : 1;
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
        if constexpr (epi_swiglu(EPI)) v = silu_mul(acc[0][mm], acc[1][mm]);
        if constexpr (EPI == kEpiResidual) v += __half2float(p.res[m * p.ldy + warp_global]);
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
// device (the attribute is per device; `done` is a bit mask of ordinals below
// 64; higher ordinals set it on every call).
template <typename Kernel>
int ensure_smem_attribute(Kernel kernel, int bytes, std::atomic<std::uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    const std::uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return kSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    done.fetch_or(bit, std::memory_order_acq_rel);
    return kSuccess;
}

// Streaming multiprocessors of the current device (cached per ordinal).
inline int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    const bool cached = dev >= 0 && dev < 64;
    int v = cached ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        if (cached) cache[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

template <int NT, int MC, bool XF32, bool OF32, int EPI, int STAGES>
int launch_gemv(const Params& p, int ctas_per_sm, cudaStream_t stream) {
    auto kernel = q4_0_gemv_kernel<NT, MC, XF32, OF32, EPI, STAGES>;
    static std::atomic<std::uint64_t> configured{0};
    const int st = ensure_smem_attribute(kernel, kMaxSmem, configured);
    if (st != kSuccess) return st;
    const std::uint32_t groups = kWarps >> p.split_shift;
    // CTAs per part of K; the grid holds the same number for every part
    const std::uint32_t cap = max(1u, static_cast<std::uint32_t>(sm_count() * ctas_per_sm) / p.parts);
    std::uint32_t grid = min((p.tiles + groups - 1) / groups, cap) * p.parts;
    if (EPI == kEpiPeers && grid == 0) grid = 1;  // every rank joins the handshake
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes(static_cast<int>(p.x_bytes), NT, STAGES, EPI == kEpiPeers);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <bool XF32, bool OF32, int EPI, int NT, int MC>
int launch_gemv_stages(const Params& p, int stages, int ctas, cudaStream_t stream) {
    switch (stages) {
        case 4: return launch_gemv<NT, MC, XF32, OF32, EPI, 4>(p, ctas, stream);
        case 3: return launch_gemv<NT, MC, XF32, OF32, EPI, 3>(p, ctas, stream);
        default: return launch_gemv<NT, MC, XF32, OF32, EPI, 2>(p, ctas, stream);
    }
}

// Staged activation rows select the MMA column layout: more than 8 rows take
// two n8 tiles; otherwise the rows are packed MC to a column group.
template <bool XF32, bool OF32, int EPI>
int launch_gemv_config(const Params& p, int stages, int ctas, cudaStream_t stream) {
    if (p.x_rows > 8) return launch_gemv_stages<XF32, OF32, EPI, 2, 8>(p, stages, ctas, stream);
    if (p.x_rows > 4) return launch_gemv_stages<XF32, OF32, EPI, 1, 8>(p, stages, ctas, stream);
    if (p.x_rows > 2) return launch_gemv_stages<XF32, OF32, EPI, 1, 4>(p, stages, ctas, stream);
    if (p.x_rows > 1) return launch_gemv_stages<XF32, OF32, EPI, 1, 2>(p, stages, ctas, stream);
    return launch_gemv_stages<XF32, OF32, EPI, 1, 1>(p, stages, ctas, stream);
}

// Picks tokens per launch, n8 tiles and ring depth so the staged
// activations fit next to the ring.  Returns false if not even one token
// fits (then the generic kernel runs).
inline bool plan_gemv(std::uint64_t M, std::uint64_t K, bool xf32, bool peers, std::uint32_t& tokens,
                      int& nt, int& stages, int& ctas_per_sm, std::uint32_t& x_rows,
                      std::uint32_t& x_stride, std::uint32_t& x_bytes) {
    const std::uint32_t rows_per_token = xf32 ? 2 : 1;
    std::uint32_t m = static_cast<std::uint32_t>(
        M < static_cast<std::uint64_t>(kMaxXRows / rows_per_token) ? M : kMaxXRows / rows_per_token);
    if (K > (1ull << 24)) return false;
    x_stride = static_cast<std::uint32_t>(K * 2 + 32);
    // Preference: two CTAs per SM (16 warps to hide latency) with a deep
    // ring, then one CTA per SM with the deepest ring that fits.
    constexpr int kOptions[5][2] = {{2, 4}, {2, 3}, {1, 4}, {1, 3}, {1, 2}};
    for (; m >= 1; m = m / 2) {
        x_rows = m * rows_per_token;
        x_bytes = ((x_rows + 1) * x_stride + 127u) & ~127u;  // + the zero row
        nt = x_rows <= 8 ? 1 : 2;
        for (const auto& opt : kOptions) {
            const int bytes = smem_bytes(static_cast<int>(x_bytes), nt, opt[1], peers);
            if (bytes <= kMaxSmem && opt[0] * (bytes + kSmemReservedPerCta) <= kSmemPerSm) {
                ctas_per_sm = opt[0];
                stages = opt[1];
                tokens = m;
                return true;
            }
        }
        if (m == 1) break;
    }
    return false;
}

// log2 of the warps per tile (split-K factor).  Measured with every split
// forced (K = 2048..8192, 128..8016 tiles, 8 or 16 warps per SM), the best
// split follows r = 1.2 x (warps / tiles).  With the whole K in one CTA:
// 8 warps per tile for r >= 5.66 (small problems spread every tile over a
// CTA), 4 for r >= 2, else 2 -- whole tiles per warp were never the
// fastest: at lm_head size (r = 0.18..0.35) pairs of warps beat them by
// 3.5-4.6 %, the rounds of tiles per group divide more evenly.  With K
// split over `parts` CTAs (a quarter of K each, two n8 token tiles) every
// extra split costs more: 2 warps from r >= 1.41, 4 from 2.83, 8 from 5.66.
inline std::uint32_t choose_split_shift(std::uint32_t tiles, std::uint32_t units,
                                        std::uint32_t ctas, std::uint32_t parts) {
    const double r = 1.2 * kWarps * static_cast<double>(ctas) / static_cast<double>(tiles);
    std::uint32_t sh = parts > 1 ? (r >= 1.4142) + (r >= 2.8284) + (r >= 5.6569)
                                 : 1 + (r >= 2.0) + (r >= 5.6569);
    while (sh > 0 && (1u << sh) > units) --sh;
    return sh;
}

// Runs the linear for M rows of x, in as few persistent launches as the
// activation staging allows (consecutive launches on the same stream).
// Workspace of a K split over `parts` CTAs.  The first kCounterBytes hold
// one arrival counter per tile (tile t at word t, for up to kCounterTiles
// tiles) at a fixed place: the counters must be zero before the first call,
// every call leaves them zero, and no call ever writes partial sums there,
// whatever the shapes of earlier calls.  The partial sums [parts][tiles]
// [nt * 128] floats follow.
constexpr std::uint64_t kCounterTiles = 65536;
constexpr std::uint64_t kCounterBytes = kCounterTiles * 4;
inline std::uint64_t part_workspace_bytes(std::uint64_t parts, std::uint64_t tiles, int nt) {
    return kCounterBytes + parts * tiles * nt * 128 * 4;
}

// Status of mote_cuda_quantized_linear_q4_0_f16_noalloc when the request's
// K split needs more than its static scratch (above every CUDA runtime code).
constexpr int kScratchTooSmall = 10200;

// kEpiPeers destinations and handshake flags (see peer_handshake).
struct PeerArgs {
    __half* const* outputs;
    unsigned* const* flags;
    unsigned* own_flags;
    std::uint64_t col0;
    std::uint32_t rank;
    std::uint32_t nranks;
    // kEpiNorm*: RMSNorm of the staged rows
    const __half* gamma;
    float eps;
    // kEpiNormRope: the first rope_rows output rows are rope_rows / head_dim
    // heads rotated with cos/sin [M, head_dim/2] (f32); tiles below
    // rope_tiles pair rows d and d + head_dim/2 of a head
    const float* rope_cos;
    const float* rope_sin;
    std::uint32_t rope_rows;
    std::uint32_t rope_tiles;
    std::uint32_t head_dim;
    // K split across CTAs: CTA b works on part b % parts of K (its own
    // units and activation columns); the parts of a tile meet in the
    // workspace -- partial sums part_buf[part][tile][NT*128] and arrival
    // counters part_cnt[tile] (zero between calls: the last part to arrive
    // adds the partials in part order, stores and resets its counter)
    std::uint32_t parts;
    float* part_buf;
    unsigned* part_cnt;
};

template <bool XF32, bool OF32, int EPI>
int run_linear(const void* x, const void* w, const void* w2, void* y, std::uint64_t M,
               std::uint64_t N, std::uint64_t K, std::uint64_t ldy, cudaStream_t stream,
               const void* res = nullptr, const PeerArgs* peers = nullptr,
               const Params* fused = nullptr, void* workspace = nullptr,
               std::uint64_t workspace_bytes = 0, bool workspace_must_fit = false) {
    const std::size_t osz = OF32 ? 4 : 2;
    // epilogues that exist only on the fast path
    constexpr bool kFastOnly = EPI == kEpiPeers || epi_norm(EPI);
    if constexpr (EPI == kEpiPeers) {
        if (peers == nullptr) return kInvalidValue;
    }
    if constexpr (epi_norm(EPI)) {
        if (fused == nullptr) return kInvalidValue;
    }
    if constexpr (kFastOnly) {
        if (K == 0) return kInvalidValue;
    }
    if (K == 0) {
        // Every dot product is empty: the reference writes zeros
        // (crates/mote-backend-hip/tests/quantized_linear.rs:142-158).  For
        // SwiGLU silu(0) * 0 = 0 as well.
        if constexpr (EPI == kEpiResidual) {
            // empty dot products: y = residual
            if (y == res) return kSuccess;
            return static_cast<int>(cudaMemcpy2DAsync(y, ldy * osz, res, ldy * osz, N * osz, M,
                                                      cudaMemcpyDeviceToDevice, stream));
        }
        return static_cast<int>(cudaMemset2DAsync(y, ldy * osz, 0, N * osz, M, stream));
    }
    // Prefill-shaped problems (more tokens than one GEMV launch stages) run as
    // a dense contraction on the tcgen05 tensor cores.
    if constexpr (!XF32 && EPI == kEpiPlain) {
        if (M > static_cast<std::uint64_t>(kMaxXRows) && ldy == N &&
            gemm::supported(x, w, y, M, N, K, osz))
        {
            // the workspace past the tile counters holds the split parts
            void* parts = nullptr;
            std::uint64_t parts_bytes = 0;
            if (workspace != nullptr && workspace_bytes > kCounterBytes) {
                parts = static_cast<std::uint8_t*>(workspace) + kCounterBytes;
                parts_bytes = workspace_bytes - kCounterBytes;
            }
            return gemm::launch<OF32>(x, w, y, M, N, K, stream, parts, parts_bytes);
        }
    }
    Params p{};
    p.w = static_cast<const std::uint8_t*>(w);
    p.res = static_cast<const __half*>(res);
    p.w2 = static_cast<const std::uint8_t*>(w2);
    p.N = static_cast<std::uint32_t>(N);
    p.K = K;
    p.pitch = (K / 32) * 18;
    p.units = static_cast<std::uint32_t>(K / 256);
    p.ldy = ldy;
    if (peers != nullptr) {
        p.peer_y = peers->outputs;
        p.peer_flags = peers->flags;
        p.own_flags = peers->own_flags;
        p.col0 = peers->col0;
        p.rank = peers->rank;
        p.nranks = peers->nranks;
    }
    if (fused != nullptr) {
        p.gamma = fused->gamma;
        p.eps = fused->eps;
        p.rope_cos = fused->rope_cos;
        p.rope_sin = fused->rope_sin;
        p.rope_rows = fused->rope_rows;
        p.rope_tiles = fused->rope_tiles;
        p.head_dim = fused->head_dim;
    }
    const std::uint64_t rows_per_tile = epi_swiglu(EPI) ? 8 : 16;
    p.tiles = static_cast<std::uint32_t>((N + rows_per_tile - 1) / rows_per_tile);
    if constexpr (epi_rope(EPI))
        p.tiles = p.rope_tiles + static_cast<std::uint32_t>((N - p.rope_rows + 15) / 16);
    const std::size_t xes = XF32 ? 4 : 2;
    bool fast = (K % 256 == 0) && (reinterpret_cast<std::uintptr_t>(w) % 16 == 0) &&
                (reinterpret_cast<std::uintptr_t>(x) % 16 == 0);
    if (epi_swiglu(EPI)) fast = fast && (reinterpret_cast<std::uintptr_t>(w2) % 16 == 0);
    std::uint32_t tokens = 0;
    int nt = 1, stages = 2, ctas = 1;
    if (fast)
        fast = plan_gemv(M, K, XF32, EPI == kEpiPeers, tokens, nt, stages, ctas, p.x_rows,
                         p.x_stride, p.x_bytes);
    if (kFastOnly && !fast) return kInvalidValue;
    if constexpr (EPI == kEpiPeers) {
        // More than 16 tokens: the tcgen05 GEMM with the peer-store epilogue
        // and one handshake per call on every rank (the token count is the
        // same on every rank; a rank without real rows only joins the
        // handshake).
        if (M > static_cast<std::uint64_t>(kMaxXRows)) {
            const gemm::Peers gp{p.peer_y, p.peer_flags, p.own_flags, p.col0, ldy,
                                 p.rank,   p.nranks};
            if (N == 0) return gemm::launch_handshake_only(gp, stream);
            return gemm::launch_peers(x, w, M, N, K, gp, stream);
        }
    }
    p.parts = 1;
    // With a workspace, when the staged activations leave room for only one
    // CTA per SM, split K over 2 or 4 CTAs: each stages its part's columns
    // only, two CTAs fit per SM, and the parts meet in the workspace.
    if constexpr (!kFastOnly) {
        // Measured on the decode sweep (16 tokens, K = 4096): the split into
        // four parts (two CTAs per SM) beats the unsplit three-stage ring at
        // 896 tiles (17.5 vs 17.8 us) but loses at 688 and 256 tiles (16.4 vs
        // 14.8 us, 8.8 vs 8.4 us: fewer tile rounds per warp group, and the
        // partial sums' fences stall); with 8 or fewer tokens, or lm_head-sized
        // N, the unsplit kernel is faster.
        if (fast && workspace != nullptr && ctas == 1 && nt == 2 && p.tiles >= 850 &&
            p.tiles <= 4096) {
            for (std::uint32_t parts = 2; parts <= 4; parts *= 2) {
                if (p.units < parts) break;
                const std::uint64_t kp = ((p.units + parts - 1) / parts) * 256ull;
                std::uint32_t tk = 0, xr = 0, xst = 0, xb = 0;
                int nt2 = 1, st2 = 2, c2 = 1;
                if (!plan_gemv(M, kp, XF32, false, tk, nt2, st2, c2, xr, xst, xb)) continue;
                if (c2 < 2 || tk < tokens) continue;
                if (part_workspace_bytes(parts, p.tiles, nt2) > workspace_bytes) {
                    // a fixed-size workspace that cannot hold the split
                    if (workspace_must_fit) return kScratchTooSmall;
                    continue;
                }
                p.parts = parts;
                stages = st2;
                ctas = c2;
                p.x_stride = xst;
                p.x_bytes = xb;
                p.part_cnt = static_cast<unsigned*>(workspace);
                p.part_buf = reinterpret_cast<float*>(static_cast<std::uint8_t*>(workspace) +
                                                      kCounterBytes);
                break;
            }
        }
    }
    if (fast)
        p.split_shift = choose_split_shift(
            p.tiles, (p.units + p.parts - 1) / p.parts,
            max(1u, static_cast<std::uint32_t>(sm_count() * ctas) / p.parts), p.parts);
    const std::uint64_t chunk = fast ? tokens : kGenericTokens * 65535ull;
    for (std::uint64_t m0 = 0; m0 < M; m0 += chunk) {
        const std::uint64_t mc = (M - m0 < chunk) ? (M - m0) : chunk;
        p.M = static_cast<std::uint32_t>(mc);
        p.x = static_cast<const std::uint8_t*>(x) + m0 * K * xes;
        p.y = static_cast<std::uint8_t*>(y) + m0 * ldy * osz;
        if (res != nullptr) p.res = static_cast<const __half*>(res) + m0 * ldy;
        if (fused != nullptr && fused->rope_cos != nullptr) {  // per-token RoPE tables
            p.rope_cos = fused->rope_cos + m0 * (fused->head_dim / 2);
            p.rope_sin = fused->rope_sin + m0 * (fused->head_dim / 2);
        }
        int st;
        if (fast) {
            p.x_rows = static_cast<std::uint32_t>(mc) * (XF32 ? 2 : 1);
            p.x_zero_row = p.x_rows;
            st = launch_gemv_config<XF32, OF32, EPI>(p, stages, ctas, stream);
        } else if constexpr (!kFastOnly) {
            const dim3 grid(static_cast<unsigned>((N + 3) / 4),
                            static_cast<unsigned>((mc + kGenericTokens - 1) / kGenericTokens));
            q4_0_linear_generic_kernel<XF32, OF32, EPI><<<grid, 128, 0, stream>>>(p);
            st = static_cast<int>(cudaGetLastError());
        } else {
            st = kInvalidValue;
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
constexpr int kEmpty = -2;
inline int check_linear_args(const void* x, const void* w, const void* y, std::uint64_t rows,
                             std::uint64_t n, std::uint64_t k, const void* stream) {
    if (x == nullptr || w == nullptr || y == nullptr || stream == nullptr) return kInvalidValue;
    if (k % 32 != 0) return kInvalidValue;
    if (rows == 0 || n == 0) return kEmpty;
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
    if (c == kEmpty) return mote::kSuccess;
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
    if (c == kEmpty) return mote::kSuccess;
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
    if (c == kEmpty) return mote::kSuccess;
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
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    return run_linear<false, false, kEpiSwiGLU>(input, gate_weights, up_weights, output, rows,
                                                ffn_features, input_features, ffn_features,
                                                static_cast<cudaStream_t>(stream));
}

// output = input * weights^T + residual (f16 in, f16 residual/out, f32
// accumulation, one rounding).  No reference counterpart: the decoder layer's
// down projection with its residual add.  output may alias residual (each
// element is read and written by the same thread); argument rules as the
// linear entry points, plus a null residual is an invalid value.
extern "C" int mote_cuda_quantized_linear_q4_0_f16_residual(const void* input, const void* weights,
                                                            const void* residual, void* output,
                                                            std::uint64_t rows,
                                                            std::uint64_t output_features,
                                                            std::uint64_t input_features,
                                                            void* stream) {
    using namespace mote::q4;
    if (residual == nullptr) return mote::kInvalidValue;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    return run_linear<false, false, kEpiResidual>(input, weights, nullptr, output, rows,
                                                  output_features, input_features,
                                                  output_features,
                                                  static_cast<cudaStream_t>(stream), residual);
}

// Column-sharded linear with the all-gather fused into the epilogue: this
// rank's rows [rank * shard, rank * shard + shard) of the full weight matrix
// (`weights` holds only those rows) produce output columns that are stored
// directly into every rank's full output buffer [rows, total_features]
// (outputs: device array of nranks pointers, peers mapped over CUDA IPC),
// followed by the flag handshake of the peer all-gather.  No reference
// counterpart.  Fast-path shapes only (K % 256 == 0, K > 0, 16-byte aligned
// input and weights, total_features % 8 == 0); every rank must pass the
// same rows.
extern "C" int mote_cuda_quantized_linear_q4_0_f16_allgather(
    const void* input, const void* weights, void* const* outputs, unsigned* const* flag_ptrs,
    unsigned* own_flags, std::uint64_t rows, std::uint64_t shard_features,
    std::uint64_t input_features, std::uint64_t total_features, std::uint32_t rank,
    std::uint32_t nranks, void* stream) {
    using namespace mote::q4;
    if (outputs == nullptr || flag_ptrs == nullptr || own_flags == nullptr || nranks == 0 ||
        rank >= nranks || shard_features % 16 != 0 || total_features % 8 != 0)
        return mote::kInvalidValue;
    const int c = check_linear_args(input, weights, outputs, rows, total_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    if (input_features == 0 || input_features % 256 != 0) return mote::kInvalidValue;
    const std::uint64_t col0 = static_cast<std::uint64_t>(rank) * shard_features;
    const std::uint64_t real = col0 >= total_features
                                   ? 0
                                   : (total_features - col0 < shard_features ? total_features - col0
                                                                             : shard_features);
    PeerArgs peers{reinterpret_cast<__half* const*>(outputs), flag_ptrs, own_flags, col0, rank,
                   nranks};
    return run_linear<false, false, kEpiPeers>(input, weights, nullptr, nullptr, rows, real,
                                               input_features, total_features,
                                               static_cast<cudaStream_t>(stream), nullptr, &peers);
}

// ---------------------------------------------------------------------------
// Decoder-layer fusions.  No reference counterparts: the reference runs
// rms_norm_f16 (crates/mote-backend-hip/src/rms_norm.hip) and the linear as
// separate launches.  Each takes f16 input rows, RMS-normalises them with
// gamma (eps finite and >= 0) inside the projection's activation staging,
// then projects.  Fast-path shapes only: K % 256 == 0, K > 0, 16-byte
// aligned input, gamma and weights; otherwise 1.  rows == 0 or no output
// features -> 0 without a launch; rows * N beyond 32 bits -> 9.
// ---------------------------------------------------------------------------
namespace mote {
namespace q4 {
inline int check_fused_norm(const void* gamma, float eps) {
    if (gamma == nullptr || !isfinite(eps) || eps < 0.0f) return kInvalidValue;
    if (reinterpret_cast<std::uintptr_t>(gamma) % 16 != 0) return kInvalidValue;
    return kSuccess;
}
}  // namespace q4
}  // namespace mote

extern "C" int mote_cuda_q4_0_rms_norm_linear_f16(const void* input, const void* gamma,
                                                  const void* weights, void* output,
                                                  std::uint64_t rows,
                                                  std::uint64_t output_features,
                                                  std::uint64_t input_features, float epsilon,
                                                  void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    if (const int n = check_fused_norm(gamma, epsilon); n != 0) return n;
    Params f{};
    f.gamma = static_cast<const __half*>(gamma);
    f.eps = epsilon;
    return run_linear<false, false, kEpiNormPlain>(input, weights, nullptr, output, rows,
                                                   output_features, input_features,
                                                   output_features,
                                                   static_cast<cudaStream_t>(stream), nullptr,
                                                   nullptr, &f);
}

extern "C" int mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16(
    const void* input, const void* gamma, const void* gate_weights, const void* up_weights,
    void* output, std::uint64_t rows, std::uint64_t ffn_features, std::uint64_t input_features,
    float epsilon, void* stream) {
    using namespace mote::q4;
    if (up_weights == nullptr) return mote::kInvalidValue;
    const int c = check_linear_args(input, gate_weights, output, rows, ffn_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    if (const int n = check_fused_norm(gamma, epsilon); n != 0) return n;
    Params f{};
    f.gamma = static_cast<const __half*>(gamma);
    f.eps = epsilon;
    return run_linear<false, false, kEpiNormSwiGLU>(input, gate_weights, up_weights, output, rows,
                                                    ffn_features, input_features, ffn_features,
                                                    static_cast<cudaStream_t>(stream), nullptr,
                                                    nullptr, &f);
}

// QKV projection of a decoder layer: output [rows, (q_heads + 2 kv_heads) *
// head_dim] = norm(input) @ W^T, with RoPE (HalfSplit, rotary_dim =
// head_dim) applied to the q and k heads from the f32 accumulators, cos/sin
// f32 [rows, head_dim/2] as mote_cuda_rope_f16 takes them.  head_dim a
// multiple of 16.
extern "C" int mote_cuda_q4_0_rms_norm_qkv_rope_f16(
    const void* input, const void* gamma, const void* weights, const void* cos, const void* sin,
    void* output, std::uint64_t rows, std::uint64_t q_heads, std::uint64_t kv_heads,
    std::uint64_t head_dim, std::uint64_t input_features, float epsilon, void* stream) {
    using namespace mote::q4;
    if (cos == nullptr || sin == nullptr) return mote::kInvalidValue;
    if (head_dim == 0 || head_dim % 16 != 0 || head_dim > 65536 || q_heads > 65536 ||
        kv_heads > 65536)
        return mote::kInvalidValue;
    if ((reinterpret_cast<std::uintptr_t>(cos) | reinterpret_cast<std::uintptr_t>(sin)) % 4 != 0)
        return mote::kInvalidValue;
    const std::uint64_t n = (q_heads + 2 * kv_heads) * head_dim;
    const int c = check_linear_args(input, weights, output, rows, n, input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    if (const int e = check_fused_norm(gamma, epsilon); e != 0) return e;
    Params f{};
    f.gamma = static_cast<const __half*>(gamma);
    f.eps = epsilon;
    f.rope_cos = static_cast<const float*>(cos);
    f.rope_sin = static_cast<const float*>(sin);
    f.head_dim = static_cast<std::uint32_t>(head_dim);
    f.rope_rows = static_cast<std::uint32_t>((q_heads + kv_heads) * head_dim);
    f.rope_tiles = f.rope_rows / 16;
    return run_linear<false, false, kEpiNormRope>(input, weights, nullptr, output, rows, n,
                                                  input_features, n,
                                                  static_cast<cudaStream_t>(stream), nullptr,
                                                  nullptr, &f);
}

// The f16 linear with a caller workspace (zeroed once before its first use;
// every call leaves its first 256 KiB -- the tile counters -- zero again).
// When a launch stages more than 8 activation rows and they would leave
// room for only one CTA per SM (9 or more tokens at K = 4096), and N has at
// most 4096 row tiles, K is split over 2 or 4 CTAs through the workspace; with a null or
// too small workspace the call behaves as mote_cuda_quantized_linear_q4_0_f16.
// Calls sharing a workspace must not overlap (one stream per workspace).
// No reference counterpart.
extern "C" int mote_cuda_quantized_linear_q4_0_f16_ws(const void* input, const void* weights,
                                                      void* output, std::uint64_t rows,
                                                      std::uint64_t output_features,
                                                      std::uint64_t input_features,
                                                      void* workspace,
                                                      std::uint64_t workspace_bytes,
                                                      void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    if (workspace != nullptr && reinterpret_cast<std::uintptr_t>(workspace) % 256 != 0)
        return mote::kInvalidValue;
    return run_linear<false, false, kEpiPlain>(input, weights, nullptr, output, rows,
                                               output_features, input_features, output_features,
                                               static_cast<cudaStream_t>(stream), nullptr,
                                               nullptr, nullptr, workspace, workspace_bytes);
}

// Workspace size that lets mote_cuda_quantized_linear_q4_0_f16_ws use its
// widest K split for these sizes (an upper bound; 0 if no split applies).
extern "C" int mote_cuda_q4_0_linear_workspace_bytes(std::uint64_t rows,
                                                     std::uint64_t output_features,
                                                     std::uint64_t input_features,
                                                     std::uint64_t* bytes) {
    using namespace mote::q4;
    if (bytes == nullptr) return mote::kInvalidValue;
    *bytes = 0;
    if (rows == 0 || output_features == 0 || input_features % 256 != 0 || input_features == 0)
        return mote::kSuccess;
    const std::uint64_t tiles = (output_features + 15) / 16;
    if (tiles <= kCounterTiles) *bytes = part_workspace_bytes(4, tiles, 2);
    if (rows > static_cast<std::uint64_t>(kMaxXRows) && output_features % 16 == 0) {
        // tcgen05 shapes: the K split of a partial last wave
        const std::uint64_t split = mote::gemm::split_workspace_bytes(rows, output_features,
                                                                      input_features);
        if (split != 0 && kCounterBytes + split > *bytes) *bytes = kCounterBytes + split;
    }
    return mote::kSuccess;
}

// ---------------------------------------------------------------------------
// No-allocation variant of mote_cuda_quantized_linear_q4_0_f16_ws.
//
// For callers that cannot allocate or pass a workspace -- e.g. a kernel
// resolved through mote-kernel's KernelImpl::launch, which receives only the
// opaque argument words -- the split-K scratch is a file-scope device array,
// one per device, zero at module load (its tile counters must be zero before
// a call, and every call leaves them zero).  Its address is looked up with
// cudaGetSymbolAddress the first time a device is used from a CUDA context
// and again whenever that device's current context changes (after a
// cudaDeviceReset the module, and with it the array, is loaded anew); no
// memory is allocated.  Limits: kNoAllocScratchBytes of scratch per device;
// on the decode path (at most 16 tokens per launch) a request whose K split
// needs more returns kScratchTooSmall (10200) before anything is enqueued,
// even where an unsplit launch would fit, while prefill shapes (more than 16
// tokens, the tensor-core GEMM) run their last wave unsplit instead; device
// ordinals from kNoAllocDevices up are rejected (1); and one scratch per
// device, so calls on that device must not overlap (on any stream).  The
// first call on a device performs the lookup and must be made before any
// stream capture that includes this entry point.  No reference counterpart.
// ---------------------------------------------------------------------------
namespace mote {
namespace q4 {
constexpr std::uint64_t kNoAllocScratchBytes = 8ull << 20;  // 8 MiB per device
constexpr int kNoAllocDevices = 64;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name) {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &sym, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        return reinterpret_cast<Fn>(sym);
    return nullptr;
}

// Unique id of the calling thread's current context (0 if there is none).
inline unsigned long long current_context_id() {
    static const CtxGetCurrentFn get = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
    static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
    CUcontext cur = nullptr;
    unsigned long long id = 0;
    if (get == nullptr || get_id == nullptr || get(&cur) != CUDA_SUCCESS || cur == nullptr ||
        get_id(cur, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Address of this device's scratch, cached per device ordinal together with
// the id of the context it was looked up in (context ids are never reused,
// unlike context handles).
inline int noalloc_scratch(void** out) {
    struct Slot {
        std::mutex lock;
        unsigned long long ctx = 0;
        void* addr = nullptr;
    };
    static Slot slots[kNoAllocDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 0 || dev >= kNoAllocDevices) return kInvalidValue;
    Slot& s = slots[dev];
    std::lock_guard<std::mutex> guard(s.lock);
    unsigned long long id = current_context_id();
    if (s.addr == nullptr || id == 0 || s.ctx != id) {
        // the lookup also makes the device's primary context current
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return static_cast<int>(e);
        if (id == 0) id = current_context_id();
        s.addr = p;
        s.ctx = id;
    }
    *out = s.addr;
    return kSuccess;
}
}  // namespace q4
}  // namespace mote

extern "C" int mote_cuda_quantized_linear_q4_0_f16_noalloc(const void* input, const void* weights,
                                                           void* output, std::uint64_t rows,
                                                           std::uint64_t output_features,
                                                           std::uint64_t input_features,
                                                           void* stream) {
    using namespace mote::q4;
    const int c = check_linear_args(input, weights, output, rows, output_features,
                                    input_features, stream);
    if (c == kEmpty) return mote::kSuccess;
    if (c != 0) return c;
    void* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st != mote::kSuccess) return st;
    return run_linear<false, false, kEpiPlain>(input, weights, nullptr, output, rows,
                                               output_features, input_features, output_features,
                                               static_cast<cudaStream_t>(stream), nullptr,
                                               nullptr, nullptr, scratch, kNoAllocScratchBytes,
                                               true);
}
