// Prefill-shaped Q4_0 (and Q8_0, Q4_K, Q6_K) GEMM on the 5th-generation
// tensor cores (tcgen05/TMEM).  The kernel is written for Q4_0; the weight
// format WF selects the raw rows and the converter: Q8_0 stages hold 272-byte
// rows (convert_block_q8), Q4_K stages one 144-byte super-block per row --
// the Q4_0 geometry -- (convert_slice_q4k), Q6_K a 240-byte window around
// each 210-byte super-block (convert_slice_q6k).
//
//   Y[M, N] = X[M, K] * W[N, K]^T,  X f16, W ggml Q4_0 (18-byte blocks), Y f16/f32,
//   for M large enough that the contraction, not the weight stream, bounds
//   the time (the reference computes it in f32 per output,
//   crates/mote-reference/src/quantized.rs:89-144).
//
// One CTA computes a tile of 128 features x 256 tokens.  The dequantized
// weights are the MMA's A operand (M = 128 rows) and the activations its B
// operand (N = 256), so every weight converted to f16 feeds 256 tokens:
// * warp 16 (producer) streams activation tiles (64 k x 256 tokens, TMA
//   with 128-byte swizzle) and raw Q4_0 row slices (128 rows x 144 bytes = 8
//   blocks per row, TMA 2-D tile of bytes) into shared memory, each as soon
//   as a stage of its own ring is free;
// * warps 0-15 (converters, two groups of 8 taking alternate 64-k slices)
//   dequantize each slice of the raw rows into f16 (q - 8) * d -- correctly
//   rounded, exactly what a dense f16 weight would hold -- written straight
//   into the 128-byte-swizzled K-major layout the tensor core reads (in a
//   group, warps 0-3 the even block of the slice, warps 4-7 the odd one: no
//   divergence);
// * warp 17 allocates the TMEM columns and one thread issues
//   tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) per 16-k step,
//   accumulating in f32 in TMEM; tcgen05.commit releases the operand stages;
// * after the last k-slice the converter warps read the accumulator with
//   tcgen05.ld (warp w owns TMEM lanes = features 32*(w%4).. and a slice of
//   the token columns) and store it: for each token, a warp writes 32
//   consecutive features.
// Stages are tracked with mbarriers; every wait is bounded and an expired
// wait aborts the whole CTA (which still frees its TMEM).  No TMA load uses
// cluster multicast.

#include "mote_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <type_traits>

namespace mote {
namespace gemm {

constexpr int kFT = 128;                 // features per tile = A rows = TMEM lanes
constexpr int kBK = 64;                  // k per operand stage (one 128-B f16 swizzle row)
constexpr int kSuperK = 256;             // k per raw weight stage (8 blocks, 144 B per row)
// Four operand stages (4 x 48 KB at TT = 256) keep three 64-k slices of
// MMA work queued behind the one in flight, enough to cover the TMA
// latency of the activation tiles.  Three operand stages ran at 931
// TFLOP/s, four at 1008 (M=2048, K=4096, N=14336, 8 converter warps).
constexpr int kStages = 4;               // operand stages
// Raw weight rows of a 256-k stage: 8 Q4_0 blocks (144 bytes) or 8 Q8_0
// blocks (272 bytes; its TMA box counts 2-byte elements, a box edge being
// at most 256 elements).
constexpr int kWQ4_0 = 0;  // weight formats of the converter
constexpr int kWQ8_0 = 1;
constexpr int kWQ4_K = 2;
constexpr int kWQ6_K = 3;
// Q6_K: a 16-byte-aligned 240-byte window that covers one 210-byte
// super-block (K % 2048 == 0 keeps every row a whole number of 16-byte
// chunks; the block starts 2 * (u mod 8) bytes into the window).  224 bytes
// would cover it, but 240-byte rows (60 words) cut the bank conflicts of the
// converters' per-row loads from 8-way to 4-way; the window of a row's last
// block reaches 16 bytes past the row, which the TMA fills with zeros.
template <int WF>
constexpr int kRawRowBytes = WF == kWQ8_0 ? 272 : WF == kWQ6_K ? 240 : 144;
template <int WF>
constexpr int kRawBytes = kFT * kRawRowBytes<WF>;  // 34 KB or 18 KB
// Converter warps form kConvGroups groups of 8; group g converts the 64-k
// slices kb with kb % kConvGroups == g, so each group has kConvGroups MMA
// slices of time per slice it converts.
constexpr int kConvGroups = 2;
constexpr int kConvWarps = 8 * kConvGroups;
constexpr int kProducerWarp = kConvWarps;
constexpr int kMmaWarp = kConvWarps + 1;
constexpr int kThreads = (kConvWarps + 2) * 32;

// Raw weight stages (256 k each) of a CTA: as many as fit, up to four, in
// the shared memory that keeps the kernel's CTAs per SM (two for TT <= 128,
// one at 256 tokens).  The producer refills a raw stage as soon as the
// converters free it, independently of the activation stages, so the weight
// stream runs that many stages ahead: at 64 tokens a raw stage is converted
// faster than its DRAM latency.
constexpr int raw_stages(int tt, int raw_bytes) {
    const int budget = tt <= 128 ? 115712 : 232448;  // per-CTA shared memory
    const int r = (budget - kStages * tt * kBK * 2 - 2048) / raw_bytes;
    return r < 1 ? 1 : r > 4 ? 4 : r;
}

// The converted weights (the MMA's A operand) live in tensor memory, next
// to the accumulator: the converters write them with tcgen05.st (a warp
// reaches exactly the 32 TMEM lanes = weight rows it converts) and the MMA
// reads A from TMEM.  Against A in shared memory this takes 32 KB per slice
// of traffic off shared memory and the proxy fence off the converters.
constexpr int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p *= 2;
    return p;
}

// Shared-memory layout for a token tile of TT (64, 128 or 256) tokens = the
// MMA's N and the accumulator's TMEM columns: activations TT x 64 k per
// stage (B).
template <int TT, int WF>
struct Layout {
    static constexpr int kXBytes = TT * kBK * 2;
    static constexpr int kOffX = 0;
    static constexpr int kOffRaw = kOffX + kStages * kXBytes;
    // TMEM: accumulator columns [0, TT), then A stage s at kAColBase + 32 s
    // (64 k of f16 = 32 columns of 32 bits per lane)
    static constexpr int kAColBase = TT;
    static constexpr int kTmemCols = pow2_at_least(TT + kStages * 32);
    static_assert(kTmemCols <= 512, "tensor memory");
    static constexpr int kRawStages = raw_stages(TT, kRawBytes<WF>);
    static constexpr int kOffBar = kOffRaw + kRawStages * kRawBytes<WF>;
    // barriers: x_full[S], w_full[S], empty[S], raw_full[R], raw_empty[R], accum
    static constexpr int kNumBars = 3 * kStages + 2 * kRawStages + 1;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kSmemBytes = kOffAbort + 4 + 1024;  // + slack for 1024-B alignment
    static_assert(kSmemBytes <= (TT <= 128 ? 115712 : 232448), "CTAs per SM");
    // Instruction descriptor, kind::f16: F32 accumulate, A = B = F16, both
    // K-major, N >> 3 at bit 17, M >> 4 at bit 24.
    static constexpr std::uint32_t kIdesc = (1u << 4) | (static_cast<std::uint32_t>(TT >> 3) << 17) |
                                            (static_cast<std::uint32_t>(kFT >> 4) << 24);
    static_assert(TT == 64 || TT == 128 || TT == 256, "token tile");
};

// Tiles are numbered feature-tile-fastest: tile t covers features
// 128 * (t % tiles_n) and tokens TT * (t / tiles_n).  CTA b < full computes
// tile b over all of K.  With a workspace, the tiles of a partial last wave
// are split along K instead: CTA full + j computes part j % parts (K/parts
// of K) of tile full + j / parts and stores its f32 accumulator to
// part_buf[j] as [TT tokens][128 features]; q4_0_gemm_reduce_kernel adds
// the parts in part order afterwards.
struct Params {
    void* y;
    std::uint32_t M, N, K;
    std::uint64_t ldy;
    std::uint32_t tiles_n;
    std::uint32_t full;     // CTAs that compute a whole tile
    std::uint32_t parts;    // K parts of a split tile (1: no split)
    float* part_buf;
    // Column-sharded linear with the all-gather fused (PEERS kernels): this
    // rank's f16 results go to every rank's [M, ldy] output at columns
    // col0 + n, then the grid ends with the flag handshake (flag array per
    // rank: [q] epoch of rank q, [nranks] arrival counter, [nranks + 1] own
    // epoch).
    __half* const* peer_y;
    unsigned* const* peer_flags;
    unsigned* own_flags;
    std::uint64_t col0;
    std::uint32_t rank;
    std::uint32_t nranks;
};

// End of a PEERS grid, thread 0 of every CTA after a CTA barrier: one
// cumulative system fence publishes the CTA's peer stores before its arrival
// is counted; the last CTA advances this rank's epoch, stores it to every
// rank's flags (fence + strong relaxed stores: a release pattern) and waits,
// bounded, until every rank's epoch has arrived.
__device__ __forceinline__ void peer_grid_handshake(const Params& p) {
    __threadfence_system();
    const unsigned arrived = atomicAdd(&p.own_flags[p.nranks], 1u);
    if (arrived != gridDim.x - 1) return;
    p.own_flags[p.nranks] = 0u;
    const unsigned epoch = p.own_flags[p.nranks + 1] + 1u;
    p.own_flags[p.nranks + 1] = epoch;
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

// ---- PTX wrappers ------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(std::uint32_t dst, const CUtensorMap* map, int x,
                                            int y, std::uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(std::uint32_t slot_smem, std::uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     slot_smem),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, cta_group::1: A read
// from tensor memory (128 lanes = rows, 8 columns of two f16 = 16 k per
// step), B from shared memory.
__device__ __forceinline__ void umma_f16_ta(std::uint32_t tmem_d, std::uint32_t tmem_a,
                                            std::uint64_t bdesc, std::uint32_t idesc,
                                            std::uint32_t accumulate) {
    const std::uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask), "r"(mask), "r"(mask),
        "r"(mask)
        : "memory");
}

__device__ __forceinline__ void umma_commit(std::uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// 32 lanes x 32 consecutive f32 columns: thread i gets row (lane base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(std::uint32_t taddr, std::uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128
// bytes, 8-row groups 1024 bytes apart (SBO = 64 x 16 B), LBO unused (1),
// descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ std::uint64_t smem_desc_sw128(std::uint32_t addr) {
    std::uint64_t d = 0;
    d |= static_cast<std::uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<std::uint64_t>(1) << 16;   // LBO
    d |= static_cast<std::uint64_t>(64) << 32;  // SBO
    d |= static_cast<std::uint64_t>(1) << 46;   // version
    d |= static_cast<std::uint64_t>(2) << 61;   // SWIZZLE_128B
    return d;
}

// Bounded wait that also gives up as soon as another role aborted.
__device__ __forceinline__ bool wait_or_abort(std::uint64_t* bar, std::uint32_t parity,
                                              volatile std::uint32_t* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - start > kWaitCycles) {
            *abort_flag = 1u;
            atomicOr(&g_device_status, kDevWaitTimeout);
            return false;
        }
    }
    return true;
}

// One Q4_0 block -- scale bits `dbits`, quant words q[0..3] = bytes 0..15 --
// to 32 f16 values (q - 8) * d (exact subtraction, one rounding in the
// product): o[j] holds elements 2j, 2j+1.
__device__ __forceinline__ void convert_block(std::uint32_t dbits, const std::uint32_t (&q)[4],
                                              std::uint32_t (&o)[16]) {
    const std::uint32_t d2 = dbits | (dbits << 16);
    std::uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const std::uint32_t a = prmt(q[i], 0u, 0x4140u);  // bytes 4i, 4i+1
        const std::uint32_t b = prmt(q[i], 0u, 0x4342u);  // bytes 4i+2, 4i+3
        lo[2 * i] = and_or(a, 0x000F000Fu, 0x64006400u);
        lo[2 * i + 1] = and_or(b, 0x000F000Fu, 0x64006400u);
        hi[2 * i] = and_or(a, 0x00F000F0u, 0x54005400u);
        hi[2 * i + 1] = and_or(b, 0x00F000F0u, 0x54005400u);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        std::uint32_t t;
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(t) : "r"(lo[i]), "r"(0x64086408u));
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[i]) : "r"(t), "r"(d2));
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(t) : "r"(hi[i]), "r"(0x54805480u));
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[8 + i]) : "r"(t), "r"(d2));
    }
}

// The 32 converted values of this lane's row into 16 consecutive TMEM
// columns of its lane (the warp's 32 lanes at once).
__device__ __forceinline__ void store_block_tmem(const std::uint32_t (&o)[16], std::uint32_t taddr) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3]), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7]),
        "r"(o[8]), "r"(o[9]), "r"(o[10]), "r"(o[11]), "r"(o[12]), "r"(o[13]), "r"(o[14]),
        "r"(o[15])
        : "memory");
}

// Converts one Q4_0 block (PAR = 0: the even, 1: the odd block) of 64-k
// slice SUB (0..3) of a 144-byte raw row (16-byte aligned at `raw_row`) into
// the 16 TMEM columns at `taddr` (this lane's row).  The slice spans bytes [36*SUB, 36*SUB +
// 36); three aligned 16-byte loads cover it (rows are 144 = 9 x 16 bytes
// apart, so a warp's loads are bank-conflict free) and byte permutes pick
// the block out.
template <int SUB, int PAR>
__device__ __forceinline__ void convert_half_slice(std::uint32_t raw_row, std::uint32_t taddr) {
    constexpr int kStart = 36 * SUB;
    constexpr int kChunk0 = kStart / 16;
    constexpr int kW = (kStart % 16) / 4;  // first word of the slice within the 12 loaded
    std::uint32_t w[12];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int chunk = kChunk0 + c < 9 ? kChunk0 + c : 8;  // never past the row
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                     : "r"(raw_row + chunk * 16));
    }
    std::uint32_t o[16];
    if constexpr (PAR == 0) {
        // even block: scale = low half of word kW, quants start 2 bytes later
        std::uint32_t q0[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q0[i] = prmt(w[kW + i], w[kW + i + 1], 0x5432u);
        convert_block(w[kW] & 0xFFFFu, q0, o);
    } else {
        // odd block: scale = high half of word kW+4, quants are words kW+5..kW+8
        const std::uint32_t q1[4] = {w[kW + 5], w[kW + 6], w[kW + 7], w[kW + 8]};
        convert_block(w[kW + 4] >> 16, q1, o);
    }
    store_block_tmem(o, taddr);
}

// Converts Q8_0 block 2*SUB + PAR of a 272-byte raw row (8 blocks of 34
// bytes: f16 scale, 32 signed bytes) into the 16 TMEM columns at `taddr`:
// q exactly as f16 ((q ^ 0x80) under the exponent of 1024, minus 1152),
// then q * d rounded once.  The block spans at most three 16-byte chunks.
template <int SUB, int PAR>
__device__ __forceinline__ void convert_block_q8(std::uint32_t raw_row, std::uint32_t taddr) {
    constexpr int kOff = 34 * (2 * SUB + PAR);
    constexpr int kChunk0 = kOff / 16;
    constexpr int kO = kOff % 16;  // even: the scale's byte offset in the loaded words
    std::uint32_t w[12];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int chunk = kChunk0 + c < 17 ? kChunk0 + c : 16;  // never past the row
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                     : "r"(raw_row + chunk * 16));
    }
    const std::uint32_t dbits = (kO % 4 == 0) ? (w[kO / 4] & 0xFFFFu) : (w[kO / 4] >> 16);
    const std::uint32_t d2 = dbits | (dbits << 16);
    std::uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        constexpr int kQ = kO + 2;  // first quant byte
        std::uint32_t q;
        if constexpr (kQ % 4 == 0)
            q = w[kQ / 4 + i];
        else
            q = prmt(w[kQ / 4 + i], w[kQ / 4 + i + 1], 0x5432u);
        const std::uint32_t v = q ^ 0x80808080u;  // q + 128 per byte
        std::uint32_t lo, hi;
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(prmt(v, 0x64646464u, 0x4140u)), "r"(0x64806480u));
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(prmt(v, 0x64646464u, 0x4342u)), "r"(0x64806480u));
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[2 * i]) : "r"(lo), "r"(d2));
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[2 * i + 1]) : "r"(hi), "r"(d2));
    }
    store_block_tmem(o, taddr);
}

// Q4_K slice SUB of a 144-byte super-block row (16-byte aligned at
// `raw_row`: f16 d, f16 dmin, 12 bytes of 6-bit scales and mins, 128 quant
// bytes): quant bytes [32 SUB, 32 SUB + 32) hold sub-block 2 SUB in their low
// nibbles (PAR = 0) and 2 SUB + 1 in their high nibbles (PAR = 1).  Each value
// is (d * sc) * q - dmin * m in f32 -- the product is exact, so this is the
// published decode's f32 value -- rounded once to f16, into the 16 TMEM
// columns at `taddr`.
template <int SUB, int PAR>
__device__ __forceinline__ void convert_slice_q4k(std::uint32_t raw_row, std::uint32_t taddr) {
    constexpr int J = 2 * SUB + PAR;  // sub-block
    std::uint32_t h[4], w[8];
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
                 : "r"(raw_row));
#pragma unroll
    for (int c = 0; c < 2; ++c)
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                     : "r"(raw_row + 16 + 32 * SUB + 16 * c));
    // scale byte i of the 12 is byte i % 4 of h[1 + i / 4]
    auto sbyte = [&](int i) { return (h[1 + i / 4] >> (8 * (i % 4))) & 0xFFu; };
    std::uint32_t sc, m;
    if constexpr (J < 4) {
        sc = sbyte(J) & 63u;
        m = sbyte(J + 4) & 63u;
    } else {
        sc = (sbyte(J + 4) & 0x0Fu) | ((sbyte(J - 4) >> 6) << 4);
        m = (sbyte(J + 4) >> 4) | ((sbyte(J) >> 6) << 4);
    }
    const float ds = half_bits_to_float(h[0] & 0xFFFFu) * static_cast<float>(sc);
    const float ndm = -(half_bits_to_float(h[0] >> 16) * static_cast<float>(m));
    std::uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const std::uint32_t a = prmt(w[i], 0u, 0x4140u);  // bytes 4i, 4i+1
        const std::uint32_t b = prmt(w[i], 0u, 0x4342u);  // bytes 4i+2, 4i+3
        std::uint32_t qa, qb;                             // exact f16 pairs of q
        if constexpr (PAR == 0) {
            asm("sub.rn.f16x2 %0, %1, %2;"
                : "=r"(qa)
                : "r"(and_or(a, 0x000F000Fu, 0x64006400u)), "r"(0x64006400u));
            asm("sub.rn.f16x2 %0, %1, %2;"
                : "=r"(qb)
                : "r"(and_or(b, 0x000F000Fu, 0x64006400u)), "r"(0x64006400u));
        } else {
            asm("sub.rn.f16x2 %0, %1, %2;"
                : "=r"(qa)
                : "r"(and_or(a, 0x00F000F0u, 0x54005400u)), "r"(0x54005400u));
            asm("sub.rn.f16x2 %0, %1, %2;"
                : "=r"(qb)
                : "r"(and_or(b, 0x00F000F0u, 0x54005400u)), "r"(0x54005400u));
        }
        const float v0 = fmaf(ds, half_bits_to_float(qa & 0xFFFFu), ndm);
        const float v1 = fmaf(ds, half_bits_to_float(qa >> 16), ndm);
        const float v2 = fmaf(ds, half_bits_to_float(qb & 0xFFFFu), ndm);
        const float v3 = fmaf(ds, half_bits_to_float(qb >> 16), ndm);
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o[2 * i]) : "f"(v1), "f"(v0));
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o[2 * i + 1]) : "f"(v3), "f"(v2));
    }
    store_block_tmem(o, taddr);
}

// Q6_K slice SUB of a 210-byte super-block at `blk` (2-byte aligned: 128
// bytes of low nibbles, 64 of 2-bit high parts, 16 int8 scales, f16 d).
// Elements 64 SUB + 32 PAR + l (l = 0..31) sit in half h = SUB / 2: low
// nibble (SUB % 2) of ql byte 64h + 32 PAR + l, bit pair 2 (SUB % 2) + PAR of
// qh byte 32h + l, scale 4 SUB + 2 PAR + l / 16.  Each value is
// (d * sc) * (q - 32) in f32 as the published decode (d * sc exact, one
// rounding in the product), rounded once to f16 into the 16 TMEM columns at
// `taddr`.  The block is only 2-byte aligned: odd blocks (MIS) take their
// words from aligned neighbours.
__device__ __forceinline__ std::uint32_t lds_word2(std::uint32_t addr) {
    std::uint16_t lo, hi;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(lo) : "r"(addr));
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hi) : "r"(addr + 2));
    return static_cast<std::uint32_t>(lo) | (static_cast<std::uint32_t>(hi) << 16);
}

// 8 consecutive words at `addr`, which is word-aligned, or (MIS) 2 bytes
// past a word: then 9 aligned words are loaded and each output word is a
// PRMT of two neighbours.
template <bool MIS>
__device__ __forceinline__ void lds_words8(std::uint32_t addr, std::uint32_t (&w)[8]) {
    if constexpr (MIS) {
        std::uint32_t a[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) a[i] = lds32(addr - 2 + 4 * i);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = prmt(a[i], a[i + 1], 0x5432u);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = lds32(addr + 4 * i);
    }
}

template <int SUB, int PAR, bool MIS>
__device__ __forceinline__ void convert_slice_q6k(std::uint32_t blk, std::uint32_t taddr) {
    constexpr int h = SUB / 2;
    constexpr int n = SUB % 2;              // nibble of ql
    constexpr int j = 2 * (SUB % 2) + PAR;  // bit pair of qh
    constexpr int kSc = 4 * SUB + 2 * PAR;  // scales of elements 0..15 and 16..31
    std::uint16_t dbits;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(dbits) : "r"(blk + 208));
    const float d = half_bits_to_float(dbits);
    const std::uint32_t scw = lds_word2(blk + 192 + kSc);  // two int8 scales, low half
    const float ds0 = d * static_cast<float>(static_cast<std::int8_t>(scw & 0xFFu));
    const float ds1 = d * static_cast<float>(static_cast<std::int8_t>((scw >> 8) & 0xFFu));
    std::uint32_t Lw[8], Hw[8];
    lds_words8<MIS>(blk + 64 * h + 32 * PAR, Lw);
    lds_words8<MIS>(blk + 128 + 32 * h, Hw);
    std::uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const std::uint32_t L = Lw[i];
        const std::uint32_t H = Hw[i];
        const std::uint32_t q =
            ((L >> (4 * n)) & 0x0F0F0F0Fu) | (((H >> (2 * j)) & 0x03030303u) << 4);
        std::uint32_t qa, qb;  // exact f16 pairs of q - 32
        asm("sub.rn.f16x2 %0, %1, %2;"
            : "=r"(qa)
            : "r"(prmt(q, 0x64646464u, 0x4140u)), "r"(0x64206420u));
        asm("sub.rn.f16x2 %0, %1, %2;"
            : "=r"(qb)
            : "r"(prmt(q, 0x64646464u, 0x4342u)), "r"(0x64206420u));
        const float ds = i < 4 ? ds0 : ds1;  // elements 4i..4i+3
        const float v0 = __fmul_rn(ds, half_bits_to_float(qa & 0xFFFFu));
        const float v1 = __fmul_rn(ds, half_bits_to_float(qa >> 16));
        const float v2 = __fmul_rn(ds, half_bits_to_float(qb & 0xFFFFu));
        const float v3 = __fmul_rn(ds, half_bits_to_float(qb >> 16));
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o[2 * i]) : "f"(v1), "f"(v0));
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o[2 * i + 1]) : "f"(v3), "f"(v2));
    }
    store_block_tmem(o, taddr);
}

template <int TT, bool OF32, int WF, bool PEERS>
__global__ void __launch_bounds__(kThreads, 1)
    q4_0_gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_x,
                             const __grid_constant__ CUtensorMap map_w, const Params p) {
    using L = Layout<TT, WF>;
    constexpr int kOffX = L::kOffX, kOffRaw = L::kOffRaw, kOffBar = L::kOffBar;
    constexpr int kRawRow = kRawRowBytes<WF>;
    constexpr int kRaw = kRawBytes<WF>;
    constexpr int kOffTmemSlot = L::kOffTmemSlot, kOffAbort = L::kOffAbort;
    constexpr int kXBytes = L::kXBytes;
    extern __shared__ std::uint8_t smem_raw[];
    // 1024-byte aligned base (SW128 atoms and TMA swizzle need it)
    const std::uint32_t raw_base = smem_u32(smem_raw);
    const std::uint32_t base = (raw_base + 1023u) & ~1023u;
    std::uint8_t* smem = smem_raw + (base - raw_base);

    std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(smem + kOffBar);
    std::uint64_t* x_full = bars;
    std::uint64_t* w_full = bars + kStages;
    std::uint64_t* empty = bars + 2 * kStages;
    std::uint64_t* raw_full = bars + 3 * kStages;
    constexpr int kRawStages = L::kRawStages;
    std::uint64_t* raw_empty = raw_full + kRawStages;
    std::uint64_t* accum = raw_empty + kRawStages;
    volatile std::uint32_t* tmem_slot = reinterpret_cast<volatile std::uint32_t*>(smem + kOffTmemSlot);
    volatile std::uint32_t* abort_flag = reinterpret_cast<volatile std::uint32_t*>(smem + kOffAbort);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // this CTA's tile and K range (in 64-k slices: [kb0, kb0 + num_kb))
    const bool split = blockIdx.x >= p.full;
    const std::uint32_t j = blockIdx.x - p.full;  // split CTAs only
    const std::uint32_t tile = split ? p.full + j / p.parts : blockIdx.x;
    const std::uint32_t n0 = (tile % p.tiles_n) * kFT;  // first feature (weight row)
    const std::uint32_t m0 = (tile / p.tiles_n) * TT;   // first token
    const std::uint32_t num_kb = split ? p.K / kBK / p.parts : p.K / kBK;
    const std::uint32_t kb0 = split ? (j % p.parts) * num_kb : 0;
    constexpr int kTmemCols = L::kTmemCols;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&x_full[s], 1);
            mbar_init(&w_full[s], 8);  // the 8 warps of the slice's group
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < kRawStages; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], kConvWarps);
        }
        mbar_init(accum, 1);
        *abort_flag = 0u;
        fence_mbarrier_init();
    }
    if (warp == kMmaWarp) tmem_alloc(base + kOffTmemSlot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const std::uint32_t tmem_d = *tmem_slot;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // One thread feeds both rings: each pass issues the next raw
            // stage and the next activation stage whose slots are free
            // (non-blocking tests); no progress for kWaitCycles aborts.
            const std::uint32_t nsb = num_kb / (kSuperK / kBK);
            std::uint32_t kb = 0, sb = 0;
            long long idle_since = clock64();
            while (kb < num_kb || sb < nsb) {
                bool progress = false;
                if (sb < nsb && (sb < kRawStages ||
                                 mbar_test_wait(&raw_empty[sb % kRawStages],
                                                ((sb / kRawStages) - 1) & 1u))) {
                    const int r = sb % kRawStages;
                    mbar_arrive_expect_tx(&raw_full[r], kRaw);
                    // x in the map's elements: bytes (Q4_0, Q4_K) or 2-byte
                    // units (Q8_0; Q6_K from the window's aligned start)
                    const std::uint32_t u = kb0 / (kSuperK / kBK) + sb;
                    const int rx = WF == kWQ6_K  ? static_cast<int>(((u * 210u) & ~15u) / 2)
                                   : WF == kWQ8_0 ? static_cast<int>(u * kRawRow / 2)
                                                  : static_cast<int>(u * kRawRow);
                    tma_load_2d(base + kOffRaw + r * kRaw, &map_w, rx, static_cast<int>(n0),
                                smem_u32(&raw_full[r]));
                    ++sb;
                    progress = true;
                }
                if (kb < num_kb &&
                    (kb < kStages ||
                     mbar_test_wait(&empty[kb % kStages], ((kb / kStages) - 1) & 1u))) {
                    const int s = kb % kStages;
                    mbar_arrive_expect_tx(&x_full[s], kXBytes);
                    tma_load_2d(base + kOffX + s * kXBytes, &map_x,
                                static_cast<int>((kb0 + kb) * kBK), static_cast<int>(m0),
                                smem_u32(&x_full[s]));
                    ++kb;
                    progress = true;
                }
                if (progress) {
                    idle_since = clock64();
                } else {
                    if (*abort_flag) break;
                    if (clock64() - idle_since > kWaitCycles) {
                        *abort_flag = 1u;
                        atomicOr(&g_device_status, kDevWaitTimeout);
                        break;
                    }
                }
            }
        }
        __syncwarp();  // reconverge before the block-wide barrier below
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            for (std::uint32_t kb = 0; kb < num_kb; ++kb) {
                const int s = kb % kStages;
                const std::uint32_t ph = (kb / kStages) & 1u;
                if (!wait_or_abort(&x_full[s], ph, abort_flag)) break;
                if (!wait_or_abort(&w_full[s], ph, abort_flag)) break;
                tc_fence_after();
                const std::uint32_t x_addr = base + kOffX + s * kXBytes;
#pragma unroll
                for (int k = 0; k < kBK / 16; ++k) {
                    // B: +32 bytes per 16-element step inside the 128-byte
                    // swizzle row; A in TMEM: +8 columns (16 f16) per step
                    umma_f16_ta(tmem_d, tmem_d + L::kAColBase + s * 32 + k * 8,
                                smem_desc_sw128(x_addr + k * 32), L::kIdesc,
                                (kb | k) != 0 ? 1u : 0u);
                }
                umma_commit(smem_u32(&empty[s]));
            }
            umma_commit(smem_u32(accum));
        }
        __syncwarp();
    } else {
        // converters: warp w of group g = w / 8 converts the even (w % 8 < 4)
        // or odd block of the group's 64-k slices, weight row 32*(w%4) + lane
        const int row = 32 * (warp % 4) + lane;  // 0..127
        const bool odd = (warp % 8) >= 4;
        const int group = warp / 8;
        const std::uint32_t nsb = num_kb / (kSuperK / kBK);
        bool ok = true;
        for (std::uint32_t sb = 0; sb < nsb && ok; ++sb) {
            const int r = sb % kRawStages;
            ok = __all_sync(0xffffffffu, wait_or_abort(&raw_full[r], (sb / kRawStages) & 1u,
                                                       abort_flag));
            const std::uint32_t raw_row = base + kOffRaw + r * kRaw + row * kRawRow;
            auto slice = [&](auto sub_tag) {
                constexpr int SUB = decltype(sub_tag)::value;
                const std::uint32_t kb = sb * (kSuperK / kBK) + SUB;
                const int s = kb % kStages;
                if (ok && kb >= kStages)
                    ok = __all_sync(0xffffffffu, wait_or_abort(&empty[s], ((kb / kStages) - 1) & 1u,
                                                               abort_flag));
                if (!ok) return;  // warp-uniform
                // this warp's 32 TMEM lanes, the block's 16 columns of stage s
                const std::uint32_t ta = tmem_d + (static_cast<std::uint32_t>(32 * (warp % 4)) << 16) +
                                         static_cast<std::uint32_t>(L::kAColBase + s * 32 +
                                                                    (odd ? 16 : 0));
                if constexpr (WF == kWQ8_0) {
                    if (odd)  // warp-uniform
                        convert_block_q8<SUB, 1>(raw_row, ta);
                    else
                        convert_block_q8<SUB, 0>(raw_row, ta);
                } else if constexpr (WF == kWQ4_K) {
                    if (odd)  // warp-uniform
                        convert_slice_q4k<SUB, 1>(raw_row, ta);
                    else
                        convert_slice_q4k<SUB, 0>(raw_row, ta);
                } else if constexpr (WF == kWQ6_K) {
                    // the super-block's offset in its window
                    const std::uint32_t rem = ((kb0 / (kSuperK / kBK) + sb) * 210u) & 15u;
                    if (rem & 2u) {  // warp-uniform, as `odd`
                        if (odd)
                            convert_slice_q6k<SUB, 1, true>(raw_row + rem, ta);
                        else
                            convert_slice_q6k<SUB, 0, true>(raw_row + rem, ta);
                    } else {
                        if (odd)
                            convert_slice_q6k<SUB, 1, false>(raw_row + rem, ta);
                        else
                            convert_slice_q6k<SUB, 0, false>(raw_row + rem, ta);
                    }
                } else {
                    if (odd)  // warp-uniform
                        convert_half_slice<SUB, 1>(raw_row, ta);
                    else
                        convert_half_slice<SUB, 0>(raw_row, ta);
                }
                // the TMEM stores complete before the MMA warp is told
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                                     smem_u32(&w_full[s]))
                                 : "memory");
                    // the group's last slice of this raw stage
                    if (SUB + kConvGroups >= kSuperK / kBK)
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                                         smem_u32(&raw_empty[r]))
                                     : "memory");
                }
            };
            static_assert(kConvGroups == 2 && kSuperK / kBK == 4, "slice assignment");
            if (group == 0) {  // warp-uniform
                slice(std::integral_constant<int, 0>{});
                slice(std::integral_constant<int, 2>{});
            } else {
                slice(std::integral_constant<int, 1>{});
                slice(std::integral_constant<int, 3>{});
            }
        }
        // epilogue: warp w reads TMEM lanes (features) 32*(w%4).. and a
        // slice of kCols token columns (all converter warps for TT >= 128,
        // group 0 for TT = 64: a TMEM load takes 32 columns); for each token
        // the warp stores 32 consecutive features
        constexpr int kEpiWarps = TT >= 128 ? kConvWarps : 8;
        constexpr int kCols = TT / (kEpiWarps / 4);
        if (warp < kEpiWarps &&
            __all_sync(0xffffffffu, ok && wait_or_abort(accum, 0, abort_flag))) {
            tc_fence_after();
            const int lane_base = 32 * (warp % 4);
            const int col_base = kCols * (warp / 4);
            const std::uint32_t n = n0 + lane_base + lane;
            const bool n_ok = n < p.N;
#pragma unroll 1
            for (int cb = 0; cb < kCols; cb += 32) {
                std::uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_d + (static_cast<std::uint32_t>(lane_base) << 16) +
                                       static_cast<std::uint32_t>(col_base + cb),
                                   v);
                if (split) {
                    // f32 part [token][feature] of split tile j / parts: for
                    // each token the warp stores 32 consecutive features
                    float* part = p.part_buf + static_cast<std::uint64_t>(j) * TT * kFT +
                                  static_cast<std::uint32_t>(col_base + cb) * kFT + lane_base +
                                  lane;
#pragma unroll
                    for (int i = 0; i < 32; ++i) part[i * kFT] = __uint_as_float(v[i]);
                    continue;
                }
                const std::uint32_t mb = m0 + col_base + cb;
                if constexpr (PEERS || !OF32) {
                    // f16 out in 16-byte vectors: the warp's 32 features x 32
                    // tokens are transposed through 2 KB of the (drained)
                    // activation stages, then each lane stores 8 features of a
                    // token per vector -- to this GPU's output, or (PEERS) to
                    // every rank's output at columns col0 + n, over NVLink for
                    // the peers.  Rows come in whole groups of 8 (N % 16 == 0 on
                    // the plain path; shard % 16 == 0 and total % 8 == 0 with
                    // PEERS).
                    __half* tr = reinterpret_cast<__half*>(smem + kOffX) + warp * 32 * 32;
#pragma unroll
                    for (int i = 0; i < 32; ++i) tr[i * 32 + lane] = __float2half_rn(__uint_as_float(v[i]));
                    __syncwarp();
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        const int c = lane + 32 * c4;
                        const int i = c >> 2;          // token within the chunk
                        const int f = (c & 3) * 8;     // first of 8 features
                        const std::uint32_t nf = n0 + lane_base + f;
                        if (mb + i < p.M && nf < p.N) {
                            const uint4 vec = *reinterpret_cast<const uint4*>(tr + i * 32 + f);
                            const std::uint64_t at =
                                static_cast<std::uint64_t>(mb + i) * p.ldy + p.col0 + nf;
                            if constexpr (PEERS) {
                                for (std::uint32_t r = 0; r < p.nranks; ++r)
                                    *reinterpret_cast<uint4*>(p.peer_y[r] + at) = vec;
                            } else {
                                *reinterpret_cast<uint4*>(static_cast<__half*>(p.y) + at) = vec;
                            }
                        }
                    }
                    __syncwarp();
                } else {  // f32 out: for each token the warp stores 32 features
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const std::uint32_t m = mb + i;
                        if (n_ok && m < p.M)
                            static_cast<float*>(p.y)[m * p.ldy + n] = __uint_as_float(v[i]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_d, kTmemCols);
    }
    if constexpr (PEERS) {
        if (threadIdx.x == 0) peer_grid_handshake(p);
    }
}

// The split tiles: y[token][feature] = sum over parts, in part order, of
// part_buf[(tile - full) * parts + part][token - m0][feature - n0].  One
// thread per token and 4 consecutive features (reads and writes coalesced
// along features).
template <int TT, bool OF32>
__global__ void __launch_bounds__(256) q4_0_gemm_reduce_kernel(const Params p,
                                                              std::uint32_t split_tiles) {
    pdl_launch_dependents();
    pdl_wait();
    const std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const std::uint64_t per_tile = static_cast<std::uint64_t>(TT) * (kFT / 4);
    if (i >= per_tile * split_tiles) return;
    const std::uint32_t st = static_cast<std::uint32_t>(i / per_tile);
    const std::uint32_t rem = static_cast<std::uint32_t>(i % per_tile);
    const std::uint32_t tok = rem / (kFT / 4);
    const std::uint32_t f4 = (rem % (kFT / 4)) * 4;
    const std::uint32_t tile = p.full + st;
    const std::uint32_t n = (tile % p.tiles_n) * kFT + f4;
    const std::uint32_t m = (tile / p.tiles_n) * TT + tok;
    if (m >= p.M || n >= p.N) return;  // N % 16 == 0: a 4-feature group is all in or out
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (std::uint32_t q = 0; q < p.parts; ++q) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(
            p.part_buf + (static_cast<std::uint64_t>(st) * p.parts + q) * TT * kFT +
            static_cast<std::uint64_t>(tok) * kFT + f4));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    if constexpr (OF32) {
        *reinterpret_cast<float4*>(static_cast<float*>(p.y) + m * p.ldy + n) = acc;
    } else {
        __half2 h[2] = {__floats2half2_rn(acc.x, acc.y), __floats2half2_rn(acc.z, acc.w)};
        *reinterpret_cast<uint2*>(static_cast<__half*>(p.y) + m * p.ldy + n) =
            *reinterpret_cast<const uint2*>(h);
    }
}

// ---- host side ------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* sym = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(sym);
    });
    return fn;
}

// Whether the tcgen05 path takes this problem: K a multiple of 256 (whole
// 144-byte raw stages; every TMA coordinate 16-byte aligned), N a multiple
// of 16, 16-byte aligned operands.
inline bool supported(const void* x, const void* w, const void* y, std::uint64_t M,
                      std::uint64_t N, std::uint64_t K, std::size_t out_size) {
    return M > 0 && K % kSuperK == 0 && K > 0 && N % 16 == 0 && M <= 0x7fffffffull &&
           N <= 0x7fffffffull && K <= 0x7fffffffull &&
           reinterpret_cast<std::uintptr_t>(x) % 16 == 0 &&
           reinterpret_cast<std::uintptr_t>(w) % 16 == 0 &&
           reinterpret_cast<std::uintptr_t>(y) % 16 == 0 && (N * out_size) % 16 == 0;
}

// Split of the partial last wave: with T tiles on `slots` resident CTAs and
// r = T mod slots tiles left for the last wave (at most half of it), each of
// those r tiles is split along K into `parts` (a power of two dividing K/256
// with r * parts <= slots) so the last wave fills the GPU; the parts meet in
// the workspace.  Returns parts (1: no split) and the bytes it needs.
struct SplitPlan {
    std::uint32_t full = 0, parts = 1, split_tiles = 0;
    std::uint64_t bytes = 0;
};
template <int TT>
inline SplitPlan plan_split(std::uint64_t tiles, std::uint64_t K, std::uint64_t slots) {
    SplitPlan sp;
    sp.full = static_cast<std::uint32_t>(tiles);
    if (slots == 0 || tiles <= slots) return sp;
    const std::uint64_t r = tiles % slots;
    if (r == 0 || 2 * r > slots) return sp;
    std::uint64_t parts = 1;
    while ((K / kSuperK) % (parts * 2) == 0 && r * parts * 2 <= slots) parts *= 2;
    if (parts < 2) return sp;
    sp.full = static_cast<std::uint32_t>(tiles - r);
    sp.parts = static_cast<std::uint32_t>(parts);
    sp.split_tiles = static_cast<std::uint32_t>(r);
    sp.bytes = r * parts * TT * kFT * 4;
    return sp;
}

// Resident CTAs per SM of a kernel (cached per device ordinal).
template <typename Kernel>
int ctas_per_sm(Kernel kernel, int smem, std::atomic<int> (&cache)[64], int dev) {
    const bool cached = dev >= 0 && dev < 64;  // higher ordinals are looked up every call
    int v = cached ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (v == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, kThreads, smem) !=
                cudaSuccess ||
            v <= 0)
            v = 1;
        if (cached) cache[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

// Fused all-gather destinations of a column-sharded linear (PEERS).
struct Peers {
    __half* const* outputs;   // device array of nranks [M, ldy] f16 buffers
    unsigned* const* flags;   // device array of the ranks' flag arrays
    unsigned* own_flags;
    std::uint64_t col0;       // this rank's first column
    std::uint64_t ldy;        // total columns
    std::uint32_t rank, nranks;
};

template <int TT, bool OF32, int WF, bool PEERS = false>
int launch_tile(const void* x, const void* w, void* y, std::uint64_t M, std::uint64_t N,
                std::uint64_t K, cudaStream_t stream, void* workspace,
                std::uint64_t workspace_bytes, const Peers* peers = nullptr) {
    using L = Layout<TT, WF>;
    auto encode = encode_fn();
    if (encode == nullptr) return static_cast<int>(cudaErrorNotSupported);
    CUtensorMap map_x{}, map_w{};
    {
        const cuuint64_t dims[2] = {K, M};
        const cuuint64_t strides[1] = {K * 2};
        const cuuint32_t box[2] = {kBK, TT};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&map_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return static_cast<int>(cudaErrorInvalidValue);
    }
    {
        // Q4_0 and Q4_K rows as bytes (both 144 bytes per 256 k); Q8_0 rows
        // as 2-byte units (a 272-byte box edge is over the 256-element
        // limit); all pitches are multiples of 16
        const std::uint64_t pitch =
            WF == kWQ6_K ? (K / 256) * 210 : (K / 32) * (WF == kWQ8_0 ? 34 : 18);
        const std::uint64_t esize = WF == kWQ8_0 || WF == kWQ6_K ? 2 : 1;
        const cuuint64_t dims[2] = {pitch / esize, N};
        const cuuint64_t strides[1] = {pitch};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRawRowBytes<WF> / esize), kFT};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&map_w, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                   const_cast<void*>(w), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return static_cast<int>(cudaErrorInvalidValue);
    }
    auto kernel = q4_0_gemm_tcgen05_kernel<TT, OF32, WF, PEERS>;
    static std::atomic<std::uint64_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    // the attribute is per device: set once per ordinal below 64, every call above
    const std::uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0;
    if (bit == 0 || !(configured.load() & bit)) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 L::kSmemBytes);
        if (e != cudaSuccess) return static_cast<int>(e);
        configured.fetch_or(bit);
    }
    const std::uint64_t tiles_n = (N + kFT - 1) / kFT;
    const std::uint64_t tiles = tiles_n * ((M + TT - 1) / TT);
    SplitPlan sp;
    sp.full = static_cast<std::uint32_t>(tiles);
    if (!PEERS && workspace != nullptr && reinterpret_cast<std::uintptr_t>(workspace) % 16 == 0) {
        static std::atomic<int> occ[64];
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return static_cast<int>(e);
        const SplitPlan cand = plan_split<TT>(
            tiles, K,
            static_cast<std::uint64_t>(sms) * ctas_per_sm(kernel, L::kSmemBytes, occ, dev));
        if (cand.parts > 1 && cand.bytes <= workspace_bytes) sp = cand;
    }
    Params p{};
    p.y = y;
    p.M = static_cast<std::uint32_t>(M);
    p.N = static_cast<std::uint32_t>(N);
    p.K = static_cast<std::uint32_t>(K);
    p.ldy = N;
    p.tiles_n = static_cast<std::uint32_t>(tiles_n);
    p.full = sp.full;
    p.parts = sp.parts;
    p.part_buf = static_cast<float*>(workspace);
    if constexpr (PEERS) {
        p.peer_y = peers->outputs;
        p.peer_flags = peers->flags;
        p.own_flags = peers->own_flags;
        p.col0 = peers->col0;
        p.ldy = peers->ldy;
        p.rank = peers->rank;
        p.nranks = peers->nranks;
    }
    unsigned grid = sp.full + sp.split_tiles * sp.parts;
    if (PEERS && grid == 0) grid = 1;  // every rank joins the handshake
    kernel<<<grid, kThreads, L::kSmemBytes, stream>>>(map_x, map_w, p);
    e = cudaGetLastError();
    if (e != cudaSuccess || sp.parts == 1) return static_cast<int>(e);
    const std::uint64_t threads = static_cast<std::uint64_t>(sp.split_tiles) * TT * (kFT / 4);
    return launch_pdl(q4_0_gemm_reduce_kernel<TT, OF32>,
                      dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), stream, p,
                      sp.split_tiles);
}

// Workspace bytes the split of a partial last wave can use for this shape
// (0: no split), for the widest token tile of the shape.
inline std::uint64_t split_workspace_bytes(std::uint64_t M, std::uint64_t N, std::uint64_t K) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        sms = 148;
    const std::uint64_t tiles_n = (N + kFT - 1) / kFT;
    // M > 128 runs 256-token tiles, one CTA per SM; narrower tiles at most 2 per SM
    if (M > 128) return plan_split<256>(tiles_n * ((M + 255) / 256), K, sms).bytes;
    const std::uint64_t a = plan_split<128>(tiles_n * ((M + 127) / 128), K, 2ull * sms).bytes;
    const std::uint64_t b = plan_split<128>(tiles_n * ((M + 127) / 128), K, sms).bytes;
    return a > b ? a : b;
}

// Token tile: the narrowest of 64 / 128 / 256 that holds M (wider tiles
// waste MMA columns on missing tokens), 256 beyond.
// A rank whose shard has no real rows still takes part in the handshake.
__global__ void peer_handshake_only_kernel(const Params p) {
    if (threadIdx.x == 0) peer_grid_handshake(p);
}

inline int launch_handshake_only(const Peers& peers, cudaStream_t stream) {
    Params p{};
    p.peer_flags = peers.flags;
    p.own_flags = peers.own_flags;
    p.rank = peers.rank;
    p.nranks = peers.nranks;
    peer_handshake_only_kernel<<<1, 32, 0, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

// The column-sharded Q4_0 linear with the all-gather fused into the
// epilogue (see Peers), for more than 16 tokens: N = this rank's real rows.
inline int launch_peers(const void* x, const void* w, std::uint64_t M, std::uint64_t N,
                        std::uint64_t K, const Peers& peers, cudaStream_t stream) {
    if (M <= 64)
        return launch_tile<64, false, kWQ4_0, true>(x, w, nullptr, M, N, K, stream, nullptr, 0,
                                                   &peers);
    if (M <= 128)
        return launch_tile<128, false, kWQ4_0, true>(x, w, nullptr, M, N, K, stream, nullptr, 0,
                                                    &peers);
    return launch_tile<256, false, kWQ4_0, true>(x, w, nullptr, M, N, K, stream, nullptr, 0,
                                                &peers);
}

// WF selects the weight format: kWQ4_0, kWQ8_0, kWQ4_K or kWQ6_K (which
// also needs K % 2048 == 0).
template <bool OF32, int WF = kWQ4_0>
int launch(const void* x, const void* w, void* y, std::uint64_t M, std::uint64_t N,
           std::uint64_t K, cudaStream_t stream, void* workspace = nullptr,
           std::uint64_t workspace_bytes = 0) {
    if (M <= 64)
        return launch_tile<64, OF32, WF>(x, w, y, M, N, K, stream, workspace, workspace_bytes);
    if (M <= 128)
        return launch_tile<128, OF32, WF>(x, w, y, M, N, K, stream, workspace, workspace_bytes);
    return launch_tile<256, OF32, WF>(x, w, y, M, N, K, stream, workspace, workspace_bytes);
}

}  // namespace gemm
}  // namespace mote
