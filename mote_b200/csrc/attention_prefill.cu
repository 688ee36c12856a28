// Causal grouped-query attention for prefill chunks on the tcgen05 tensor
// cores (no reference counterpart; see attention.cu).
//
//   out[t, h] = softmax_{p <= start + t}(scale * q[t, h] . K[p, h / g]) . V[p, h / g]
//
// q/out [tokens, q_heads, 64] f16 (queries at positions start .. start +
// tokens - 1); K/V from the cache rows row0 .. row0 + start + tokens - 1
// ([cache rows, kv_heads, 64] f16, this chunk's K/V already appended).
//
// Persistent: one CTA per SM walks work items (128 query rows of one query
// head; longest first) with tensor memory allocated once, so the next
// item's Q and first K/V tiles load while the current item finishes
// (flash attention per item):
// * warp 8 loads each item's Q tile (two buffers) and the K and V tiles
//   of 128 positions (TMA, 128-byte swizzle, four stages shared by all
//   items; tensor maps end at the last attended row, so rows past it
//   arrive as zeros);
// * warp 9 allocates tensor memory and one thread issues the MMAs:
//   S = Q K^T (tcgen05.mma kind::f16, M = 128 queries, N = 128 positions,
//   A and B K-major in shared memory) into one of two S buffers in TMEM, so
//   S for the next tile is computed while the softmax works on this one;
//   then O += P V (M = 128, N = 64, A = P read from tensor memory, B = V
//   MN-major in shared memory) into the O accumulator in TMEM;
// * warps 0-7 run the softmax in two groups of four: group g takes the
//   tiles j with j % 2 == g (S buffer g) and keeps, per query row (= TMEM
//   lane, one thread), its own reference maximum, sum and O accumulator
//   O_g, so the groups never wait for each other and one group's softmax
//   overlaps the other's hand-offs.  A thread reads its S row (tcgen05.ld),
//   masks positions past its row's, keeps the maximum and sum (exp2 with
//   the scale folded in), writes P as f16 over the first half of the S
//   buffer (tcgen05.st), rescales O_g only when the maximum grew by more
//   than 8 (log2 units; probabilities stay below 2^8), then releases the
//   P.V MMA into O_g.  At the end the groups exchange maxima and sums and
//   each thread writes half of its row: (O_0 w_0 + O_1 w_1) / sum.
// Every wait is bounded; an expired wait aborts the CTA, which waits for its
// issued MMAs (bounded) and frees its tensor memory.  No load uses cluster
// multicast.
#include "mote_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace mote {
namespace attnp {

constexpr int kBM = 128;      // query rows per CTA (TMEM lanes)
constexpr int kBN = 128;      // positions per K/V tile
constexpr int kD = 64;        // head_dim (one 128-byte swizzle row)
constexpr int kKV = 4;        // K/V tile stages (TMA ring)
constexpr int kSBuf = 2;      // S buffers in tensor memory
// Softmax: two groups of four warps (tiles of even and odd index).
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
// Warps 10 and 11 only complete the third warpgroup (register split below).
constexpr int kThreads = 12 * 32;
// Register split (setmaxnreg, per warpgroup): launched at 168 per thread
// (12 warps: 3 per SM sub-partition); the producer/MMA warpgroup gives up to
// 40 and the two softmax warpgroups take 232:  384 x 168 = 64512 =
// 256 x 232 + 128 x 40, and per sub-partition 32 x (232 + 232 + 40) <= 16384.
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 232;
constexpr int kOtherRegs = 40;
static_assert(kThreads * kLaunchRegs == 256 * kSoftmaxRegs + 128 * kOtherRegs, "register split");
static_assert(32 * (2 * kSoftmaxRegs + kOtherRegs) <= 16384, "registers of a sub-partition");
constexpr int kTileBytes = kBN * kD * 2;  // 16 KB (also the Q tile)

// TMEM columns: S0 [0, 128), S1 [128, 256), O_0 [256, 320), O_1 [320, 384);
// P_j (f16, two per column) over the first 64 columns of S_{j % 2}.
constexpr std::uint32_t kColO = 256;  // O_g at kColO + 64 g (g = tile parity)
constexpr std::uint32_t kTmemCols = 512;

struct Smem {
    static constexpr int kQ = 0;                              // [2] Q tiles (items alternate)
    static constexpr int kK = kQ + 2 * kTileBytes;            // [kKV] tiles
    static constexpr int kV = kK + kKV * kTileBytes;          // [kKV] tiles
    static constexpr int kBar = kV + kKV * kTileBytes;
    // q_full[2], q_empty[2], k_full[kKV], v_full[kKV], kv_empty[kKV], s_full[2],
    // p_ready[2], o_done[2], epi_done, drained
    static constexpr int kNumBars = 4 + 3 * kKV + 3 * kSBuf + 2;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kAbort = kTmemSlot + 4;
    // the softmax groups' row maxima and sums, by item parity: [2][2][kBM] f32 each
    static constexpr int kXchg = (kAbort + 4 + 15) / 16 * 16;
    static constexpr int kSums = kXchg + 2 * 2 * kBM * 4;
    static constexpr int kUsed = kSums + 2 * 2 * kBM * 4 + 1024;  // + 1024-byte alignment slack
    // at least 120 KB: one CTA per SM, so a CTA's 512 TMEM columns never
    // wait for another CTA of this kernel on the same SM
    static constexpr int kBytes = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
};

// Instruction descriptors, kind::f16, f32 accumulate, f16 operands:
// S: M = 128, N = 128, A and B K-major; PV: M = 128, N = 64, B MN-major.
constexpr std::uint32_t kIdescS = (1u << 4) | ((kBN >> 3) << 17) | ((kBM >> 4) << 24);
constexpr std::uint32_t kIdescPV = (1u << 4) | (1u << 16) | ((kD >> 3) << 17) | ((kBM >> 4) << 24);

struct Params {
    __half* out;
    std::uint32_t tokens, start;
    std::uint32_t q_heads, kv_heads;
    std::uint64_t out_row_stride;  // elements between tokens (q_heads * 64)
    float scale_log2;
    std::uint32_t q_tiles;
};

__device__ __forceinline__ void tma_load_3d(std::uint32_t dst, const CUtensorMap* map, int x,
                                            int y, int z, std::uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16, cta_group::1.
__device__ __forceinline__ void umma_f16_ss(std::uint32_t tmem_d, std::uint64_t adesc,
                                            std::uint64_t bdesc, std::uint32_t idesc,
                                            std::uint32_t accumulate) {
    const std::uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask), "r"(mask), "r"(mask),
        "r"(mask)
        : "memory");
}

// 32 lanes x 32 consecutive columns, no wait (the caller waits once).
__device__ __forceinline__ void tmem_ld32_nowait(std::uint32_t taddr, std::uint32_t (&r)[32]) {
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
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(std::uint32_t taddr, const std::uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float2 half2_bits_to_float2_f(std::uint32_t v) {
    __half2 h;
    memcpy(&h, &v, sizeof(h));
    return __half22float2(h);
}

// Packed f32 pairs (Blackwell f32x2 arithmetic) and the three-input maximum.
__device__ __forceinline__ std::uint64_t pack_f32x2(float lo, float hi) {
    std::uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack_f32x2(std::uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ std::uint64_t fma_f32x2(std::uint64_t a, std::uint64_t b, std::uint64_t c) {
    std::uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ std::uint64_t add_f32x2(std::uint64_t a, std::uint64_t b) {
    std::uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float m;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
    return m;
}

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    gqa_prefill_kernel(const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const Params p) {
    using gemm::smem_desc_sw128;
    using gemm::wait_or_abort;
    extern __shared__ std::uint8_t smem_raw[];
    const std::uint32_t raw_base = smem_u32(smem_raw);
    const std::uint32_t base = (raw_base + 1023u) & ~1023u;
    std::uint8_t* smem = smem_raw + (base - raw_base);
    std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(smem + Smem::kBar);
    std::uint64_t* q_full = bars;
    std::uint64_t* q_empty = bars + 2;
    std::uint64_t* k_full = bars + 4;
    std::uint64_t* v_full = k_full + kKV;
    std::uint64_t* kv_empty = v_full + kKV;
    std::uint64_t* s_full = kv_empty + kKV;
    std::uint64_t* p_ready = s_full + kSBuf;
    std::uint64_t* o_done = p_ready + kSBuf;
    std::uint64_t* epi_done = o_done + kSBuf;
    std::uint64_t* drained = epi_done + 1;
    volatile std::uint32_t* tmem_slot = reinterpret_cast<volatile std::uint32_t*>(smem + Smem::kTmemSlot);
    volatile std::uint32_t* abort_flag = reinterpret_cast<volatile std::uint32_t*>(smem + Smem::kAbort);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Work items (query tile, query head), longest first (causal: later
    // query tiles attend more positions): item i is query tile
    // q_tiles - 1 - i / q_heads of head i % q_heads; CTA b takes items
    // b, b + gridDim.x, ...
    const std::uint32_t items = p.q_tiles * p.q_heads;
    struct Item {
        std::uint32_t h, kvh, q0, nkt;
    };
    auto item_at = [&](std::uint32_t i) {
        Item it;
        const std::uint32_t qt = p.q_tiles - 1 - i / p.q_heads;
        it.h = i % p.q_heads;
        it.kvh = it.h / (p.q_heads / p.kv_heads);
        it.q0 = qt * kBM;
        const std::uint32_t q_end = min(it.q0 + kBM, p.tokens);  // exclusive
        it.nkt = (p.start + q_end + kBN - 1) / kBN;              // tiles of attended positions
        return it;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&q_full[s], 1);
            mbar_init(&q_empty[s], 1);
        }
        for (int s = 0; s < kKV; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int s = 0; s < kSBuf; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&p_ready[s], kSoftmaxWarps / 2);  // the tile parity's group
            mbar_init(&o_done[s], 1);
        }
        mbar_init(epi_done, kSoftmaxWarps);
        mbar_init(drained, 1);
        *abort_flag = 0u;
        fence_mbarrier_init();
    }
    if (warp == kMmaWarp) gemm::tmem_alloc(base + Smem::kTmemSlot, kTmemCols);
    gemm::tc_fence_before();
    __syncthreads();
    gemm::tc_fence_after();
    const std::uint32_t tmem = *tmem_slot;
    // the tensor-map descriptors are kernel parameters (not written by the
    // previous kernel): fetch them while it may still be running
    if (warp == kProducerWarp && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<std::uint64_t>(&map_q))
                     : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<std::uint64_t>(&map_k))
                     : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<std::uint64_t>(&map_v))
                     : "memory");
    }
    pdl_wait();

    if (warp >= kSoftmaxWarps) {
      // the third warpgroup (producer, MMA issuer, two idle warps) gives up
      // registers for the softmax warpgroups
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kOtherRegs));
      if (warp == kProducerWarp) {
        if (lane == 0) {
            // runs ahead across items: the next item's Q and first K/V tiles
            // load while the current item is still in its last tiles
            std::uint32_t kt = 0;  // K/V tiles loaded by this CTA
            bool ok = true;
            std::uint32_t n = 0;
            for (std::uint32_t i = blockIdx.x; ok && i < items; i += gridDim.x, ++n) {
                const Item it = item_at(i);
                const int qb = n & 1;
                if (n >= 2 && !wait_or_abort(&q_empty[qb], ((n / 2) - 1) & 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&q_full[qb], kTileBytes);
                tma_load_3d(base + Smem::kQ + qb * kTileBytes, &map_q, 0, static_cast<int>(it.h),
                            static_cast<int>(it.q0), smem_u32(&q_full[qb]));
                for (std::uint32_t j = 0; j < it.nkt; ++j, ++kt) {
                    const int s = kt % kKV;
                    if (kt >= kKV &&
                        !wait_or_abort(&kv_empty[s], ((kt / kKV) - 1) & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&k_full[s], kTileBytes);
                    tma_load_3d(base + Smem::kK + s * kTileBytes, &map_k, 0, static_cast<int>(it.kvh),
                                static_cast<int>(j * kBN), smem_u32(&k_full[s]));
                    mbar_arrive_expect_tx(&v_full[s], kTileBytes);
                    tma_load_3d(base + Smem::kV + s * kTileBytes, &map_v, 0, static_cast<int>(it.kvh),
                                static_cast<int>(j * kBN), smem_u32(&v_full[s]));
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            std::uint32_t kt = 0;                // K/V tiles consumed
            std::uint32_t cnt0 = 0, cnt1 = 0;   // P.V into O_0 / O_1 so far (all items)
            bool ok = true;
            std::uint32_t n = 0;
            for (std::uint32_t i = blockIdx.x; ok && i < items; i += gridDim.x, ++n) {
                const Item it = item_at(i);
                const int qb = n & 1;
                const std::uint32_t qaddr = base + Smem::kQ + qb * kTileBytes;
                const std::uint32_t kt0 = kt;
                auto issue_s = [&](std::uint32_t j) -> bool {
                    const std::uint32_t t = kt0 + j;
                    const int kv = t % kKV, sb = j % kSBuf;
                    if (!wait_or_abort(&k_full[kv], (t / kKV) & 1u, abort_flag)) return false;
                    gemm::tc_fence_after();
                    const std::uint32_t kaddr = base + Smem::kK + kv * kTileBytes;
#pragma unroll
                    for (int k = 0; k < kD / 16; ++k)
                        umma_f16_ss(tmem + sb * kBN, smem_desc_sw128(qaddr + k * 32),
                                    smem_desc_sw128(kaddr + k * 32), kIdescS, k != 0 ? 1u : 0u);
                    gemm::umma_commit(smem_u32(&s_full[sb]));
                    // the item's last S: its Q buffer is free once it completes
                    if (j + 1 == it.nkt) gemm::umma_commit(smem_u32(&q_empty[qb]));
                    return true;
                };
                ok = wait_or_abort(&q_full[qb], (n / 2) & 1u, abort_flag) && issue_s(0);
                // the previous item's epilogue has read O_0 and O_1 before the
                // first P.V of this item overwrites them
                if (ok && n > 0) ok = wait_or_abort(epi_done, (n - 1) & 1u, abort_flag);
                for (std::uint32_t j = 0; ok && j < it.nkt; ++j) {
                    const std::uint32_t t = kt0 + j;
                    const int kv = t % kKV, sb = j % kSBuf;
                    if (j + 1 < it.nkt && !issue_s(j + 1)) {
                        ok = false;
                        break;
                    }
                    if (!wait_or_abort(&p_ready[sb], (sb ? cnt1 : cnt0) & 1u, abort_flag) ||
                        !wait_or_abort(&v_full[kv], (t / kKV) & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    gemm::tc_fence_after();
                    const std::uint32_t vaddr = base + Smem::kV + kv * kTileBytes;
#pragma unroll
                    for (int k = 0; k < kBN / 16; ++k)
                        // A = P (16 positions = 8 columns per step), B = V rows
                        // of 16 positions (2048 bytes per step, MN-major)
                        gemm::umma_f16_ta(tmem + kColO + 64u * static_cast<std::uint32_t>(sb),
                                          tmem + sb * kBN + k * 8,
                                          smem_desc_sw128(vaddr + k * 2048), kIdescPV,
                                          (j >= static_cast<std::uint32_t>(kSBuf) || k != 0) ? 1u : 0u);
                    gemm::umma_commit(smem_u32(&o_done[sb]));
                    gemm::umma_commit(smem_u32(&kv_empty[kv]));
                    if (sb) ++cnt1; else ++cnt0;
                }
                kt = kt0 + it.nkt;
            }
            // every issued MMA completes before the tensor memory is freed
            gemm::umma_commit(smem_u32(drained));
            mbar_wait_bounded(drained, 0, &g_device_status);
        }
        __syncwarp();
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
        // softmax: group g = warp / 4 takes the tiles j with j % 2 == g, one
        // thread per query row r = TMEM lane, with its own reference maximum,
        // sum and O accumulator O_g; the groups meet once per item.  Every
        // softmax thread walks every item of the CTA (a failed wait only
        // skips work), so all reach each item's named barrier.
        const int quarter = warp % 4, grp = warp / 4;
        const int r = 32 * quarter + lane;
        const std::uint32_t lane_off = static_cast<std::uint32_t>(32 * quarter) << 16;
        const std::uint32_t o_col = kColO + 64u * static_cast<std::uint32_t>(grp);
        const float sc = p.scale_log2;
        std::uint32_t cnt0 = 0, cnt1 = 0;  // tiles of each parity group (all items)
        bool ok = true;
        std::uint32_t n = 0;
        for (std::uint32_t i = blockIdx.x; i < items; i += gridDim.x, ++n) {
            const Item it = item_at(i);
            const std::int64_t qpos = static_cast<std::int64_t>(p.start) + it.q0 + r;
            const std::uint32_t n0 = (it.nkt + 1) / 2, n1 = it.nkt / 2;  // tiles per group
            float m = -INFINITY, l = 0.f;
            std::uint32_t jj = 0;  // this group's tiles of the item
            for (std::uint32_t j = static_cast<std::uint32_t>(grp); j < it.nkt && ok; j += kSBuf, ++jj) {
                const std::uint32_t c = (grp ? cnt1 : cnt0) + jj;  // this group's tile, all items
                ok = __all_sync(0xffffffffu, wait_or_abort(&s_full[grp], c & 1u, abort_flag));
                if (!ok) break;
                gemm::tc_fence_after();
                std::uint32_t v[4][32];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) tmem_ld32_nowait(tmem + lane_off + grp * kBN + 32 * cc, v[cc]);
                tmem_wait_ld();
                // causal mask (position j*128 + col past the row's) as -inf;
                // the scale is positive, so the maximum of the raw scores
                // gives the maximum of the scaled ones
                const std::int64_t kbase = static_cast<std::int64_t>(j) * kBN;
                if (kbase + kBN - 1 > static_cast<std::int64_t>(p.start) + it.q0) {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (kbase + 32 * cc + e > qpos) v[cc][e] = __float_as_uint(-INFINITY);
                }
                float mx8[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                    for (int e = 0; e < 32; e += 2)
                        mx8[(e / 2) % 8] = max3f(mx8[(e / 2) % 8], __uint_as_float(v[cc][e]),
                                                 __uint_as_float(v[cc][e + 1]));
                const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
                // The reference maximum m (raw units) moves, and O_g and the
                // sum are rescaled, only when the row maximum exceeds it by
                // more than 8 in log2 units: a probability stays below 2^8
                // (exact in f16 as any other) and most tiles skip the rescale
                // and its wait for the previous P.V.  A row can have no
                // attended position in a tile of group 1 (its first tile
                // starts at position 128): while m is -inf its probabilities
                // are exact zeros and nothing moves.
                const float mnew = fmaxf(m, mx);
                const bool grow = (mnew - m) * sc > 8.f;  // false while both are -inf (NaN)
                float alpha = 1.f;
                if (grow) {
                    alpha = ex2f((m - mnew) * sc);  // 0 when m was -inf
                    m = mnew;
                }
                const float neg_m = m == -INFINITY ? 0.f : -m * sc;
                // pairs of probabilities with packed f32x2 arithmetic: one
                // FMA for both exponents, one add for both sums
                const std::uint64_t sc2 = pack_f32x2(sc, sc), nm2 = pack_f32x2(neg_m, neg_m);
                std::uint64_t acc2[4] = {0, 0, 0, 0};  // (+0, +0) per pair of lanes
                std::uint32_t pk[2][32];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        float xa, xb;
                        unpack_f32x2(fma_f32x2(pack_f32x2(__uint_as_float(v[cc][e]),
                                                          __uint_as_float(v[cc][e + 1])),
                                               sc2, nm2),
                                     xa, xb);
                        const float a = ex2f(xa);
                        const float b = ex2f(xb);
                        acc2[(e / 2) % 4] = add_f32x2(acc2[(e / 2) % 4], pack_f32x2(a, b));
                        std::uint32_t h2;
                        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h2) : "f"(b), "f"(a));
                        pk[cc / 2][(cc % 2) * 16 + e / 2] = h2;
                    }
                float sum = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float x0, x1;
                    unpack_f32x2(acc2[i], x0, x1);
                    sum += x0 + x1;
                }
                l = fmaf(l, alpha, sum);
                // P over the first 64 columns of this group's S buffer
                tmem_st32(tmem + lane_off + grp * kBN, pk[0]);
                tmem_st32(tmem + lane_off + grp * kBN + 32, pk[1]);
                tmem_wait_st();
                if (jj > 0 && __any_sync(0xffffffffu, grow)) {
                    // the group's previous P.V must be complete before O_g moves
                    ok = __all_sync(0xffffffffu, wait_or_abort(&o_done[grp], (c - 1) & 1u, abort_flag));
                    if (!ok) break;
                    gemm::tc_fence_after();
                    std::uint32_t o[2][32];
                    tmem_ld32_nowait(tmem + lane_off + o_col, o[0]);
                    tmem_ld32_nowait(tmem + lane_off + o_col + 32, o[1]);
                    tmem_wait_ld();
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc)
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[cc][e] = __float_as_uint(__uint_as_float(o[cc][e]) * alpha);
                    tmem_st32(tmem + lane_off + o_col, o[0]);
                    tmem_st32(tmem + lane_off + o_col + 32, o[1]);
                    tmem_wait_st();
                }
                gemm::tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&p_ready[grp]))
                                 : "memory");
            }
            cnt0 += n0;
            cnt1 += n1;
            // The groups' states meet (by item parity in shared memory), then
            // the thread of group g writes dimensions [32 g, 32 g + 32) of its
            // row from O_0 and O_1 and releases them for the next item.
            float* xm = reinterpret_cast<float*>(smem + Smem::kXchg) + (n & 1u) * 2 * kBM;
            float* xl = reinterpret_cast<float*>(smem + Smem::kSums) + (n & 1u) * 2 * kBM;
            xm[grp * kBM + r] = m;
            xl[grp * kBM + r] = l;
            named_bar_sync(1, kSoftmaxWarps * 32);
            const float m0 = xm[r], m1 = xm[kBM + r];
            const float mt = fmaxf(m0, m1);
            const float w0 = m0 == -INFINITY ? 0.f : ex2f((m0 - mt) * sc);
            const float w1 = (n1 == 0 || m1 == -INFINITY) ? 0.f : ex2f((m1 - mt) * sc);
            const float lrow = xl[r] * w0 + (n1 > 0 ? xl[kBM + r] * w1 : 0.f);
            if (ok)
                ok = __all_sync(0xffffffffu, wait_or_abort(&o_done[0], (cnt0 - 1) & 1u, abort_flag));
            if (ok && n1 > 0)
                ok = __all_sync(0xffffffffu, wait_or_abort(&o_done[1], (cnt1 - 1) & 1u, abort_flag));
            if (ok) {
                gemm::tc_fence_after();
                const std::uint32_t dcol = 32u * static_cast<std::uint32_t>(grp);
                std::uint32_t a[32], b[32];
                tmem_ld32_nowait(tmem + lane_off + kColO + dcol, a);
                if (n1 > 0) tmem_ld32_nowait(tmem + lane_off + kColO + 64 + dcol, b);
                tmem_wait_ld();
                gemm::tc_fence_before();
                __syncwarp();
                if (lane == 0)  // O_0 and O_1 are read: the next item may overwrite them
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(epi_done))
                                 : "memory");
                if (it.q0 + r < p.tokens) {
                    const float inv = lrow > 0.f ? 1.f / lrow : 0.f;
                    uint4* dst = reinterpret_cast<uint4*>(p.out + (static_cast<std::uint64_t>(it.q0) + r) *
                                                                       p.out_row_stride +
                                                          static_cast<std::uint64_t>(it.h) * kD + dcol);
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        std::uint32_t wv[4];
#pragma unroll
                        for (int e2 = 0; e2 < 4; ++e2) {
                            const int k0 = e + 2 * e2;
                            float x0 = __uint_as_float(a[k0]) * w0, x1 = __uint_as_float(a[k0 + 1]) * w0;
                            if (n1 > 0) {
                                x0 = fmaf(__uint_as_float(b[k0]), w1, x0);
                                x1 = fmaf(__uint_as_float(b[k0 + 1]), w1, x1);
                            }
                            asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(wv[e2]) : "f"(x1 * inv), "f"(x0 * inv));
                        }
                        dst[e / 8] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                    }
                }
            }
        }
    }
    gemm::tc_fence_before();
    __syncthreads();
    gemm::tc_fence_after();
    if (warp == kMmaWarp) gemm::tmem_dealloc(tmem, kTmemCols);
    pdl_launch_dependents();
}

// 3-D tensor map over [rows, heads, 64] f16 (64 elements innermost), boxes
// of 128 rows x 1 head x 64, 128-byte swizzle; rows past `rows` read zero.
inline int make_map(CUtensorMap* map, const void* ptr, std::uint64_t rows, std::uint64_t heads) {
    auto encode = gemm::encode_fn();
    if (encode == nullptr) return static_cast<int>(cudaErrorNotSupported);
    const cuuint64_t dims[3] = {kD, heads, rows};
    const cuuint64_t strides[2] = {kD * 2, heads * kD * 2};
    const cuuint32_t box[3] = {kD, 1, kBN};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return static_cast<int>(cudaErrorInvalidValue);
    return kSuccess;
}

}  // namespace attnp
}  // namespace mote

// Causal prefill attention of `tokens` queries at positions start .. start +
// tokens - 1 over cache rows row0 .. row0 + start + tokens - 1 (see the
// header for the layout).  head_dim 64; q_heads % kv_heads == 0; scale > 0;
// 16-byte aligned tensors; tokens == 0 returns 0.
extern "C" int mote_cuda_gqa_attention_prefill_f16(const void* q, const void* k_cache,
                                                   const void* v_cache, void* out,
                                                   uint64_t tokens, uint64_t start,
                                                   uint64_t q_heads, uint64_t kv_heads,
                                                   uint64_t head_dim, uint64_t row0,
                                                   uint64_t cache_rows, float scale,
                                                   void* stream) {
    using namespace mote;
    using namespace mote::attnp;
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr ||
        stream == nullptr)
        return kInvalidValue;
    if (tokens == 0 || q_heads == 0) return kSuccess;
    if (head_dim != kD || kv_heads == 0 || q_heads % kv_heads != 0 || q_heads > 65535 ||
        !std::isfinite(scale) || !(scale > 0.f))
        return kInvalidValue;
    if (tokens > 0x7fffffffull || start > 0x7fffffffull || row0 + start + tokens > cache_rows ||
        start + tokens > 0x7fffffffull)
        return kInvalidValue;
    for (const void* ptr : {q, k_cache, v_cache, static_cast<const void*>(out)})
        if (reinterpret_cast<std::uintptr_t>(ptr) % 16 != 0) return kInvalidValue;
    CUtensorMap map_q{}, map_k{}, map_v{};
    int st = make_map(&map_q, q, tokens, q_heads);
    // K/V maps start at the sequence's first row and end at its last
    // attended row: positions past it read zeros
    const std::uint64_t off = row0 * kv_heads * kD;
    if (st == kSuccess)
        st = make_map(&map_k, static_cast<const __half*>(k_cache) + off, start + tokens, kv_heads);
    if (st == kSuccess)
        st = make_map(&map_v, static_cast<const __half*>(v_cache) + off, start + tokens, kv_heads);
    if (st != kSuccess) return st;
    Params p{};
    p.out = static_cast<__half*>(out);
    p.tokens = static_cast<std::uint32_t>(tokens);
    p.start = static_cast<std::uint32_t>(start);
    p.q_heads = static_cast<std::uint32_t>(q_heads);
    p.kv_heads = static_cast<std::uint32_t>(kv_heads);
    p.out_row_stride = q_heads * kD;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.q_tiles = static_cast<std::uint32_t>((tokens + kBM - 1) / kBM);
    static std::atomic<std::uint64_t> done{0};
    st = ensure_dynamic_smem(gqa_prefill_kernel, Smem::kBytes, done);
    if (st != kSuccess) return st;
    // The register split is exact for a launch at kLaunchRegs per thread; a
    // build that allocated another count could leave setmaxnreg.inc waiting
    // for registers that do not exist, so it is never launched.
    static std::atomic<int> regs_checked{0};
    if (regs_checked.load(std::memory_order_acquire) == 0) {
        cudaFuncAttributes fa{};
        const cudaError_t ea = cudaFuncGetAttributes(&fa, gqa_prefill_kernel);
        if (ea != cudaSuccess) return static_cast<int>(ea);
        if (fa.numRegs != kLaunchRegs) return static_cast<int>(cudaErrorInvalidConfiguration);
        regs_checked.store(1, std::memory_order_release);
    }
    // persistent: one CTA per SM (at most one per item)
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    const std::uint64_t items = static_cast<std::uint64_t>(p.q_tiles) * q_heads;
    const unsigned grid = static_cast<unsigned>(items < static_cast<std::uint64_t>(sms) ? items : sms);
    return launch_pdl_smem(gqa_prefill_kernel, dim3(grid), dim3(kThreads), Smem::kBytes,
                           static_cast<cudaStream_t>(stream), map_q, map_k, map_v, p);
}
