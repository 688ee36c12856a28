// Grouped-query attention over a KV cache, and the cache append.
//
// No reference counterpart: the reference names "attention (GQA) with KV
// cache" and "KV-cache operations" as planned primitives
// (docs/roadmap.md:58-60, docs/architecture.md:185-191) and ships none.
// The math is standard scaled dot-product attention: query head h reads
// KV head h / (q_heads / kv_heads); scores = scale * q.k; softmax over the
// attended positions; output = softmax . V.
//
// Layouts (f16, row-major, head_dim innermost):
//   cache   [cache_rows, kv_heads, head_dim]   (K and V alike)
//           a batch of sequences uses rows b * seq_capacity + position
//   q       [batch, q_heads, head_dim]           (decode: one token each)
//   out     [batch, q_heads, head_dim]
//
// * kv_cache_append: copies new K/V rows into the cache at caller-given
//   rows (one slot per token), 16-byte vectors; a slot outside the cache
//   sets an error flag and is skipped (as the embedding gather does).
// * Decode (one query token per sequence) is HBM-bound: every cached K and
//   V byte of the sequence is read once.  Flash-decoding on the tensor
//   cores: a CTA takes one (sequence, KV head, group of up to 16 query
//   heads, chunk of positions); its query heads are the 16 rows of
//   mma.sync.m16n8k16 (f16 in, f32 accumulate).  Each of its eight warps
//   streams tiles of 2048 / head_dim positions through a private
//   three-stage cp.async ring (K and V rows swizzled for conflict-free
//   ldmatrix) and computes S = Q K^T, an online softmax on the S
//   accumulators (exp2 with the scale folded in), and O += P V with the S
//   accumulators reused as the A operand.  P is split into f16 hi + lo
//   parts (two MMAs), so the probabilities keep ~22 bits.  The warps'
//   states meet in shared memory; the CTA writes its output, or the chunks
//   of a sequence merge inside a thread-block cluster (up to 8), or write
//   unnormalised partials with their max and sum for a merge kernel.
#include "mote_common.cuh"

namespace mote {
namespace attn {

// Decode split kernel: eight warps, each with a three-stage ring of 8 KB
// tiles (K and V of 2048 / head_dim positions), 192 KB per CTA.  Four warps
// with 16 KB tiles measured 7-10 % slower (one warp per scheduler left the
// MMA and ldmatrix latencies exposed).
constexpr int kWarpsPerCta = 8;
constexpr int kThreads = 32 * kWarpsPerCta;
constexpr int kStageBytes = 8192;    // K and V of one tile
constexpr int kStagesPerWarp = 3;
constexpr int kHeadsPerCta = 16;     // query heads per CTA (the MMA rows)
constexpr int kSplitSmem = kWarpsPerCta * kStagesPerWarp * kStageBytes;
// Cluster path: a CTA's merged state (O [16][D] f32, max [16], sum [16]) at
// 12 KB into warp 0's ring, after that warp's own state (at most 8.2 KB).
constexpr int kClusterStateOffset = 12 * 1024;
static_assert(kClusterStateOffset + (16 * 128 + 32) * 4 <= kStagesPerWarp * kStageBytes,
              "the cluster state fits in warp 0's ring");
// At most 8 chunks to a cluster (the portable size): 16-CTA clusters of
// full-SM CTAs measured slower (fewer of them fit on the GPCs at a time).
constexpr int kMaxClusterChunks = 8;

// ---------------------------------------------------------------------------
// KV-cache append
// ---------------------------------------------------------------------------
__global__ void kv_cache_append_kernel(const uint4* __restrict__ k_new,
                                       const uint4* __restrict__ v_new, uint4* k_cache,
                                       uint4* v_cache, const std::int32_t* __restrict__ slots,
                                       std::uint64_t tokens, std::uint32_t row_vecs,
                                       std::uint64_t cache_rows, unsigned* error_flag) {
    pdl_wait();
    const std::uint64_t total = tokens * row_vecs;
    for (std::uint64_t i = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         i < total; i += static_cast<std::uint64_t>(gridDim.x) * blockDim.x) {
        const std::uint64_t t = i / row_vecs;
        const std::uint32_t c = static_cast<std::uint32_t>(i - t * row_vecs);
        const std::int64_t slot = slots[t];
        if (slot < 0 || static_cast<std::uint64_t>(slot) >= cache_rows) {
            if (c == 0 && error_flag != nullptr) atomicOr(error_flag, 1u);
            continue;
        }
        const std::uint64_t dst = static_cast<std::uint64_t>(slot) * row_vecs + c;
        k_cache[dst] = k_new[i];
        v_cache[dst] = v_new[i];
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Decode: split over positions, then merge
// ---------------------------------------------------------------------------
struct DecodeParams {
    const __half* q;            // [batch, q_heads, D]
    const __half* k_cache;      // [cache_rows, kv_heads, D]
    const __half* v_cache;
    const std::int32_t* seq_lens;  // [batch]
    __half* out;                // [batch, q_heads, D]
    float* part_o;              // [batch, q_heads, chunks, D]
    float* part_ml;             // [batch, q_heads, chunks, 2] (max, sum), log2 units
    std::uint64_t seq_capacity; // cache rows per sequence
    std::uint32_t q_heads, kv_heads, group;  // group = q_heads / kv_heads
    std::uint32_t head_groups;               // CTAs per KV head: ceil(group / 16)
    std::uint32_t chunks, chunk_len;         // positions per chunk (whole tiles)
    std::uint64_t max_len;      // positions beyond are not attended
    float scale_log2;           // scale * log2(e)
};

__device__ __forceinline__ float2 half2_bits_to_float2(std::uint32_t v) {
    __half2 h;
    memcpy(&h, &v, sizeof(h));
    return __half22float2(h);
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ std::uint32_t cluster_rank() {
    std::uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// A float of cluster CTA `rank`'s shared memory at this CTA's address `addr`.
__device__ __forceinline__ float ld_dsmem_f32(std::uint32_t addr, std::uint32_t rank) {
    std::uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Geometry of the decode split kernel for head_dim D.  A tile is kPos
// cached positions of one KV head: K (8 KB) then V (8 KB) in shared memory,
// each [kPos rows][D] f16 with the 16-byte chunk c of row r stored at chunk
// c ^ (r & 7), so the eight rows an ldmatrix reads at one chunk column fall
// in eight different 16-byte bank groups.
template <int D>
struct DecodeTile {
    static constexpr int kPos = kStageBytes / (4 * D);  // D = 64: 32, D = 128: 16
    static constexpr int kCpr = D / 8;                 // 16-byte chunks per row
    static constexpr int kHalfBytes = kPos * D * 2;    // the K (or V) rows
    static constexpr int kChunksPerLane = kHalfBytes / 16 / 32;
    static constexpr int kRowStep = 32 / kCpr;         // rows between a lane's chunks
    static_assert(2 * kHalfBytes == kStageBytes, "a stage holds K and V of one tile");
    static_assert(kPos % 16 == 0, "whole k16 steps of positions");
};

__device__ __forceinline__ void ldsm_x4(std::uint32_t addr, std::uint32_t& r0, std::uint32_t& r1,
                                        std::uint32_t& r2, std::uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(std::uint32_t addr, std::uint32_t& r0,
                                              std::uint32_t& r1, std::uint32_t& r2,
                                              std::uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ std::uint32_t half2_bits(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    std::uint32_t u;
    memcpy(&u, &h, sizeof(u));
    return u;
}

// p = hi + lo with hi = f16(p) and lo = f16(p - hi): the probabilities keep
// about 22 bits through the f16 P.V contraction.
__device__ __forceinline__ void split_pair(float a, float b, std::uint32_t& hi,
                                           std::uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    memcpy(&hi, &h, sizeof(hi));
    lo = half2_bits(a - f.x, b - f.y);
}

// One CTA: sequence b = blockIdx.z, (KV head, head group) = blockIdx.y,
// chunk = blockIdx.x.  The CTA's up to 16 query heads are the MMA rows.
// Warp w takes the chunk's tiles w, w + 8, ... through its own ring of
// kStagesPerWarp stages and keeps its own online softmax; the eight warps'
// states meet in shared memory at the end.
// CLUSTER: the chunks of a (sequence, head group) are one thread-block
// cluster (grid.x = chunks <= kMaxClusterChunks); each CTA leaves its merged
// state in its own shared memory and the cluster's CTAs merge the chunks over
// distributed shared memory, so no partials go to global memory and no merge
// kernel follows.
template <int D, bool CLUSTER>
__global__ void __launch_bounds__(kThreads, 1) gqa_decode_split_kernel(const DecodeParams p) {
    using T = DecodeTile<D>;
    constexpr int TP = T::kPos;
    constexpr int CPR = T::kCpr;
    constexpr int NK = T::kChunksPerLane;
    constexpr int RS = T::kRowStep;
    constexpr int NT = TP / 8;   // n8 tiles of S per tile
    constexpr int DN = D / 8;    // n8 tiles of O
    constexpr int DK = D / 16;   // k16 steps of S
    extern __shared__ __align__(128) std::uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const std::uint32_t b = blockIdx.z;
    const std::uint32_t kvh = blockIdx.y / p.head_groups;
    const std::uint32_t hgrp = blockIdx.y - kvh * p.head_groups;
    const std::uint32_t chunk = blockIdx.x;
    const std::uint32_t h0 = kvh * p.group + hgrp * kHeadsPerCta;  // first query head
    const std::uint32_t nh = min(static_cast<std::uint32_t>(kHeadsPerCta),
                                 p.group - hgrp * kHeadsPerCta);
    std::uint8_t* wsm = smem + warp * (kStagesPerWarp * kStageBytes);
    const std::uint32_t ring = smem_u32(wsm);

    pdl_wait();
    const std::int64_t len = min(static_cast<std::int64_t>(p.seq_lens[b]),
                                 static_cast<std::int64_t>(p.max_len));
    const std::int64_t t0 = static_cast<std::int64_t>(chunk) * p.chunk_len;
    const std::int64_t t1 = min(len, t0 + static_cast<std::int64_t>(p.chunk_len));
    const int chunk_tiles = t1 > t0 ? static_cast<int>((t1 - t0 + TP - 1) / TP) : 0;
    const int my_tiles = chunk_tiles > warp ? (chunk_tiles - warp + kWarpsPerCta - 1) / kWarpsPerCta : 0;

    // Q as the MMA A operand: rows g and g + 8 (query heads h0 + row; rows
    // past the CTA's heads are zero), k-step s covers dimensions 16s .. 16s+15.
    std::uint32_t qa[DK][4];
    {
        const __half* q_b = p.q + static_cast<std::uint64_t>(b) * p.q_heads * D;
        const bool r0ok = static_cast<std::uint32_t>(g) < nh, r1ok = static_cast<std::uint32_t>(g + 8) < nh;
        const std::uint32_t* q0 = reinterpret_cast<const std::uint32_t*>(q_b + (h0 + g) * D);
        const std::uint32_t* q1 = reinterpret_cast<const std::uint32_t*>(q_b + (h0 + g + 8) * D);
#pragma unroll
        for (int s = 0; s < DK; ++s) {
            qa[s][0] = r0ok ? q0[8 * s + t] : 0u;
            qa[s][1] = r1ok ? q1[8 * s + t] : 0u;
            qa[s][2] = r0ok ? q0[8 * s + 4 + t] : 0u;
            qa[s][3] = r1ok ? q1[8 * s + 4 + t] : 0u;
        }
    }

    // Loader: lane l copies chunks l + 32k (row r0 + k RS, chunk column c)
    // of K and of V; rows past the chunk's end re-read its last row (their
    // scores are masked, and re-read rows hold finite cache data).
    const int r0 = lane / CPR, c = lane % CPR;
    const std::uint64_t row_bytes = static_cast<std::uint64_t>(p.kv_heads) * D * 2;
    const std::uint8_t* kbase = reinterpret_cast<const std::uint8_t*>(p.k_cache) +
                                (static_cast<std::uint64_t>(b) * p.seq_capacity * p.kv_heads + kvh) * D * 2 + c * 16;
    const std::uint8_t* vbase = reinterpret_cast<const std::uint8_t*>(p.v_cache) +
                                (static_cast<std::uint64_t>(b) * p.seq_capacity * p.kv_heads + kvh) * D * 2 + c * 16;
    auto issue = [&](int n) {
        if (n < my_tiles) {
            const std::int64_t pos0 = t0 + static_cast<std::int64_t>(warp + kWarpsPerCta * n) * TP;
            const std::uint32_t dst0 = ring + (n % kStagesPerWarp) * kStageBytes;
#pragma unroll
            for (int k = 0; k < NK; ++k) {
                const int r = r0 + k * RS;
                const std::int64_t pos = min(pos0 + r, t1 - 1);
                const std::uint64_t off = static_cast<std::uint64_t>(pos) * row_bytes;
                const std::uint32_t dst = dst0 + (r * CPR + (c ^ (r & 7))) * 16;
                cp_async_16_default(dst, kbase + off);
                cp_async_16_default(dst + T::kHalfBytes, vbase + off);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s + 1 < kStagesPerWarp; ++s) issue(s);

    // ldmatrix lane addresses (bytes from a stage): matrix i = lane / 8,
    // row r = lane % 8.  K (non-transposed): rows 8j + r, chunk 4kk + i.
    // V (transposed): rows 16kk + 8 (i & 1) + r, chunk n + (i >> 1).
    const int li = lane >> 3, lr = lane & 7;
    std::uint32_t koff[DK / 2];
#pragma unroll
    for (int kk = 0; kk < DK / 2; ++kk) koff[kk] = (lr * CPR + ((4 * kk + li) ^ lr)) * 16;
    std::uint32_t voff[DN / 2];
#pragma unroll
    for (int n = 0; n < DN / 2; ++n)
        voff[n] = T::kHalfBytes + ((8 * (li & 1) + lr) * CPR + ((2 * n + (li >> 1)) ^ lr)) * 16;

    float m0 = -INFINITY, m1 = -INFINITY;  // running max of rows g, g + 8 (log2 units)
    float l0 = 0.f, l1 = 0.f;              // this lane's share of the running sums
    float o[DN][4];
#pragma unroll
    for (int n = 0; n < DN; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    for (int n = 0; n < my_tiles; ++n) {
        issue(n + kStagesPerWarp - 1);
        cp_async_wait<kStagesPerWarp - 1>();
        __syncwarp();
        const std::uint32_t st = ring + (n % kStagesPerWarp) * kStageBytes;
        // S = Q K^T for the tile's TP positions (columns)
        float s[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < DK / 2; ++kk) {
                std::uint32_t b0, b1, b2, b3;
                ldsm_x4(st + koff[kk] + j * 8 * CPR * 16, b0, b1, b2, b3);
                mma_16816(s[j], qa[2 * kk][0], qa[2 * kk][1], qa[2 * kk][2], qa[2 * kk][3], b0, b1, s[j]);
                mma_16816(s[j], qa[2 * kk + 1][0], qa[2 * kk + 1][1], qa[2 * kk + 1][2], qa[2 * kk + 1][3],
                          b2, b3, s[j]);
            }
        }
        // scale into log2 units; mask positions past the chunk's end
        const std::int64_t valid = t1 - (t0 + static_cast<std::int64_t>(warp + kWarpsPerCta * n) * TP);
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 8 * j + 2 * t + (e & 1);
                float x = s[j][e] * p.scale_log2;
                if (valid < TP && col >= valid) x = -INFINITY;
                s[j][e] = x;
                if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // every tile holds a valid position, so the new maxima are finite
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float a0 = ex2(m0 - mn0), a1 = ex2(m1 - mn1);  // ex2(-inf) = 0
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            s[j][0] = ex2(s[j][0] - mn0);
            s[j][1] = ex2(s[j][1] - mn0);
            s[j][2] = ex2(s[j][2] - mn1);
            s[j][3] = ex2(s[j][3] - mn1);
            ps0 += s[j][0] + s[j][1];
            ps1 += s[j][2] + s[j][3];
        }
        l0 = fmaf(l0, a0, ps0);
        l1 = fmaf(l1, a1, ps1);
#pragma unroll
        for (int dn = 0; dn < DN; ++dn) {
            o[dn][0] *= a0;
            o[dn][1] *= a0;
            o[dn][2] *= a1;
            o[dn][3] *= a1;
        }
        // O += P V: the S accumulators of n8 tiles 2kk, 2kk+1 are the A
        // fragment of k-step kk (positions 16kk .. 16kk+15)
#pragma unroll
        for (int kk = 0; kk < TP / 16; ++kk) {
            std::uint32_t ah[4], al[4];
            split_pair(s[2 * kk][0], s[2 * kk][1], ah[0], al[0]);
            split_pair(s[2 * kk][2], s[2 * kk][3], ah[1], al[1]);
            split_pair(s[2 * kk + 1][0], s[2 * kk + 1][1], ah[2], al[2]);
            split_pair(s[2 * kk + 1][2], s[2 * kk + 1][3], ah[3], al[3]);
#pragma unroll
            for (int dn = 0; dn < DN / 2; ++dn) {
                std::uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(st + voff[dn] + kk * 16 * CPR * 16, b0, b1, b2, b3);
                mma_16816(o[2 * dn], ah[0], ah[1], ah[2], ah[3], b0, b1, o[2 * dn]);
                mma_16816(o[2 * dn], al[0], al[1], al[2], al[3], b0, b1, o[2 * dn]);
                mma_16816(o[2 * dn + 1], ah[0], ah[1], ah[2], ah[3], b2, b3, o[2 * dn + 1]);
                mma_16816(o[2 * dn + 1], al[0], al[1], al[2], al[3], b2, b3, o[2 * dn + 1]);
            }
        }
        __syncwarp();  // the slot is refilled by the next iteration's issue
    }
    cp_async_wait<0>();
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // The warps' states meet in shared memory, each warp writing into its
    // own (drained) ring: O [16][D] f32, then max [16] and sum [16].
    __syncwarp();
    float* co = reinterpret_cast<float*>(wsm);
    float* cm = co + kHeadsPerCta * D;
    float* cl = cm + kHeadsPerCta;
#pragma unroll
    for (int dn = 0; dn < DN; ++dn) {
        *reinterpret_cast<float2*>(co + g * D + 8 * dn + 2 * t) = make_float2(o[dn][0], o[dn][1]);
        *reinterpret_cast<float2*>(co + (g + 8) * D + 8 * dn + 2 * t) = make_float2(o[dn][2], o[dn][3]);
    }
    if (t == 0) {
        cm[g] = m0;
        cm[g + 8] = m1;
        cl[g] = l0;
        cl[g + 8] = l1;
    }
    __syncthreads();
    const std::uint64_t qh0 = static_cast<std::uint64_t>(b) * p.q_heads + h0;
    for (std::uint32_t i = threadIdx.x; i < nh * D; i += kThreads) {
        const std::uint32_t row = i / D, d = i - row * D;
        float mw[kWarpsPerCta];
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarpsPerCta; ++w) {
            mw[w] = reinterpret_cast<const float*>(smem + w * (kStagesPerWarp * kStageBytes))[kHeadsPerCta * D + row];
            M = fmaxf(M, mw[w]);
        }
        float acc = 0.f, L = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kWarpsPerCta; ++w) {
                const float* cw = reinterpret_cast<const float*>(smem + w * (kStagesPerWarp * kStageBytes));
                const float wt = ex2(mw[w] - M);  // a warp without tiles: ex2(-inf) = 0
                acc = fmaf(cw[row * D + d], wt, acc);
                L = fmaf(cw[kHeadsPerCta * D + kHeadsPerCta + row], wt, L);
            }
        }
        if constexpr (CLUSTER) {
            // this chunk's state, in warp 0's ring past its O/max/sum area
            float* cr = reinterpret_cast<float*>(smem + kClusterStateOffset);
            cr[row * D + d] = acc;
            if (d == 0) {
                cr[kHeadsPerCta * D + row] = M;
                cr[kHeadsPerCta * D + kHeadsPerCta + row] = L;
            }
        } else if (p.chunks == 1) {
            p.out[(qh0 + row) * D + d] = __float2half_rn(L > 0.f ? acc / L : 0.f);
        } else {
            p.part_o[((qh0 + row) * p.chunks + chunk) * D + d] = acc;
            if (d == 0) {
                p.part_ml[((qh0 + row) * p.chunks + chunk) * 2] = M;
                p.part_ml[((qh0 + row) * p.chunks + chunk) * 2 + 1] = L;
            }
        }
    }
    if constexpr (CLUSTER) {
        cluster_sync();  // every chunk's state is in its CTA's shared memory
        // Each CTA merges a share of the elements: the chunks' weights per
        // row first (into this CTA's warp-1 ring), then the outputs.
        const std::uint32_t rank = cluster_rank();
        const std::uint32_t cr = smem_u32(smem + kClusterStateOffset);
        float* wts = reinterpret_cast<float*>(smem + kStagesPerWarp * kStageBytes);
        constexpr int WS = kMaxClusterChunks + 1;  // weights of a row, then its sum
        if (threadIdx.x < nh) {
            const std::uint32_t row = threadIdx.x;
            float mc[kMaxClusterChunks];
            float Mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < kMaxClusterChunks; ++c) {
                mc[c] = static_cast<std::uint32_t>(c) < p.chunks
                            ? ld_dsmem_f32(cr + (kHeadsPerCta * D + row) * 4, c)
                            : -INFINITY;
                Mx = fmaxf(Mx, mc[c]);
            }
            float L = 0.f;
#pragma unroll
            for (int c = 0; c < kMaxClusterChunks; ++c) {
                float w = 0.f;
                if (Mx != -INFINITY && mc[c] != -INFINITY) {
                    w = ex2(mc[c] - Mx);
                    L = fmaf(ld_dsmem_f32(cr + (kHeadsPerCta * D + kHeadsPerCta + row) * 4, c), w, L);
                }
                wts[row * WS + c] = w;
            }
            wts[row * WS + kMaxClusterChunks] = L;
        }
        __syncthreads();
        for (std::uint32_t i = rank * kThreads + threadIdx.x; i < nh * D; i += p.chunks * kThreads) {
            const std::uint32_t row = i / D, d = i - row * D;
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < kMaxClusterChunks; ++c)
                if (static_cast<std::uint32_t>(c) < p.chunks)
                    acc = fmaf(ld_dsmem_f32(cr + (row * D + d) * 4, c), wts[row * WS + c], acc);
            const float L = wts[row * WS + kMaxClusterChunks];
            p.out[(qh0 + row) * D + d] = __float2half_rn(L > 0.f ? acc / L : 0.f);
        }
        cluster_sync();  // a CTA's shared memory stays until the others have read it
    }
    pdl_launch_dependents();
}

// Merges the chunks of one (sequence, query head): one CTA of D threads.
template <int D>
__global__ void __launch_bounds__(D) gqa_decode_merge_kernel(const DecodeParams p) {
    pdl_wait();
    const std::uint64_t qh = blockIdx.x;  // b * q_heads + h
    const int d = threadIdx.x;
    float M = -INFINITY;
    for (std::uint32_t c = 0; c < p.chunks; ++c) M = fmaxf(M, p.part_ml[(qh * p.chunks + c) * 2]);
    float L = 0.f, acc = 0.f;
    if (M != -INFINITY) {
        for (std::uint32_t c = 0; c < p.chunks; ++c) {
            const float mc = p.part_ml[(qh * p.chunks + c) * 2];
            if (mc == -INFINITY) continue;
            const float w = ex2(mc - M);
            L = fmaf(p.part_ml[(qh * p.chunks + c) * 2 + 1], w, L);
            acc = fmaf(p.part_o[(qh * p.chunks + c) * D + d], w, acc);
        }
    }
    p.out[qh * D + d] = __float2half_rn(L > 0.f ? acc / L : 0.f);
}

// Chunks per sequence.  The split kernel holds one CTA per SM (192 KB of
// rings); a chunk is a whole number of tiles, dealt to the eight warps.
// Cost model: waves of CTAs x (tiles per warp + kFixedTiles), plus
// kMergePenalty when the chunks need the merge kernel (more chunks than a
// cluster holds); the fewest chunks that reach the minimum.  cluster:
// the chunks (2 .. kMaxClusterChunks) merge inside a thread-block cluster.
// Fixed latency of a CTA and the merge kernel's cost, in tiles of the
// warps' work: each about 32 KB of K and V per warp.
constexpr std::uint64_t kFixedTiles = 32768 / kStageBytes;
constexpr std::uint64_t kMergePenalty = 32768 / kStageBytes;

inline void decode_plan(std::uint64_t batch, std::uint64_t kv_heads, std::uint64_t head_groups,
                        std::uint64_t head_dim, std::uint64_t max_len, std::uint32_t& chunks,
                        std::uint32_t& chunk_len, bool& cluster) {
    const std::uint64_t tp = kStageBytes / (4 * head_dim);  // positions per tile
    const std::uint64_t tiles = (max_len + tp - 1) / tp;
    chunks = 1;
    chunk_len = static_cast<std::uint32_t>(tp * (tiles > 0 ? tiles : 1));
    cluster = false;
    if (tiles == 0) return;
    const std::uint64_t units = batch * kv_heads * head_groups;
    std::uint64_t best = ~0ull;
    for (std::uint64_t c = 1; c <= tiles && c <= 4096; ++c) {
        const std::uint64_t tpc = (tiles + c - 1) / c;
        if ((tiles + tpc - 1) / tpc != c) continue;  // same split as a smaller c
        const std::uint64_t waves = (units * c + 147) / 148;
        const std::uint64_t cost =
            waves * ((tpc + kWarpsPerCta - 1) / kWarpsPerCta + kFixedTiles) +
            (c > static_cast<std::uint64_t>(kMaxClusterChunks) ? kMergePenalty : 0);
        if (cost < best) {
            best = cost;
            chunks = static_cast<std::uint32_t>(c);
            chunk_len = static_cast<std::uint32_t>(tpc * tp);
        }
    }
    cluster = chunks > 1 && chunks <= static_cast<std::uint32_t>(kMaxClusterChunks);
}

inline void decode_plan(std::uint64_t batch, std::uint64_t kv_heads, std::uint64_t head_groups,
                        std::uint64_t head_dim, std::uint64_t max_len, std::uint32_t& chunks,
                        std::uint32_t& chunk_len) {
    bool cluster;
    decode_plan(batch, kv_heads, head_groups, head_dim, max_len, chunks, chunk_len, cluster);
}

// Launches the split kernel with the chunks of each (sequence, head group)
// as one cluster, once the device has been seen to fit such a cluster
// (cudaOccupancyMaxActiveClusters, remembered per device and size).  Returns
// false, launching nothing, when it does not.
template <int D>
inline bool launch_decode_cluster(const DecodeParams& p, dim3 grid, cudaStream_t s, int& st) {
    auto kernel = gqa_decode_split_kernel<D, true>;
    static std::atomic<std::uint64_t> smem_done{0};
    static std::atomic<std::uint64_t> fits[kMaxClusterChunks + 1];  // bit dev: 1 = fits
    static std::atomic<std::uint64_t> seen[kMaxClusterChunks + 1];  // bit dev: checked
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    const std::uint64_t bit = 1ull << dev;
    const std::uint32_t n = p.chunks;
    st = ensure_dynamic_smem(kernel, kSplitSmem, smem_done);
    if (st != kSuccess) return true;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSplitSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    if (!(seen[n].load(std::memory_order_acquire) & bit)) {
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            clusters = 0;
        }
        if (clusters > 0) fits[n].fetch_or(bit, std::memory_order_acq_rel);
        seen[n].fetch_or(bit, std::memory_order_acq_rel);
    }
    if (!(fits[n].load(std::memory_order_acquire) & bit)) return false;
    cfg.numAttrs = 2;
    st = static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, p));
    return true;
}

}  // namespace attn
}  // namespace mote

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
// k_new, v_new [tokens, kv_heads, head_dim] f16 -> rows slots[t] of the
// caches [cache_rows, kv_heads, head_dim]; a slot outside [0, cache_rows)
// sets *error_flag (if given) to 1 and is skipped.  kv_heads * head_dim a
// multiple of 8, 16-byte aligned buffers; tokens == 0 returns 0.
extern "C" int mote_cuda_kv_cache_append_f16(const void* k_new, const void* v_new, void* k_cache,
                                             void* v_cache, const void* slots, uint64_t tokens,
                                             uint64_t kv_heads, uint64_t head_dim,
                                             uint64_t cache_rows, void* error_flag, void* stream) {
    using namespace mote;
    if (k_new == nullptr || v_new == nullptr || k_cache == nullptr || v_cache == nullptr ||
        slots == nullptr || stream == nullptr)
        return kInvalidValue;
    if (tokens == 0 || kv_heads == 0 || head_dim == 0) return kSuccess;
    const std::uint64_t row = kv_heads * head_dim;
    if (row % 8 != 0 || row / 8 > 0xffffffffull) return kInvalidValue;
    for (const void* ptr : {k_new, v_new, static_cast<const void*>(k_cache),
                            static_cast<const void*>(v_cache)})
        if (reinterpret_cast<std::uintptr_t>(ptr) % 16 != 0) return kInvalidValue;
    const std::uint64_t total = tokens * (row / 8);
    const std::uint64_t want = (total + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(want < 4096 ? want : 4096);
    return launch_pdl(attn::kv_cache_append_kernel, dim3(blocks), dim3(256),
                      static_cast<cudaStream_t>(stream), static_cast<const uint4*>(k_new),
                      static_cast<const uint4*>(v_new), static_cast<uint4*>(k_cache),
                      static_cast<uint4*>(v_cache), static_cast<const std::int32_t*>(slots),
                      tokens, static_cast<std::uint32_t>(row / 8), cache_rows,
                      static_cast<unsigned*>(error_flag));
}

// Workspace bytes mote_cuda_gqa_attention_decode_f16 needs (0: none).
extern "C" int mote_cuda_gqa_attention_decode_workspace_bytes(uint64_t batch, uint64_t q_heads,
                                                               uint64_t kv_heads,
                                                               uint64_t head_dim,
                                                               uint64_t max_len, uint64_t* bytes) {
    using namespace mote;
    if (bytes == nullptr) return kInvalidValue;
    *bytes = 0;
    if (batch == 0 || q_heads == 0 || kv_heads == 0 || head_dim == 0) return kSuccess;
    if (kv_heads > q_heads || q_heads % kv_heads != 0 || (head_dim != 64 && head_dim != 128))
        return kSuccess;  // the attention call rejects these shapes
    const std::uint64_t group = q_heads / kv_heads;
    std::uint32_t chunks = 1, chunk_len = 0;
    attn::decode_plan(batch, kv_heads, (group + attn::kHeadsPerCta - 1) / attn::kHeadsPerCta,
                      head_dim, max_len, chunks, chunk_len);
    if (chunks > 1) *bytes = batch * q_heads * chunks * (head_dim + 2) * 4;
    return kSuccess;
}

// One query token per sequence attends to its sequence's first seq_lens[b]
// cached positions (the token's own K/V already appended):
//   out[b, h] = softmax(scale * q[b, h] . K[b, :len, h / group]) . V[...]
// q/out [batch, q_heads, head_dim] f16; caches [cache_rows, kv_heads,
// head_dim] f16, sequence b at rows b * seq_capacity + position; seq_lens
// int32 [batch] on the device, each <= max_len <= seq_capacity (max_len
// sizes the split over positions; a longer seq_len is clipped to max_len).
// q_heads a multiple of kv_heads, head_dim 64 or 128; 16-byte aligned
// pointers.  A sequence of length 0
// gets zeros.  workspace: mote_cuda_gqa_attention_decode_workspace_bytes.
extern "C" int mote_cuda_gqa_attention_decode_f16(const void* q, const void* k_cache,
                                                  const void* v_cache, const void* seq_lens,
                                                  void* out, uint64_t batch, uint64_t q_heads,
                                                  uint64_t kv_heads, uint64_t head_dim,
                                                  uint64_t seq_capacity, uint64_t max_len,
                                                  float scale, void* workspace,
                                                  uint64_t workspace_bytes, void* stream) {
    using namespace mote;
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || seq_lens == nullptr ||
        out == nullptr || stream == nullptr)
        return kInvalidValue;
    if (batch == 0 || q_heads == 0) return kSuccess;
    if (kv_heads == 0 || q_heads % kv_heads != 0 || (head_dim != 64 && head_dim != 128))
        return kInvalidValue;
    const std::uint64_t head_groups =
        (q_heads / kv_heads + attn::kHeadsPerCta - 1) / attn::kHeadsPerCta;
    if (max_len > seq_capacity || !std::isfinite(scale) || batch > 65535 ||
        kv_heads * head_groups > 65535 || q_heads > 0xffffffffull)
        return kInvalidValue;
    for (const void* ptr : {q, k_cache, v_cache, static_cast<const void*>(out)})
        if (reinterpret_cast<std::uintptr_t>(ptr) % 16 != 0) return kInvalidValue;
    attn::DecodeParams p{};
    p.q = static_cast<const __half*>(q);
    p.k_cache = static_cast<const __half*>(k_cache);
    p.v_cache = static_cast<const __half*>(v_cache);
    p.seq_lens = static_cast<const std::int32_t*>(seq_lens);
    p.out = static_cast<__half*>(out);
    p.seq_capacity = seq_capacity;
    p.q_heads = static_cast<std::uint32_t>(q_heads);
    p.kv_heads = static_cast<std::uint32_t>(kv_heads);
    p.group = static_cast<std::uint32_t>(q_heads / kv_heads);
    p.head_groups = static_cast<std::uint32_t>(head_groups);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.max_len = max_len;
    bool cluster = false;
    attn::decode_plan(batch, kv_heads, head_groups, head_dim, max_len, p.chunks, p.chunk_len,
                      cluster);
    if (p.chunks > 1) {
        const std::uint64_t need = batch * q_heads * p.chunks * (head_dim + 2) * 4;
        if (workspace == nullptr || workspace_bytes < need ||
            reinterpret_cast<std::uintptr_t>(workspace) % 16 != 0)
            return kInvalidValue;
        p.part_o = static_cast<float*>(workspace);
        p.part_ml = p.part_o + batch * q_heads * p.chunks * head_dim;
    }
    const dim3 grid(p.chunks, static_cast<unsigned>(kv_heads * head_groups),
                    static_cast<unsigned>(batch));
    const auto s = static_cast<cudaStream_t>(stream);
    int st = kSuccess;
    if (cluster && (head_dim == 64 ? attn::launch_decode_cluster<64>(p, grid, s, st)
                                   : attn::launch_decode_cluster<128>(p, grid, s, st)))
        return st;
    if (head_dim == 64) {
        static std::atomic<std::uint64_t> done{0};
        st = ensure_dynamic_smem(attn::gqa_decode_split_kernel<64, false>, attn::kSplitSmem, done);
        if (st == kSuccess)
            st = launch_pdl_smem(attn::gqa_decode_split_kernel<64, false>, grid, dim3(attn::kThreads),
                                 attn::kSplitSmem, s, p);
        if (st == kSuccess && p.chunks > 1)
            st = launch_pdl(attn::gqa_decode_merge_kernel<64>,
                            dim3(static_cast<unsigned>(batch * q_heads)), dim3(64), s, p);
    } else {
        static std::atomic<std::uint64_t> done{0};
        st = ensure_dynamic_smem(attn::gqa_decode_split_kernel<128, false>, attn::kSplitSmem, done);
        if (st == kSuccess)
            st = launch_pdl_smem(attn::gqa_decode_split_kernel<128, false>, grid, dim3(attn::kThreads),
                                 attn::kSplitSmem, s, p);
        if (st == kSuccess && p.chunks > 1)
            st = launch_pdl(attn::gqa_decode_merge_kernel<128>,
                            dim3(static_cast<unsigned>(batch * q_heads)), dim3(128), s, p);
    }
    return st;
}
