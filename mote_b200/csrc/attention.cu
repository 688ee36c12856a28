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
//   V byte of the sequence is read once.  Flash-decoding: a CTA takes one
//   (sequence, KV head, chunk of positions) and all q_heads / kv_heads query
//   heads that share the KV head, streams its chunk through shared memory in
//   128-position tiles (cp.async, double-buffered), keeps an online softmax
//   (running max and sum per query head, exp2 with the scale folded in) and
//   f32 output accumulators, and writes its unnormalised partial output with
//   its max and sum to the workspace; a second kernel merges the chunks.
//   With a single chunk per sequence the first kernel writes the output.
#include "mote_common.cuh"

namespace mote {
namespace attn {

constexpr int kThreads = 128;
constexpr int kTile = 128;        // cached positions per shared-memory tile
constexpr int kMaxGroupDim = 512; // (q_heads / kv_heads) * head_dim per CTA

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
    std::uint32_t chunks, chunk_len;         // positions per chunk (multiple of kTile)
    std::uint64_t max_len;      // positions beyond are not attended
    float scale_log2;           // scale * log2(e)
};

__device__ __forceinline__ float2 half2_bits_to_float2(std::uint32_t v) {
    __half2 h;
    memcpy(&h, &v, sizeof(h));
    return __half22float2(h);
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared memory of the split kernel (byte offsets).
template <int D>
struct DecodeSmem {
    static constexpr int GMAX = kMaxGroupDim / D;  // query heads per CTA
    static constexpr int kRowBytes = D * 2;        // one position of one KV head
    static constexpr int kTileBytes = kTile * kRowBytes;
    static constexpr int kK = 0;                          // [2][kTile][D] f16
    static constexpr int kV = kK + 2 * kTileBytes;        // [2][kTile][D] f16
    static constexpr int kScores = kV + 2 * kTileBytes;   // [GMAX][kTile] f32
    static constexpr int kAlpha = kScores + GMAX * kTile * 4;  // [GMAX] rescale of this tile
    static constexpr int kMax = kAlpha + GMAX * 4;        // [GMAX] running max (log2 units)
    static constexpr int kSum = kMax + GMAX * 4;          // [GMAX] running sum
    static constexpr int kBytes = kSum + GMAX * 4;
    // after the last tile the K buffers hold the 16 position lanes' partial
    // outputs [16][GMAX][D] f32
    static_assert(16 * kMaxGroupDim * 4 <= 2 * kTileBytes, "lane reduction fits the K buffers");
};

// One CTA: sequence b = blockIdx.z, KV head = blockIdx.y, chunk blockIdx.x.
// Threads: 16 position lanes x 8 dimension slices of D/8 elements.
template <int D>
__global__ void __launch_bounds__(kThreads) gqa_decode_split_kernel(const DecodeParams p) {
    using S = DecodeSmem<D>;
    constexpr int DPT = D / 8;      // dimensions per thread
    constexpr int GMAX = S::GMAX;
    constexpr int kRowBytes = S::kRowBytes;
    constexpr int kTileBytes = S::kTileBytes;
    static_assert(DPT % 8 == 0, "16-byte slices");
    extern __shared__ __align__(128) std::uint8_t smem[];
    std::uint8_t* kt = smem + S::kK;
    std::uint8_t* vt = smem + S::kV;
    float* ps = reinterpret_cast<float*>(smem + S::kScores);
    float* alpha_s = reinterpret_cast<float*>(smem + S::kAlpha);
    float* mrun = reinterpret_cast<float*>(smem + S::kMax);
    float* lrun = reinterpret_cast<float*>(smem + S::kSum);
    float* red = reinterpret_cast<float*>(smem + S::kK);

    const int tid = threadIdx.x;
    const int slice = tid & 7;
    const int lane16 = tid >> 3;
    const std::uint32_t b = blockIdx.z, kvh = blockIdx.y, chunk = blockIdx.x;
    const std::uint32_t G = p.group;
    if (tid < GMAX) {
        mrun[tid] = -INFINITY;
        lrun[tid] = 0.f;
    }

    pdl_wait();
    const std::int64_t len = min(static_cast<std::int64_t>(p.seq_lens[b]),
                                 static_cast<std::int64_t>(p.max_len));
    const std::int64_t t0 = static_cast<std::int64_t>(chunk) * p.chunk_len;
    const std::int64_t t1 = min(len, t0 + static_cast<std::int64_t>(p.chunk_len));
    const std::uint64_t rowbase = static_cast<std::uint64_t>(b) * p.seq_capacity;

    // query slices (f32) of the group's heads
    float qv[GMAX][DPT];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
#pragma unroll
        for (int j = 0; j < DPT; ++j) qv[g][j] = 0.f;
        if (static_cast<std::uint32_t>(g) < G) {
            const __half* qh = p.q + (static_cast<std::uint64_t>(b) * p.q_heads + kvh * G + g) * D +
                               slice * DPT;
#pragma unroll
            for (int j = 0; j < DPT; j += 8) {
                const uint4 w = *reinterpret_cast<const uint4*>(qh + j);
                const std::uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = half2_bits_to_float2(ws[e]);
                    qv[g][j + 2 * e] = f.x;
                    qv[g][j + 2 * e + 1] = f.y;
                }
            }
        }
    }
    float o[GMAX][DPT];
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
#pragma unroll
        for (int j = 0; j < DPT; ++j) o[g][j] = 0.f;

    const int tiles = t1 > t0 ? static_cast<int>((t1 - t0 + kTile - 1) / kTile) : 0;
    // tile loader: kTile rows of K and of V, 16-byte copies; rows past the
    // end re-read the last valid row (their scores are masked)
    auto load_tile = [&](int tile, int buf) {
        const std::int64_t base = t0 + static_cast<std::int64_t>(tile) * kTile;
        constexpr int kVecsPerRow = kRowBytes / 16;
        for (int i = tid; i < kTile * kVecsPerRow; i += kThreads) {
            const int r = i / kVecsPerRow;
            const int c = i - r * kVecsPerRow;
            const std::int64_t pos = min(base + r, t1 - 1);
            const std::uint64_t off =
                ((rowbase + static_cast<std::uint64_t>(pos)) * p.kv_heads + kvh) * kRowBytes + c * 16;
            cp_async_16_default(smem_u32(kt + buf * kTileBytes + r * kRowBytes + c * 16),
                                reinterpret_cast<const std::uint8_t*>(p.k_cache) + off);
            cp_async_16_default(smem_u32(vt + buf * kTileBytes + r * kRowBytes + c * 16),
                                reinterpret_cast<const std::uint8_t*>(p.v_cache) + off);
        }
        cp_async_commit();
    };
    if (tiles > 0) load_tile(0, 0);
    for (int tile = 0; tile < tiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < tiles) {
            load_tile(tile + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const std::int64_t base = t0 + static_cast<std::int64_t>(tile) * kTile;
        // scores: 16 positions at a time, 8 threads per position
#pragma unroll 2
        for (int kk = 0; kk < kTile / 16; ++kk) {
            const int r = kk * 16 + lane16;
            const std::uint8_t* krow = kt + buf * kTileBytes + r * kRowBytes + slice * DPT * 2;
            float kv[DPT];
#pragma unroll
            for (int j = 0; j < DPT; j += 8) {
                const uint4 w = *reinterpret_cast<const uint4*>(krow + 2 * j);
                const std::uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = half2_bits_to_float2(ws[e]);
                    kv[j + 2 * e] = f.x;
                    kv[j + 2 * e + 1] = f.y;
                }
            }
            const bool valid = base + r < t1;
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                float a = 0.f;
#pragma unroll
                for (int j = 0; j < DPT; ++j) a = fmaf(qv[g][j], kv[j], a);
                a += __shfl_xor_sync(0xffffffffu, a, 1);
                a += __shfl_xor_sync(0xffffffffu, a, 2);
                a += __shfl_xor_sync(0xffffffffu, a, 4);
                if (slice == 0 && static_cast<std::uint32_t>(g) < G)
                    ps[g * kTile + r] = valid ? a * p.scale_log2 : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax per query head: warp w takes heads w, w + 4, ...
        {
            const int w = tid >> 5, ln = tid & 31;
            for (int g = w; g < static_cast<int>(G); g += kThreads / 32) {
                float v[kTile / 32];
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < kTile / 32; ++i) {
                    v[i] = ps[g * kTile + ln + 32 * i];
                    mx = fmaxf(mx, v[i]);
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float mold = mrun[g];
                const float mnew = fmaxf(mold, mx);  // finite: a tile has a valid position
                float sum = 0.f;
#pragma unroll
                for (int i = 0; i < kTile / 32; ++i) {
                    v[i] = ex2(v[i] - mnew);
                    ps[g * kTile + ln + 32 * i] = v[i];
                    sum += v[i];
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                if (ln == 0) {
                    const float a = mold == -INFINITY ? 0.f : ex2(mold - mnew);
                    alpha_s[g] = a;
                    mrun[g] = mnew;
                    lrun[g] = fmaf(lrun[g], a, sum);
                }
            }
        }
        __syncthreads();
        // P . V: position lane lane16 takes positions lane16 + 16 kk
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (static_cast<std::uint32_t>(g) < G) {
                const float a = alpha_s[g];
#pragma unroll
                for (int j = 0; j < DPT; ++j) o[g][j] *= a;
            }
        }
#pragma unroll 2
        for (int kk = 0; kk < kTile / 16; ++kk) {
            const int r = kk * 16 + lane16;
            const std::uint8_t* vrow = vt + buf * kTileBytes + r * kRowBytes + slice * DPT * 2;
            float vv[DPT];
#pragma unroll
            for (int j = 0; j < DPT; j += 8) {
                const uint4 w = *reinterpret_cast<const uint4*>(vrow + 2 * j);
                const std::uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = half2_bits_to_float2(ws[e]);
                    vv[j + 2 * e] = f.x;
                    vv[j + 2 * e + 1] = f.y;
                }
            }
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                if (static_cast<std::uint32_t>(g) < G) {
                    const float pw = ps[g * kTile + r];
#pragma unroll
                    for (int j = 0; j < DPT; ++j) o[g][j] = fmaf(pw, vv[j], o[g][j]);
                }
            }
        }
        __syncthreads();  // the tile's buffers and scores are reused
    }
    __syncthreads();  // (no tiles) the running statistics are initialised
    // merge the 16 position lanes' partial outputs (K buffers are free now)
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
        if (static_cast<std::uint32_t>(g) < G)
#pragma unroll
            for (int j = 0; j < DPT; ++j) red[(lane16 * GMAX + g) * D + slice * DPT + j] = o[g][j];
    __syncthreads();
    const std::uint64_t qh0 = static_cast<std::uint64_t>(b) * p.q_heads + kvh * G;
    for (std::uint32_t i = tid; i < G * D; i += kThreads) {
        const std::uint32_t g = i / D, d = i - g * D;
        float acc = 0.f;
#pragma unroll 4
        for (int r = 0; r < 16; ++r) acc += red[(r * GMAX + g) * D + d];
        if (p.chunks == 1) {
            const float L = lrun[g];
            p.out[(qh0 + g) * D + d] = __float2half_rn(L > 0.f ? acc / L : 0.f);
        } else {
            p.part_o[((qh0 + g) * p.chunks + chunk) * D + d] = acc;
            if (d == 0) {
                p.part_ml[((qh0 + g) * p.chunks + chunk) * 2] = mrun[g];
                p.part_ml[((qh0 + g) * p.chunks + chunk) * 2 + 1] = lrun[g];
            }
        }
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

template <int D>
constexpr int decode_smem_bytes() {
    return DecodeSmem<D>::kBytes;
}

// Chunks per sequence: enough CTAs for two per SM, each chunk a whole number
// of tiles.
inline void decode_plan(std::uint64_t batch, std::uint64_t kv_heads, std::uint64_t max_len,
                        std::uint32_t& chunks, std::uint32_t& chunk_len) {
    const std::uint64_t tiles = (max_len + kTile - 1) / kTile;
    std::uint64_t want = (2ull * 148 + batch * kv_heads - 1) / (batch * kv_heads);
    if (want < 1) want = 1;
    if (want > tiles) want = tiles;
    if (tiles == 0) want = 1;
    const std::uint64_t tiles_per = tiles == 0 ? 1 : (tiles + want - 1) / want;
    chunk_len = static_cast<std::uint32_t>(tiles_per * kTile);
    chunks = static_cast<std::uint32_t>(tiles == 0 ? 1 : (tiles + tiles_per - 1) / tiles_per);
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
    std::uint32_t chunks = 1, chunk_len = 0;
    attn::decode_plan(batch, kv_heads, max_len, chunks, chunk_len);
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
// q_heads a multiple of kv_heads, head_dim 64 or 128, (q_heads / kv_heads)
// * head_dim <= 512; 16-byte aligned pointers.  A sequence of length 0
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
    if ((q_heads / kv_heads) * head_dim > attn::kMaxGroupDim || max_len > seq_capacity ||
        !std::isfinite(scale) || batch > 65535 || kv_heads > 65535)
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
    p.scale_log2 = scale * 1.4426950408889634f;
    p.max_len = max_len;
    attn::decode_plan(batch, kv_heads, max_len, p.chunks, p.chunk_len);
    if (p.chunks > 1) {
        const std::uint64_t need = batch * q_heads * p.chunks * (head_dim + 2) * 4;
        if (workspace == nullptr || workspace_bytes < need ||
            reinterpret_cast<std::uintptr_t>(workspace) % 16 != 0)
            return kInvalidValue;
        p.part_o = static_cast<float*>(workspace);
        p.part_ml = p.part_o + batch * q_heads * p.chunks * head_dim;
    }
    const dim3 grid(p.chunks, static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
    const auto s = static_cast<cudaStream_t>(stream);
    int st;
    if (head_dim == 64) {
        constexpr int smem = attn::decode_smem_bytes<64>();
        static std::atomic<std::uint64_t> done{0};
        st = ensure_dynamic_smem(attn::gqa_decode_split_kernel<64>, smem, done);
        if (st == kSuccess)
            st = launch_pdl_smem(attn::gqa_decode_split_kernel<64>, grid, dim3(attn::kThreads), smem,
                                 s, p);
        if (st == kSuccess && p.chunks > 1)
            st = launch_pdl(attn::gqa_decode_merge_kernel<64>,
                            dim3(static_cast<unsigned>(batch * q_heads)), dim3(64), s, p);
    } else {
        constexpr int smem = attn::decode_smem_bytes<128>();
        static std::atomic<std::uint64_t> done{0};
        st = ensure_dynamic_smem(attn::gqa_decode_split_kernel<128>, smem, done);
        if (st == kSuccess)
            st = launch_pdl_smem(attn::gqa_decode_split_kernel<128>, grid, dim3(attn::kThreads),
                                 smem, s, p);
        if (st == kSuccess && p.chunks > 1)
            st = launch_pdl(attn::gqa_decode_merge_kernel<128>,
                            dim3(static_cast<unsigned>(batch * q_heads)), dim3(128), s, p);
    }
    return st;
}
