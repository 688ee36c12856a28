// Persistent decoder stack: the non-attention ops of L Llama-style decoder
// layers at decode (one token) in one kernel launch.  No reference
// counterpart: the reference composes these operators one launch at a time
// (docs/architecture.md:180-192); the per-layer arithmetic is that of the
// four-kernel fused layer (q4_0_linear.cu: norm in the staging, RoPE in the
// QKV epilogue, SwiGLU in the gate/up epilogue, residual adds in the O and
// down epilogues).
//
// Per layer, three phases separated by grid barriers:
//   P0  qkv = rope(rms_norm(h, g1) @ Wqkv^T)      and   h1 = h + attn @ Wo^T
//   P1  a   = silu(n @ Wg^T) * (n @ Wu^T),  n = rms_norm(h1, g2)
//   P2  out = h1 + a @ Wd^T                        (the next layer's h)
// where `attn` is the layer's attention output, an input (attention is
// outside this data plane).
//
// Design (B200, HBM-bound at one token):
// * The grid is exactly the resident CTAs (two 8-warp CTAs per SM,
//   cooperative launch), each warp with the Q4_0 GEMV's private cp.async
//   ring of 16-row x 144-byte stages.  A warp's issue cursor walks its work
//   across phases and layers, so the weights of the next phase -- which do
//   not depend on the barrier -- are already streaming while the warp
//   waits at the barrier.  This replaces the per-kernel costs of separate
//   launches (grid drain, dependent-launch release, ring refill).
// * Per phase the tiles (16 weight rows) go round-robin to groups of 1-8
//   warps that split K (the smallest split that covers the phase's tiles
//   in one round); the partials meet in shared memory as in the GEMV.
// * The activations of a phase are staged by the whole CTA after the
//   barrier (coherent L2 loads: they were written during this launch) in
//   the GEMV's permuted order, RMS-normalised in place where the phase
//   needs it, with the GEMV's arithmetic.
// * The down projection (K = ffn) has few tiles (hidden / 16); when ffn / 256
//   is even its K is split in two halves on different CTAs, so every CTA
//   has work.  The halves' f32 partial sums go to a workspace and are added
//   (with h1, in f32, rounded once) by the next phase's staging, which also
//   writes the layer's `out`; after the last layer a final step writes it.
// * Grid barrier: one arrival counter (zeroed before the launch).  A CTA's
//   writes are ordered before its arrival by a CTA barrier and published by
//   the arrival itself, a release reduction (red.release.gpu); every CTA
//   polls the counter with acquire loads until all have arrived (a
//   separate release word written by the last arrival measured 2.7 us per
//   barrier against 1.3 us).  The wait is bounded (1 s of
//   %globaltimer): on expiry the CTA records the timeout in the status word
//   and raises an abort word that ends every other CTA's wait, and all
//   return.
#include "mote_common.cuh"

namespace mote {
namespace stack {

using q4::decode_word;
using q4::kStageBytes;
using q4::kThreads;
using q4::kTileRows;
using q4::kUnitBlocks;
using q4::kUnitBytes;
using q4::kWarps;
using q4::half2_bits_to_float2;
using q4::named_barrier_sync;
using q4::pack_half2;
constexpr int kStages = 4;
constexpr int kRowStride = q4::kRowStride;
constexpr int kZeroBytes = 512;               // zero B operand of the packed columns
constexpr std::uint64_t kBarrierWaitNs = 1000000000ull;
// norm scratch (2 x kWarps floats) + double-buffered group reductions
constexpr int kRedBytes = ((kWarps * 2 + 2 * kWarps * 64) * 4 + 127) / 128 * 128;

// One layer's tensors (device pointers); the C declaration is
// mote_cuda_stack_layer in include/mote_cuda.h.
struct Layer {
    const std::uint8_t* w_qkv;   // [(q_heads + 2 kv_heads) head_dim, hidden] Q4_0
    const std::uint8_t* w_o;     // [hidden, hidden]
    const std::uint8_t* w_gate;  // [ffn, hidden]
    const std::uint8_t* w_up;    // [ffn, hidden]
    const std::uint8_t* w_down;  // [hidden, ffn]
    const __half* gamma1;        // [hidden]
    const __half* gamma2;        // [hidden]
    const __half* attn;          // [hidden] attention output (input)
    const float* cos;            // [head_dim / 2]
    const float* sin;
    __half* qkv;                 // [(q_heads + 2 kv_heads) head_dim] output
    __half* h1;                  // [hidden] output: h + attn @ Wo^T
    __half* a;                   // [ffn] output: SwiGLU
    __half* out;                 // [hidden] output: h1 + a @ Wd^T
};

struct Params {
    const Layer* layers;
    std::uint32_t num_layers;
    const __half* h_in;          // layer 0 input [hidden]
    unsigned* barrier;           // [0] arrivals, [1] abort word (zero at launch)
    float* parts;                // [2 layer parity][2 halves][hidden] down partial sums
    float eps;
    std::uint32_t hidden, ffn, head_dim;
    std::uint32_t rope_rows, rope_tiles, qkv_tiles, o_tiles, gu_tiles, down_tiles;
    std::uint32_t units_h, units_f;
    std::uint32_t down_parts;    // 1, or 2 (K halves on different CTAs)
    std::uint32_t sh[3];         // log2 warps per tile of each phase
    std::uint32_t x_bytes;       // staged activation area
};

__device__ __forceinline__ std::uint64_t global_ns() {
    std::uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Tiles and K units of phase `ph`.
__device__ __forceinline__ std::uint32_t phase_tiles(const Params& p, int ph) {
    return ph == 0 ? p.qkv_tiles + p.o_tiles : ph == 1 ? p.gu_tiles : p.down_tiles * p.down_parts;
}
__device__ __forceinline__ std::uint32_t phase_units(const Params& p, int ph) {
    return ph == 2 ? p.units_f / p.down_parts : p.units_h;
}

// Weight row i (0..15) of tile `tile` of phase `ph` of layer L.
__device__ __forceinline__ const std::uint8_t* tile_row(const Params& p, const Layer& L, int ph,
                                                        std::uint32_t tile, int i) {
    const std::uint64_t pitch_h = static_cast<std::uint64_t>(p.units_h) * kUnitBytes;
    if (ph == 0) {
        if (tile < p.qkv_tiles) {
            std::uint32_t r;
            if (tile < p.rope_tiles) {
                // rope tiles pair rows d and d + head_dim/2 of a head
                const std::uint32_t per_head = p.head_dim / 16;
                const std::uint32_t h = tile / per_head;
                const std::uint32_t j0 = (tile - h * per_head) * 8;
                r = h * p.head_dim + j0 + (i & 7) + (i < 8 ? 0u : p.head_dim / 2);
            } else {
                r = p.rope_rows + (tile - p.rope_tiles) * 16u + i;
            }
            return L.w_qkv + r * pitch_h;
        }
        return L.w_o + ((tile - p.qkv_tiles) * 16u + i) * pitch_h;
    }
    if (ph == 1) {
        const std::uint32_t f = tile * 8u + (i & 7);
        return (i < 8 ? L.w_gate : L.w_up) + f * pitch_h;
    }
    // down items: tile * parts + half, each half of K its own item
    const std::uint64_t pitch_f = static_cast<std::uint64_t>(p.units_f) * kUnitBytes;
    const std::uint32_t half = tile % p.down_parts;
    return L.w_down + (tile / p.down_parts * 16u + i) * pitch_f +
           static_cast<std::uint64_t>(half) * (p.units_f / p.down_parts) * kUnitBytes;
}

// A warp's share of a phase: tiles first, first + stride, ... below `tiles`,
// units [u0, u0 + spt) of each.
struct Share {
    std::uint32_t first, stride, tiles, u0, spt, my_tiles, sh, grp, wig;
};

__device__ __forceinline__ Share share_of(const Params& p, int ph, int warp) {
    Share s;
    s.sh = ph == 0 ? p.sh[0] : ph == 1 ? p.sh[1] : p.sh[2];  // no dynamic index into the parameters
    const std::uint32_t split = 1u << s.sh;
    s.grp = static_cast<std::uint32_t>(warp) >> s.sh;
    s.wig = static_cast<std::uint32_t>(warp) & (split - 1);
    s.first = blockIdx.x + s.grp * gridDim.x;
    s.stride = gridDim.x * (kWarps >> s.sh);
    s.tiles = phase_tiles(p, ph);
    const std::uint32_t units = phase_units(p, ph);
    s.u0 = (units * s.wig) >> s.sh;
    s.spt = ((units * (s.wig + 1)) >> s.sh) - s.u0;
    s.my_tiles = s.tiles > s.first ? (s.tiles - s.first + s.stride - 1) / s.stride : 0;
    return s;
}

// Grid barrier (see the file comment).  All threads call it; returns false
// if the launch is being aborted.
__device__ __forceinline__ bool grid_barrier(const Params& p, unsigned& passed,
                                             volatile unsigned* s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        ++passed;
        const unsigned target = passed * gridDim.x;
        // arrival: a release reduction publishes the CTA's writes (ordered
        // before it by the CTA barrier) with the increment itself
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.barrier) : "memory");
        const std::uint64_t start = global_ns();
        unsigned ok = 1;
        for (;;) {
            if (static_cast<int>(ld_acquire_gpu(&p.barrier[0]) - target) >= 0) break;
            if (*reinterpret_cast<volatile unsigned*>(&p.barrier[1]) != 0u) {
                ok = 0;
                break;
            }
            if (global_ns() - start > kBarrierWaitNs) {
                atomicOr(&g_device_status, kDevWaitTimeout);
                atomicExch(&p.barrier[1], 1u);
                ok = 0;
                break;
            }
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

__global__ void __launch_bounds__(kThreads, 2) decoder_stack_kernel(const Params p) {
    extern __shared__ __align__(1024) std::uint8_t smem[];
    __shared__ unsigned s_flag;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;

    std::uint8_t* xs = smem;                                   // staged rows
    std::uint8_t* zero = smem + p.x_bytes;                     // kZeroBytes of zeros
    std::uint8_t* ring = zero + kZeroBytes + warp * kStages * kStageBytes;
    float* red = reinterpret_cast<float*>(zero + kZeroBytes + kWarps * kStages * kStageBytes);
    // phase 0: the layer input h in natural order (the O projection's residual)
    __half* hres = reinterpret_cast<__half*>(reinterpret_cast<std::uint8_t*>(red) + kRedBytes);
    for (int i = threadIdx.x; i < kZeroBytes / 16; i += kThreads)
        reinterpret_cast<uint4*>(zero)[i] = make_uint4(0u, 0u, 0u, 0u);

    // ---- issue cursor: (layer, phase, k-th tile of the share, unit) --------
    constexpr int kChunks = kTileRows * (kUnitBytes / 16);   // 144
    constexpr int kChunksPerLane = (kChunks + 31) / 32;      // 5
    std::uint32_t dst_off[kChunksPerLane];
    int chunk_row[kChunksPerLane];
    std::uint32_t src_off[kChunksPerLane];
#pragma unroll
    for (int j = 0; j < kChunksPerLane; ++j) {
        const int c = min(lane + 32 * j, kChunks - 1);
        chunk_row[j] = c / 9;
        dst_off[j] = chunk_row[j] * kRowStride + (c % 9) * 16;
        src_off[j] = (c % 9) * 16;
    }
    const std::uint32_t ring_s = smem_u32(ring);
    const std::uint64_t policy = l2_evict_first_policy();
    std::uint32_t c_layer = 0, c_k = 0, c_u = 0, c_slot = 0;
    int c_ph = 0;
    Share cs = share_of(p, 0, warp);
    const std::uint8_t* src[kChunksPerLane];
    bool c_done = false;
    // Moves the cursor to the first phase (from the current one on) in
    // which this warp has tiles, and points src at its first unit.
    auto settle = [&]() {
        while (!c_done && c_k >= cs.my_tiles) {
            c_k = 0;
            c_u = 0;
            if (++c_ph == 3) {
                c_ph = 0;
                if (++c_layer == p.num_layers) {
                    c_done = true;
                    break;
                }
            }
            cs = share_of(p, c_ph, warp);
        }
        if (c_done) return;
        const std::uint32_t tile = cs.first + c_k * cs.stride;
        const Layer& L = p.layers[c_layer];
#pragma unroll
        for (int j = 0; j < kChunksPerLane; ++j)
            src[j] = tile_row(p, L, c_ph, tile, chunk_row[j]) +
                     static_cast<std::uint64_t>(cs.u0 + c_u) * kUnitBytes + src_off[j];
    };
    settle();
    auto issue = [&]() {
        if (!c_done) {
            const std::uint32_t slot_s = ring_s + c_slot * kStageBytes;
#pragma unroll
            for (int j = 0; j < kChunksPerLane; ++j)
                if (lane + 32 * j < kChunks) cp_async_16(slot_s + dst_off[j], src[j], policy);
            if (++c_u == cs.spt) {
                c_u = 0;
                ++c_k;
                settle();
            } else {
#pragma unroll
                for (int j = 0; j < kChunksPerLane; ++j) src[j] += kUnitBytes;
            }
        }
        c_slot = c_slot + 1 == kStages ? 0 : c_slot + 1;
        cp_async_commit();
    };
    for (int s = 0; s + 1 < kStages; ++s) issue();

    // ---- consumer ------------------------------------------------------------
    unsigned passed = 0;
    std::uint32_t slot = 0;
    const std::uint32_t ring_addr = smem_u32(ring) + g * kRowStride;
    const std::uint32_t zero_s = smem_u32(zero) + 8 * t;
    bool alive = true;
    for (std::uint32_t l = 0; l < p.num_layers && alive; ++l) {
        const Layer& L = p.layers[l];
        // this layer's input: h_in, the previous layer's `out`, or (down
        // halves) the previous h1 plus the halves' partial sums
        const __half* h = l == 0 ? p.h_in : p.layers[l - 1].out;
        const bool h_from_parts = l != 0 && p.down_parts == 2;
        for (int ph = 0; ph < 3 && alive; ++ph) {
            if (l != 0 || ph != 0) {
                alive = grid_barrier(p, passed, &s_flag);
                if (!alive) break;
            }
            // ---- stage this phase's activation rows (permuted groups of 4)
            const std::uint32_t K = ph == 2 ? p.ffn : p.hidden;
            const std::uint32_t x_stride = 2 * K + 32;
            {
                const __half* row0 = ph == 0 ? h : ph == 1 ? L.h1 : L.a;
                const int nrows = ph == 0 ? 2 : 1;
                for (int r = 0; r < nrows; ++r)
                    for (std::uint32_t c = threadIdx.x; c < K / 8; c += kThreads) {
                        uint4 v;
                        if (r == 0 && ph == 0 && h_from_parts) {
                            // h = h1 + (half 0 + half 1), f32, rounded once
                            const Layer& P = p.layers[l - 1];
                            const float4* pa = reinterpret_cast<const float4*>(
                                                   p.parts + ((l - 1) & 1u) * 2 * p.hidden) + 2 * c;
                            const float4* pb = pa + p.hidden / 4;
                            const uint4 hv = __ldcg(reinterpret_cast<const uint4*>(P.h1) + c);
                            const float4 a0 = __ldcg(pa), a1 = __ldcg(pa + 1);
                            const float4 b0 = __ldcg(pb), b1 = __ldcg(pb + 1);
                            const float2 h01 = half2_bits_to_float2(hv.x);
                            const float2 h23 = half2_bits_to_float2(hv.y);
                            const float2 h45 = half2_bits_to_float2(hv.z);
                            const float2 h67 = half2_bits_to_float2(hv.w);
                            v.x = pack_half2((a0.x + b0.x) + h01.x, (a0.y + b0.y) + h01.y);
                            v.y = pack_half2((a0.z + b0.z) + h23.x, (a0.w + b0.w) + h23.y);
                            v.z = pack_half2((a1.x + b1.x) + h45.x, (a1.y + b1.y) + h45.y);
                            v.w = pack_half2((a1.z + b1.z) + h67.x, (a1.w + b1.w) + h67.y);
                            if (blockIdx.x == 0) reinterpret_cast<uint4*>(P.out)[c] = v;
                        } else {
                            v = __ldcg(reinterpret_cast<const uint4*>(r == 0 ? row0 : L.attn) + c);
                        }
                        if (r == 0 && ph == 0) reinterpret_cast<uint4*>(hres)[c] = v;
                        uint4 o;
                        o.x = prmt(v.x, v.y, 0x5410u);
                        o.y = prmt(v.x, v.y, 0x7632u);
                        o.z = prmt(v.z, v.w, 0x5410u);
                        o.w = prmt(v.z, v.w, 0x7632u);
                        *reinterpret_cast<uint4*>(xs + r * x_stride + 16 * c) = o;
                    }
                __syncthreads();
                if (ph < 2) {
                    // RMSNorm of row 0 in place (the GEMV's fused-norm
                    // arithmetic): per-thread sums of squares, a block
                    // reduction, x * inv * gamma rounded once to f16
                    float* part = red;                  // [kWarps]
                    float* inv_s = red + kWarps;
                    const std::uint32_t chunks = K / 8;
                    float ss = 0.f;
                    for (std::uint32_t i = threadIdx.x; i < chunks; i += kThreads) {
                        const uint4 v = *reinterpret_cast<const uint4*>(xs + 16 * i);
                        const std::uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            __half2 hh;
                            memcpy(&hh, &words[q], 4);
                            const float2 f = __half22float2(hh);
                            ss = __fadd_rn(ss, __fmul_rn(f.x, f.x));
                            ss = __fadd_rn(ss, __fmul_rn(f.y, f.y));
                        }
                    }
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
                    if (lane == 0) part[warp] = ss;
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        float total = 0.f;
#pragma unroll
                        for (int w = 0; w < kWarps; ++w) total += part[w];
                        *inv_s = inv_rms(total, K, p.eps);
                    }
                    __syncthreads();
                    const float inv = *inv_s;
                    const __half* gamma = ph == 0 ? L.gamma1 : L.gamma2;
                    for (std::uint32_t i = threadIdx.x; i < chunks; i += kThreads) {
                        const uint4 gr = __ldg(reinterpret_cast<const uint4*>(gamma) + i);
                        const std::uint32_t gw[4] = {prmt(gr.x, gr.y, 0x5410u), prmt(gr.x, gr.y, 0x7632u),
                                                     prmt(gr.z, gr.w, 0x5410u), prmt(gr.z, gr.w, 0x7632u)};
                        uint4* at = reinterpret_cast<uint4*>(xs + 16 * i);
                        const uint4 v = *at;
                        const std::uint32_t words[4] = {v.x, v.y, v.z, v.w};
                        std::uint32_t out[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            __half2 hx, hg;
                            memcpy(&hx, &words[q], 4);
                            memcpy(&hg, &gw[q], 4);
                            const float2 f = __half22float2(hx);
                            const float2 w = __half22float2(hg);
                            const __half2 o = __floats2half2_rn(norm_out(f.x, inv, w.x),
                                                                norm_out(f.y, inv, w.y));
                            memcpy(&out[q], &o, 4);
                        }
                        *at = make_uint4(out[0], out[1], out[2], out[3]);
                    }
                    __syncthreads();
                }
            }
            // ---- this warp's tiles of the phase
            const Share s = share_of(p, ph, warp);
            const std::uint32_t split = 1u << s.sh;
            for (std::uint32_t k = 0; k < s.my_tiles; ++k) {
                const std::uint32_t tile = s.first + k * s.stride;
                // x row of the tile: row 1 (attn) for the O tiles of phase 0
                const std::uint32_t xrow = (ph == 0 && tile >= p.qkv_tiles) ? 1u : 0u;
                // the K half of a down item starts units_f / 2 units in
                const std::uint32_t kbase = ph == 2 ? (tile % p.down_parts) *
                                                          (p.units_f / p.down_parts) * (kUnitBlocks * 64)
                                                    : 0u;
                const std::uint32_t xreal = smem_u32(xs) + xrow * x_stride + kbase + 8 * t;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                for (std::uint32_t st = 0; st < s.spt; ++st) {
                    issue();
                    cp_async_wait<kStages - 1>();
                    __syncwarp();
                    const std::uint32_t ra = ring_addr + slot * kStageBytes;
                    const std::uint32_t qa = ra + 4 * t;
                    constexpr std::uint32_t kR8 = 8 * kRowStride;
                    const std::uint32_t xo = (s.u0 + st) * (kUnitBlocks * 64);
                    // column j of the chain = block j of the unit: lane g
                    // reads the real row for j == g, the zero area otherwise
                    std::uint32_t xs_j[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) xs_j[j] = g == j ? xreal + xo : zero_s;
                    float dacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                    q4::static_for<0, 8>([&](auto bb) {
                        constexpr int b = decltype(bb)::value;
                        std::uint32_t wa, wb;
                        if constexpr (b & 1) {
                            wa = lds32i<18 * b + 2>(qa);
                            wb = lds32i<kR8 + 18 * b + 2>(qa);
                        } else {
                            wa = prmt(lds32i<18 * b>(qa), lds32i<18 * b + 4>(qa), 0x5432u);
                            wb = prmt(lds32i<kR8 + 18 * b>(qa), lds32i<kR8 + 18 * b + 4>(qa), 0x5432u);
                        }
                        std::uint32_t al02, al13, ah02, ah13, bl02, bl13, bh02, bh13;
                        decode_word(wa, al02, al13, ah02, ah13);
                        decode_word(wb, bl02, bl13, bh02, bh13);
                        const uint2 xl = lds64i<b * 64>(xs_j[b]);
                        const uint2 xh = lds64i<b * 64 + 32>(xs_j[b]);
                        mma_16816(dacc[0], al02, bl02, al13, bl13, xl.x, xl.y, dacc[0]);
                        mma_16816(dacc[1], ah02, bh02, ah13, bh13, xh.x, xh.y, dacc[1]);
                    });
                    // each column's block partial times its block's scale
                    const std::uint32_t da0 = ra + 18u * static_cast<std::uint32_t>(2 * t);
                    const std::uint32_t da1 = ra + 18u * static_cast<std::uint32_t>(2 * t + 1);
                    const float dg0 = half_bits_to_float(lds16i<0>(da0));
                    const float dh0 = half_bits_to_float(lds16i<kR8>(da0));
                    const float dg1 = half_bits_to_float(lds16i<0>(da1));
                    const float dh1 = half_bits_to_float(lds16i<kR8>(da1));
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        acc[0] = fmaf(dg0, dacc[hh][0], acc[0]);
                        acc[1] = fmaf(dg1, dacc[hh][1], acc[1]);
                        acc[2] = fmaf(dh0, dacc[hh][2], acc[2]);
                        acc[3] = fmaf(dh1, dacc[hh][3], acc[3]);
                    }
                    __syncwarp();
                    slot = slot + 1 == kStages ? 0 : slot + 1;
                }
                // fold the 8 columns: rows g (acc[0]) and g + 8 (acc[2])
                acc[0] += acc[1];
                acc[2] += acc[3];
#pragma unroll
                for (int i = 0; i < 4; i += 2) {
                    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
                    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
                }
                float v0 = acc[0], v2 = acc[2];
                bool writer = true;
                if (split > 1) {
                    // meet the group's other K slices (double-buffered area)
                    float* gred = red + kWarps * 2 + s.grp * 2 * split * 64;
                    float* mine = gred + ((k & 1u) * split + s.wig) * 64;
                    mine[lane] = v0;
                    mine[32 + lane] = v2;
                    named_barrier_sync(1 + static_cast<int>(s.grp), static_cast<int>(split) * 32);
                    writer = (k & (split - 1)) == s.wig;
                    if (writer) {
                        const float* base = gred + (k & 1u) * split * 64;
                        v0 = 0.f;
                        v2 = 0.f;
                        for (std::uint32_t w = 0; w < split; ++w) {
                            v0 += base[w * 64 + lane];
                            v2 += base[w * 64 + 32 + lane];
                        }
                    }
                }
                if (writer && t == 0) {
                    if (ph == 0 && tile < p.rope_tiles) {
                        const std::uint32_t per_head = p.head_dim / 16;
                        const std::uint32_t hd = tile / per_head;
                        const std::uint32_t j = (tile - hd * per_head) * 8 + g;
                        const std::uint32_t r1 = hd * p.head_dim + j;
                        float o1, o2;
                        rotate(v0, v2, L.cos[j], L.sin[j], o1, o2);
                        L.qkv[r1] = __float2half_rn(o1);
                        L.qkv[r1 + p.head_dim / 2] = __float2half_rn(o2);
                    } else if (ph == 0 && tile < p.qkv_tiles) {
                        const std::uint32_t r = p.rope_rows + (tile - p.rope_tiles) * 16u + g;
                        L.qkv[r] = __float2half_rn(v0);
                        L.qkv[r + 8] = __float2half_rn(v2);
                    } else if (ph == 0) {
                        const std::uint32_t r = (tile - p.qkv_tiles) * 16u + g;
                        L.h1[r] = __float2half_rn(v0 + __half2float(hres[r]));
                        L.h1[r + 8] = __float2half_rn(v2 + __half2float(hres[r + 8]));
                    } else if (ph == 1) {
                        const std::uint32_t f = tile * 8u + g;
                        L.a[f] = __float2half_rn(v0 / (1.0f + expf(-v0)) * v2);
                    } else if (p.down_parts == 1) {
                        const std::uint32_t r = tile * 16u + g;
                        L.out[r] = __float2half_rn(v0 + __half2float(__ldcg(L.h1 + r)));
                        L.out[r + 8] = __float2half_rn(v2 + __half2float(__ldcg(L.h1 + r + 8)));
                    } else {
                        // a K half: its partial sums, added by the next staging
                        const std::uint32_t r = tile / 2 * 16u + g;
                        float* dst = p.parts + ((l & 1u) * 2 + (tile & 1u)) * p.hidden;
                        dst[r] = v0;
                        dst[r + 8] = v2;
                    }
                }
            }
        }
    }
    // the last layer's `out` when its down projection ran in halves
    if (alive && p.down_parts == 2 && grid_barrier(p, passed, &s_flag)) {
        const std::uint32_t l = p.num_layers - 1;
        const Layer& P = p.layers[l];
        const float* pa = p.parts + (l & 1u) * 2 * p.hidden;
        const float* pb = pa + p.hidden;
        for (std::uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < p.hidden;
             i += gridDim.x * kThreads)
            P.out[i] = __float2half_rn((__ldcg(pa + i) + __ldcg(pb + i)) + __half2float(__ldcg(P.h1 + i)));
    }
    cp_async_wait<0>();
}

}  // namespace stack
}  // namespace mote

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
// Workspace bytes of mote_cuda_q4_0_decoder_stack_f16: 256 bytes of barrier
// words and the down projection's partial sums (2 x 2 x hidden f32).
extern "C" int mote_cuda_q4_0_decoder_stack_workspace_bytes(uint64_t hidden, uint64_t* bytes) {
    if (bytes == nullptr) return mote::kInvalidValue;
    *bytes = 256 + 16 * hidden;
    return mote::kSuccess;
}

// Runs the non-attention ops of num_layers decoder layers at one token (see
// the file comment; include/mote_cuda.h declares mote_cuda_stack_layer,
// which must match mote::stack::Layer).  layers: DEVICE array of
// num_layers descriptors; h_in [hidden] f16 is layer 0's input and layer
// l > 0 takes layer l-1's `out`.  workspace: the bytes
// mote_cuda_q4_0_decoder_stack_workspace_bytes gives (its first 256 are set
// to zero by this call before the launch).  hidden and ffn multiples of
// 256, head_dim a multiple of 16, q_heads a multiple of kv_heads, every
// tensor 16-byte aligned (cos/sin 4-byte); eps finite and >= 0.
// num_layers == 0 returns 0.  The launch is cooperative (all CTAs resident).
extern "C" int mote_cuda_q4_0_decoder_stack_f16(const void* layers, uint32_t num_layers,
                                                const void* h_in, uint64_t hidden, uint64_t ffn,
                                                uint64_t q_heads, uint64_t kv_heads,
                                                uint64_t head_dim, float epsilon, void* workspace,
                                                uint64_t workspace_bytes, void* stream) {
    using namespace mote;
    using namespace mote::stack;
    static_assert(sizeof(Layer) == 14 * sizeof(void*), "descriptor layout");
    if (layers == nullptr || h_in == nullptr || workspace == nullptr || stream == nullptr)
        return kInvalidValue;
    if (num_layers == 0) return kSuccess;
    if (hidden == 0 || hidden % 256 != 0 || ffn == 0 || ffn % 256 != 0 || head_dim == 0 ||
        head_dim % 16 != 0 || kv_heads == 0 || q_heads % kv_heads != 0 || hidden > (1u << 20) ||
        ffn > (1u << 20) || (q_heads + 2 * kv_heads) * head_dim > (1u << 22) ||
        !std::isfinite(epsilon) || epsilon < 0.0f)
        return kInvalidValue;
    if (reinterpret_cast<std::uintptr_t>(h_in) % 16 != 0 ||
        reinterpret_cast<std::uintptr_t>(layers) % 8 != 0 ||
        reinterpret_cast<std::uintptr_t>(workspace) % 256 != 0 ||
        workspace_bytes < 256 + 16 * hidden)
        return kInvalidValue;
    Params p{};
    p.layers = static_cast<const Layer*>(layers);
    p.num_layers = num_layers;
    p.h_in = static_cast<const __half*>(h_in);
    p.barrier = static_cast<unsigned*>(workspace);
    p.parts = reinterpret_cast<float*>(static_cast<std::uint8_t*>(workspace) + 256);
    p.eps = epsilon;
    p.hidden = static_cast<std::uint32_t>(hidden);
    p.ffn = static_cast<std::uint32_t>(ffn);
    p.head_dim = static_cast<std::uint32_t>(head_dim);
    p.rope_rows = static_cast<std::uint32_t>((q_heads + kv_heads) * head_dim);
    p.rope_tiles = p.rope_rows / 16;
    p.qkv_tiles = static_cast<std::uint32_t>((q_heads + 2 * kv_heads) * head_dim / 16);
    p.o_tiles = p.hidden / 16;
    p.gu_tiles = p.ffn / 8;
    p.down_tiles = p.hidden / 16;
    p.units_h = p.hidden / 256;
    p.units_f = p.ffn / 256;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    const std::uint32_t x_bytes_raw =
        max(2u * (2u * p.hidden + 32u), 2u * p.ffn + 32u);
    p.x_bytes = (x_bytes_raw + 127u) & ~127u;
    const int smem = static_cast<int>(p.x_bytes) + kZeroBytes + kWarps * kStages * kStageBytes +
                     kRedBytes + static_cast<int>(p.hidden) * 2;
    static std::atomic<std::uint64_t> done{0};
    int st = ensure_dynamic_smem(decoder_stack_kernel, smem, done);
    if (st != kSuccess) return st;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decoder_stack_kernel, kThreads, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm < 1) return static_cast<int>(cudaErrorInvalidConfiguration);
    const std::uint32_t grid = static_cast<std::uint32_t>(sms) * static_cast<std::uint32_t>(min(per_sm, 2));
    // the down projection in K halves when its tiles are fewer than the
    // CTAs' 8-warp groups can take twice over (and K splits evenly)
    p.down_parts = (p.units_f % 2 == 0 && p.down_tiles * 2 <= grid) ? 2u : 1u;
    // per phase: the widest warp split (at most 8 warps, at most the
    // phase's K units per tile) whose groups still cover the phase's tiles
    // in one round -- fewer units per warp, no second round
    const std::uint32_t tiles[3] = {p.qkv_tiles + p.o_tiles, p.gu_tiles,
                                    p.down_tiles * p.down_parts};
    const std::uint32_t units[3] = {p.units_h, p.units_h, p.units_f / p.down_parts};
    for (int ph = 0; ph < 3; ++ph) {
        std::uint32_t sh = 0;
        while (sh < 3 && (2u << sh) <= units[ph] && grid * (kWarps >> (sh + 1)) >= tiles[ph]) ++sh;
        p.sh[ph] = sh;
    }
    const auto s = static_cast<cudaStream_t>(stream);
    e = cudaMemsetAsync(workspace, 0, 256, s);
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = static_cast<std::size_t>(smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, decoder_stack_kernel, p));
}
