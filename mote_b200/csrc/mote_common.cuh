// Shared device helpers for the Mote CUDA data plane (sm_100a).
//
// Inline PTX wrappers for the Blackwell/Hopper asynchronous machinery the
// kernels use: mbarriers, 1-D bulk copies (global -> shared, no multicast),
// warp-level mma.sync, and bounded waits.  Every wait in this library has an
// iteration/time limit; on expiry it records an error code in a per-device
// status word that the host reads with mote_cuda_device_status(), and the
// kernel returns instead of spinning forever.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace mote {

// Status codes shared by every entry point.  Success is 0; the reference HIP
// shims return hipErrorInvalidValue (1), hipErrorInvalidConfiguration (9) or
// a private -1 ("kInternalError"), and the CUDA runtime uses the same numeric
// values for cudaErrorInvalidValue / cudaErrorInvalidConfiguration.
constexpr int kSuccess = 0;
constexpr int kInternalError = -1;
constexpr int kInvalidValue = static_cast<int>(cudaErrorInvalidValue);                    // 1
constexpr int kInvalidConfiguration = static_cast<int>(cudaErrorInvalidConfiguration);    // 9

// Device-side error codes recorded in g_device_status.
constexpr unsigned kDevWaitTimeout = 1u;
constexpr unsigned kDevIndexOutOfRange = 2u;

constexpr std::uint64_t kMaxGridX = 0xffffffffULL;

// Cycle budget for one bounded wait (~1 s at 2 GHz).
constexpr long long kWaitCycles = 2000000000LL;

__device__ __forceinline__ std::uint32_t smem_u32(const void* p) {
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(std::uint64_t* bar, std::uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(std::uint64_t* bar, std::uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(std::uint64_t* bar, std::uint32_t parity) {
    std::uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking: whether the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_test_wait(std::uint64_t* bar, std::uint32_t parity) {
    std::uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and
// records kDevWaitTimeout in *status) if it has not completed within
// kWaitCycles.
__device__ __forceinline__ bool mbar_wait_bounded(std::uint64_t* bar, std::uint32_t parity,
                                                  unsigned* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > kWaitCycles) {
            if (status) atomicOr(status, kDevWaitTimeout);
            return false;
        }
    }
    return true;
}

// ---- bulk copy (TMA engine, untiled, no multicast) -------------------------
// Copies `bytes` (multiple of 16) from 16-byte aligned global memory to
// 16-byte aligned shared memory and signals completion on `bar` via
// complete_tx.  The L2 policy marks the streamed bytes evict-first so a
// stream of weights does not push activations out of L2.
__device__ __forceinline__ std::uint64_t l2_evict_first_policy() {
    std::uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst_smem, const void* src_gmem,
                                              std::uint32_t bytes, std::uint64_t* bar,
                                              std::uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Same copy with the default L2 policy (for data many CTAs re-read).
__device__ __forceinline__ void bulk_copy_g2s_default(void* dst_smem, const void* src_gmem,
                                                      std::uint32_t bytes, std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- per-thread async copies (cp.async, 16 bytes, bypassing L1) ----------
__device__ __forceinline__ void cp_async_16(std::uint32_t dst_smem, const void* src_gmem,
                                            std::uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst_smem),
                 "l"(src_gmem), "l"(policy)
                 : "memory");
}

// Same copy with the default L2 policy (small tables many CTAs re-read).
__device__ __forceinline__ void cp_async_16_default(std::uint32_t dst_smem, const void* src_gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src_gmem)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's committed groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- programmatic dependent launch ------------------------------------------
// launch_dependents lets the next kernel in the stream (launched with the
// programmatic-serialization attribute) start its independent prologue;
// wait blocks until every prerequisite grid has completed and its memory is
// visible.  Both are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- warp MMA --------------------------------------------------------------
// D = A(16x16, f16, row) * B(16x8, f16, col) + C, f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], std::uint32_t a0, std::uint32_t a1,
                                          std::uint32_t a2, std::uint32_t a3, std::uint32_t b0,
                                          std::uint32_t b1, const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

// Shared-memory loads at a 32-bit shared address (register + immediate).
// volatile keeps them after the mbarrier wait that publishes the data.
__device__ __forceinline__ std::uint32_t lds32(std::uint32_t addr) {
    std::uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// Shared loads at base + a compile-time byte offset: the offset goes into
// the instruction's immediate field instead of a separate address add.
template <int OFF>
__device__ __forceinline__ std::uint32_t lds32i(std::uint32_t base) {
    std::uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(base), "n"(OFF));
    return v;
}

template <int OFF>
__device__ __forceinline__ uint2 lds64i(std::uint32_t base) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(base), "n"(OFF));
    return v;
}

template <int OFF>
__device__ __forceinline__ std::uint32_t lds16i(std::uint32_t base) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1+%2];" : "=h"(v) : "r"(base), "n"(OFF));
    return v;
}

__device__ __forceinline__ std::uint32_t lds16(std::uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint2 lds64(std::uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// (a & b) | c in one LOP3.
__device__ __forceinline__ std::uint32_t and_or(std::uint32_t a, std::uint32_t b,
                                                std::uint32_t c) {
    std::uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ std::uint32_t prmt(std::uint32_t a, std::uint32_t b,
                                              std::uint32_t sel) {
    std::uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ std::uint32_t hsub2_u32(std::uint32_t a, std::uint32_t b) {
    std::uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ float half_bits_to_float(std::uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// Per-device status word (error codes from bounded waits / index checks).
// The library is compiled as one translation unit (libmote_cuda.cu includes
// every component), so this definition is unique.
// RMSNorm and RoPE arithmetic in mote-reference's operation order
// (crates/mote-reference/src/lib.rs:289-299 and 170-244), correctly rounded
// f32 steps, shared by the layer kernels and the GEMV prologue/epilogue.
__device__ __forceinline__ float inv_rms(float sum_sq, std::uint64_t hidden, float eps) {
    const float mean_square = __fdiv_rn(sum_sq, static_cast<float>(hidden));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean_square, eps)));
}

__device__ __forceinline__ float norm_out(float x, float inv, float w) {
    return __fmul_rn(__fmul_rn(x, inv), w);
}

__device__ __forceinline__ void rotate(float a, float b, float c, float s, float& o1,
                                       float& o2) {
    o1 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    o2 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

__device__ unsigned g_device_status = 0;

// Launches `kernel` with programmatic dependent launch allowed: it may be
// scheduled while its predecessor in the stream drains.  Every such kernel
// calls pdl_wait() before it reads or writes memory the predecessor may
// touch (the wait returns once the predecessor grid has completed and its
// writes are visible), and pdl_launch_dependents() to let its own successor
// be scheduled early.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                      Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// launch_pdl with dynamic shared memory.
template <typename... KArgs, typename... Args>
inline int launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, int smem_bytes,
                           cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = static_cast<std::size_t>(smem_bytes);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// Opts a kernel into `bytes` of dynamic shared memory on the current device,
// once per ordinal below 64 (`done` is the bit mask), every call above.
template <typename Kernel>
inline int ensure_dynamic_smem(Kernel kernel, int bytes, std::atomic<std::uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    const std::uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return kSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    done.fetch_or(bit, std::memory_order_acq_rel);
    return kSuccess;
}

}  // namespace mote

#define MOTE_RETURN_IF_LAUNCH_FAILED() return static_cast<int>(cudaGetLastError())
