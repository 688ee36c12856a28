// Multi-GPU exchange for column-sharded linears (lm_head, FFN gate/up).
//
// Each rank owns a contiguous slice of the weight rows (output columns) and
// computes y_g [M, N/G]; the ranks then need every slice.  Two transports:
//
// * NCCL (loaded with dlopen on first use, so the library itself does not
//   depend on it): unique id / init / all-gather / destroy, mirroring the
//   NCCL calls one-to-one.  The gathered buffer is rank-major [G][count].
//
// * Peer stores over NVLink: every rank maps the other ranks' receive
//   buffers and flag words through CUDA IPC handles, and one kernel writes
//   its slice straight into all G receive buffers (16-byte stores), then
//   publishes an epoch in every peer's flag array (release, system scope)
//   and waits -- bounded -- until every peer's epoch has arrived in its own
//   array.  No library kernel ever reads peer memory, no load uses cluster
//   multicast, and no multicast object is created.
//
// Flag array of a rank (nranks + 2 words, zeroed once): [q] = last epoch
// published by rank q, [nranks] = CTA arrival counter, [nranks + 1] = this
// rank's own epoch counter.  The epoch advances on the device, so a launch
// captured in a CUDA graph synchronizes correctly on every replay.  A
// receive buffer must not be overwritten while any rank may still read the
// previous gather from it (alternate two buffers, or synchronize).
#include "mote_common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

namespace mote {
namespace comm {

// Above every CUDA runtime error code.
constexpr int kCommUnavailable = 10000;  // libnccl could not be loaded
constexpr int kCommErrorBase = 10100;    // + ncclResult_t

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    bool ok = false;
};

// The process's NCCL (an already loaded libnccl.so.2 -- e.g. the one a
// PyTorch process uses -- is found first), resolved once.
inline const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
        api.ok = api.get_unique_id && api.init_rank && api.all_gather && api.destroy;
    });
    return api;
}

inline int nccl_status(ncclResult_t r) {
    return r == ncclSuccess ? kSuccess : kCommErrorBase + static_cast<int>(r);
}

// ---------------------------------------------------------------------------
// Peer-store all-gather
// ---------------------------------------------------------------------------
struct GatherArgs {
    const uint4* send;            // this rank's slice, count16 vectors
    uint4* const* recv;           // [nranks] receive buffers (peer mappings), device array
    unsigned* const* flags;       // [nranks] flag arrays (peer mappings), device array
    unsigned* own_flags;          // this rank's flag array (nranks + 2 words)
    std::uint64_t count16;        // 16-byte vectors per rank
    std::uint32_t rank;
    std::uint32_t nranks;
};

// A strong relaxed store: after a system-scope fence by the same thread it
// completes a release pattern, and the stores to several ranks' flags can
// be in flight together (a st.release per flag would fence before each).
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) all_gather_p2p_kernel(const GatherArgs a) {
    const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * blockDim.x;
    const std::uint64_t base = static_cast<std::uint64_t>(a.rank) * a.count16;
    for (std::uint64_t i = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x;
         i < a.count16; i += stride) {
        const uint4 v = a.send[i];
        for (std::uint32_t p = 0; p < a.nranks; ++p) a.recv[p][base + i] = v;
    }
    // The CTA barrier orders every thread's stores before thread 0's
    // system-scope fence, which is cumulative: one fence per CTA publishes
    // the CTA's slice before its arrival is counted.
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const unsigned arrived = atomicAdd(&a.own_flags[a.nranks], 1u);
    if (arrived != gridDim.x - 1) return;
    // Last CTA of this rank: every slice store of the grid is fenced.
    a.own_flags[a.nranks] = 0u;  // counter ready for the next call
    const unsigned epoch = a.own_flags[a.nranks + 1] + 1u;
    a.own_flags[a.nranks + 1] = epoch;
    __threadfence_system();  // with the relaxed flag stores below: one release pattern
    for (std::uint32_t p = 0; p < a.nranks; ++p) st_relaxed_sys(a.flags[p] + a.rank, epoch);
    // Wait (bounded) for every rank's slice of this epoch.  A peer that has
    // already moved on to a later epoch also delivered this one.
    const long long start = clock64();
    for (std::uint32_t q = 0; q < a.nranks; ++q) {
        while (static_cast<int>(ld_acquire_sys(a.own_flags + q) - epoch) < 0) {
            if (clock64() - start > kWaitCycles) {
                atomicOr(&g_device_status, kDevWaitTimeout);
                return;
            }
        }
    }
}

}  // namespace comm
}  // namespace mote

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" int mote_cuda_comm_unique_id(void* id_out) {
    using namespace mote::comm;
    if (id_out == nullptr) return mote::kInvalidValue;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    ncclUniqueId id;
    const int st = nccl_status(api.get_unique_id(&id));
    if (st == mote::kSuccess) memcpy(id_out, &id, sizeof(id));
    return st;
}

extern "C" int mote_cuda_comm_init(void** comm, int nranks, const void* id, int rank) {
    using namespace mote::comm;
    if (comm == nullptr || id == nullptr || nranks < 1 || rank < 0 || rank >= nranks)
        return mote::kInvalidValue;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    const int st = nccl_status(api.init_rank(&c, nranks, uid, rank));
    *comm = st == mote::kSuccess ? static_cast<void*>(c) : nullptr;
    return st;
}

extern "C" int mote_cuda_comm_all_gather_f16(void* comm, const void* send, void* recv,
                                             std::uint64_t count, void* stream) {
    using namespace mote::comm;
    if (comm == nullptr || send == nullptr || recv == nullptr || stream == nullptr)
        return mote::kInvalidValue;
    if (count == 0) return mote::kSuccess;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    return nccl_status(api.all_gather(send, recv, count, ncclFloat16,
                                      static_cast<ncclComm_t>(comm),
                                      static_cast<cudaStream_t>(stream)));
}

extern "C" int mote_cuda_comm_destroy(void* comm) {
    using namespace mote::comm;
    if (comm == nullptr) return mote::kSuccess;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    return nccl_status(api.destroy(static_cast<ncclComm_t>(comm)));
}

extern "C" int mote_cuda_ipc_get_handle(const void* dev_ptr, void* handle_out) {
    if (dev_ptr == nullptr || handle_out == nullptr) return mote::kInvalidValue;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e == cudaSuccess) memcpy(handle_out, &h, sizeof(h));
    return static_cast<int>(e);
}

extern "C" int mote_cuda_ipc_open_handle(const void* handle, void** dev_ptr) {
    if (handle == nullptr || dev_ptr == nullptr) return mote::kInvalidValue;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return static_cast<int>(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int mote_cuda_ipc_close_handle(void* dev_ptr) {
    if (dev_ptr == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaIpcCloseMemHandle(dev_ptr));
}

extern "C" int mote_cuda_all_gather_p2p_f16(const void* send, void* const* recv_ptrs,
                                            unsigned* const* flag_ptrs, unsigned* own_flags,
                                            std::uint64_t count, std::uint32_t rank,
                                            std::uint32_t nranks, void* stream) {
    using namespace mote::comm;
    if (send == nullptr || recv_ptrs == nullptr || flag_ptrs == nullptr || own_flags == nullptr ||
        stream == nullptr || nranks == 0 || rank >= nranks)
        return mote::kInvalidValue;
    // 16-byte vectors: count f16 elements per rank must be a multiple of 8,
    // with 16-byte aligned buffers (checked for the local send buffer; the
    // receive buffers come from cudaMalloc through IPC).
    if (count % 8 != 0 || reinterpret_cast<std::uintptr_t>(send) % 16 != 0)
        return mote::kInvalidValue;
    GatherArgs a{};
    a.send = static_cast<const uint4*>(send);
    a.recv = reinterpret_cast<uint4* const*>(recv_ptrs);
    a.flags = flag_ptrs;
    a.own_flags = own_flags;
    a.count16 = count / 8;
    a.rank = rank;
    a.nranks = nranks;
    // Enough CTAs to keep NVLink busy; every CTA reaches the arrival counter.
    std::uint64_t ctas = (a.count16 + 255) / 256;
    if (ctas > 264) ctas = 264;
    if (ctas == 0) ctas = 1;
    all_gather_p2p_kernel<<<static_cast<unsigned>(ctas), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return static_cast<int>(cudaGetLastError());
}
