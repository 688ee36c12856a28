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
//
// Failure handling (the reference has only status codes,
// crates/mote-backend-hip/src/error.rs:125-131):
// * the NCCL communicator can be created nonblocking with a deadline: the
//   init is polled and, if the other ranks have not all joined in time,
//   aborted (status kCommTimeout) instead of blocking the host for good;
// * every flag wait is bounded by a limit in nanoseconds of %globaltimer
//   (1 s by default, or the caller's): on expiry the wait records
//   kDevWaitTimeout in the device status word and returns, leaving the
//   context usable;
// * after an expiry the ranks' epochs may be out of step; with no exchange
//   in flight anywhere, every rank zeroes its own flag array
//   (mote_cuda_peer_flags_reset) between two host barriers, and the epochs
//   restart together.
#include "mote_common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <memory>
#include <mutex>
#include <thread>

namespace mote {
namespace comm {

// Above every CUDA runtime error code.
constexpr int kCommUnavailable = 10000;  // libnccl could not be loaded
constexpr int kCommTimeout = 10001;      // deadline passed; the communicator was aborted
constexpr int kCommErrorBase = 10100;    // + ncclResult_t

// Default limit of one peer flag wait.
constexpr std::uint64_t kDefaultWaitNs = 1000000000ull;

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    bool ok = false;
    bool nonblocking_ok = false;  // the calls a deadline needs
};

// The handle behind the ABI's `void* comm`.
struct Comm {
    ncclComm_t nccl = nullptr;
    bool nonblocking = false;
    std::uint64_t timeout_ms = 0;  // nonblocking: limit of every poll
    bool aborted = false;
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
        api.init_rank_config = reinterpret_cast<decltype(api.init_rank_config)>(
            dlsym(h, "ncclCommInitRankConfig"));
        api.get_async_error = reinterpret_cast<decltype(api.get_async_error)>(
            dlsym(h, "ncclCommGetAsyncError"));
        api.abort = reinterpret_cast<decltype(api.abort)>(dlsym(h, "ncclCommAbort"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
        api.ok = api.get_unique_id && api.init_rank && api.all_gather && api.destroy;
        api.nonblocking_ok = api.ok && api.init_rank_config && api.get_async_error && api.abort;
    });
    return api;
}

inline int nccl_status(ncclResult_t r) {
    return r == ncclSuccess ? kSuccess : kCommErrorBase + static_cast<int>(r);
}

// Polls a nonblocking communicator until its pending operation is done.
// Returns the operation's result, or ncclInProgress if `timeout_ms` passed.
inline ncclResult_t poll_until_done(const NcclApi& api, ncclComm_t c, std::uint64_t timeout_ms) {
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t state = ncclInProgress;
        const ncclResult_t r = api.get_async_error(c, &state);
        if (r != ncclSuccess) return r;
        if (state != ncclInProgress) return state;
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - start)
                            .count();
        if (static_cast<std::uint64_t>(ms) >= timeout_ms) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// Result of a nonblocking call: waits (bounded) if it is still in progress;
// past the deadline the communicator is aborted and kCommTimeout returned.
inline int finish_nonblocking(const NcclApi& api, Comm* c, ncclResult_t r) {
    if (r == ncclInProgress) r = poll_until_done(api, c->nccl, c->timeout_ms);
    if (r == ncclInProgress) {
        api.abort(c->nccl);
        c->aborted = true;
        return kCommTimeout;
    }
    return nccl_status(r);
}

__device__ __forceinline__ std::uint64_t global_ns() {
    std::uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
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
    std::uint64_t wait_ns;        // limit of the flag wait
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
    const std::uint64_t start = global_ns();
    for (std::uint32_t q = 0; q < a.nranks; ++q) {
        while (static_cast<int>(ld_acquire_sys(a.own_flags + q) - epoch) < 0) {
            if (global_ns() - start > a.wait_ns) {
                atomicOr(&g_device_status, kDevWaitTimeout);
                return;
            }
        }
    }
}

inline int launch_all_gather_p2p(const void* send, void* const* recv_ptrs,
                                 unsigned* const* flag_ptrs, unsigned* own_flags,
                                 std::uint64_t count, std::uint32_t rank, std::uint32_t nranks,
                                 std::uint64_t wait_ns, void* stream) {
    if (send == nullptr || recv_ptrs == nullptr || flag_ptrs == nullptr || own_flags == nullptr ||
        stream == nullptr || nranks == 0 || rank >= nranks || wait_ns == 0)
        return kInvalidValue;
    // 16-byte vectors: count f16 elements per rank must be a multiple of 8,
    // with 16-byte aligned buffers (checked for the local send buffer; the
    // receive buffers come from cudaMalloc through IPC).
    if (count % 8 != 0 || reinterpret_cast<std::uintptr_t>(send) % 16 != 0)
        return kInvalidValue;
    GatherArgs a{};
    a.send = static_cast<const uint4*>(send);
    a.recv = reinterpret_cast<uint4* const*>(recv_ptrs);
    a.flags = flag_ptrs;
    a.own_flags = own_flags;
    a.count16 = count / 8;
    a.rank = rank;
    a.nranks = nranks;
    a.wait_ns = wait_ns;
    // Enough CTAs to keep NVLink busy; every CTA reaches the arrival counter.
    std::uint64_t ctas = (a.count16 + 255) / 256;
    if (ctas > 264) ctas = 264;
    if (ctas == 0) ctas = 1;
    all_gather_p2p_kernel<<<static_cast<unsigned>(ctas), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return static_cast<int>(cudaGetLastError());
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
    *comm = nullptr;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    const int st = nccl_status(api.init_rank(&c, nranks, uid, rank));
    if (st != mote::kSuccess) return st;
    *comm = new Comm{c, false, 0, false};
    return st;
}

// Nonblocking init with a deadline: if not every rank has joined within
// timeout_ms, the communicator is aborted and kCommTimeout returned (*comm
// stays null).  The communicator stays nonblocking: its later calls are
// polled against the same limit.
extern "C" int mote_cuda_comm_init_timeout(void** comm, int nranks, const void* id, int rank,
                                           std::uint64_t timeout_ms) {
    using namespace mote::comm;
    if (comm == nullptr || id == nullptr || nranks < 1 || rank < 0 || rank >= nranks ||
        timeout_ms == 0)
        return mote::kInvalidValue;
    *comm = nullptr;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    if (!api.nonblocking_ok) return kCommErrorBase + static_cast<int>(ncclInvalidUsage);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    auto c = std::make_unique<Comm>();
    c->nonblocking = true;
    c->timeout_ms = timeout_ms;
    const ncclResult_t r = api.init_rank_config(&c->nccl, nranks, uid, rank, &config);
    if (c->nccl == nullptr) return nccl_status(r == ncclSuccess ? ncclInternalError : r);
    const int st = finish_nonblocking(api, c.get(), r);
    if (st != mote::kSuccess) {
        if (!c->aborted) api.abort(c->nccl);
        return st;
    }
    *comm = c.release();
    return mote::kSuccess;
}

extern "C" int mote_cuda_comm_all_gather_f16(void* comm, const void* send, void* recv,
                                             std::uint64_t count, void* stream) {
    using namespace mote::comm;
    if (comm == nullptr || send == nullptr || recv == nullptr || stream == nullptr)
        return mote::kInvalidValue;
    auto* c = static_cast<Comm*>(comm);
    if (c->aborted) return kCommErrorBase + static_cast<int>(ncclInvalidUsage);
    if (count == 0) return mote::kSuccess;
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    const ncclResult_t r = api.all_gather(send, recv, count, ncclFloat16, c->nccl,
                                          static_cast<cudaStream_t>(stream));
    if (c->nonblocking) return finish_nonblocking(api, c, r);
    return nccl_status(r);
}

extern "C" int mote_cuda_comm_destroy(void* comm) {
    using namespace mote::comm;
    if (comm == nullptr) return mote::kSuccess;
    std::unique_ptr<Comm> c(static_cast<Comm*>(comm));
    if (c->aborted) return mote::kSuccess;  // the abort released it
    const NcclApi& api = nccl();
    if (!api.ok) return kCommUnavailable;
    // A nonblocking communicator is released with the NCCL abort, which
    // returns without waiting on the other ranks (callers synchronise their
    // streams before destroying, as for any communicator).
    if (c->nonblocking) return nccl_status(api.abort(c->nccl));
    return nccl_status(api.destroy(c->nccl));
}

// Aborts the communicator's pending and future operations and frees it
// (the NCCL abort: no barrier with the other ranks).
extern "C" int mote_cuda_comm_abort(void* comm) {
    using namespace mote::comm;
    if (comm == nullptr) return mote::kSuccess;
    std::unique_ptr<Comm> c(static_cast<Comm*>(comm));
    if (c->aborted) return mote::kSuccess;
    const NcclApi& api = nccl();
    if (!api.ok || api.abort == nullptr) return kCommUnavailable;
    return nccl_status(api.abort(c->nccl));
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
    return mote::comm::launch_all_gather_p2p(send, recv_ptrs, flag_ptrs, own_flags, count, rank,
                                             nranks, mote::comm::kDefaultWaitNs, stream);
}

// The same all-gather with the flag wait limited to wait_ns nanoseconds.
extern "C" int mote_cuda_all_gather_p2p_f16_timeout(const void* send, void* const* recv_ptrs,
                                                    unsigned* const* flag_ptrs,
                                                    unsigned* own_flags, std::uint64_t count,
                                                    std::uint32_t rank, std::uint32_t nranks,
                                                    std::uint64_t wait_ns, void* stream) {
    return mote::comm::launch_all_gather_p2p(send, recv_ptrs, flag_ptrs, own_flags, count, rank,
                                             nranks, wait_ns, stream);
}

// Zeroes a rank's flag array (epochs and arrival counter) on `stream`: the
// resynchronisation after a wait expired.  No exchange may be in flight on
// any rank; every rank calls it between two host barriers.
extern "C" int mote_cuda_peer_flags_reset(unsigned* own_flags, std::uint32_t nranks,
                                          void* stream) {
    if (own_flags == nullptr || nranks == 0 || stream == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaMemsetAsync(own_flags, 0, (nranks + 2ull) * sizeof(unsigned),
                                            static_cast<cudaStream_t>(stream)));
}
