// Runtime shim: the narrow device/stream/memory surface of the C ABI.
//
// Mirrors the `hip` module of crates/mote-backend-hip/src/ffi.rs:14-118
// (get_device_count, set_device, malloc, free, synchronous H2D/D2H copies,
// stream create/destroy/synchronize, mem_get_info) so a Rust CudaContext /
// CudaStorage pair can be written exactly like HipContext / HipStorage.  A
// few asynchronous helpers are added for callers that manage their own
// pinned buffers and timing.  Every function returns the raw cudaError_t as
// an int (0 = success).

#include "mote_common.cuh"

extern "C" int mote_cuda_get_device_count(int* count) {
    if (count == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaGetDeviceCount(count));
}

extern "C" int mote_cuda_set_device(int ordinal) {
    return static_cast<int>(cudaSetDevice(ordinal));
}

extern "C" int mote_cuda_malloc(void** pointer, std::size_t bytes) {
    if (pointer == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaMalloc(pointer, bytes));
}

extern "C" int mote_cuda_free(void* pointer) { return static_cast<int>(cudaFree(pointer)); }

extern "C" int mote_cuda_memcpy_host_to_device(void* destination, const void* source,
                                               std::size_t bytes) {
    return static_cast<int>(cudaMemcpy(destination, source, bytes, cudaMemcpyHostToDevice));
}

extern "C" int mote_cuda_memcpy_device_to_host(void* destination, const void* source,
                                               std::size_t bytes) {
    return static_cast<int>(cudaMemcpy(destination, source, bytes, cudaMemcpyDeviceToHost));
}

extern "C" int mote_cuda_stream_create(void** stream) {
    if (stream == nullptr) return mote::kInvalidValue;
    cudaStream_t s = nullptr;
    const cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e == cudaSuccess) *stream = s;
    return static_cast<int>(e);
}

extern "C" int mote_cuda_stream_destroy(void* stream) {
    return static_cast<int>(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
}

extern "C" int mote_cuda_stream_synchronize(void* stream) {
    return static_cast<int>(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
}

extern "C" int mote_cuda_mem_get_info(std::size_t* free_bytes, std::size_t* total_bytes) {
    if (free_bytes == nullptr || total_bytes == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaMemGetInfo(free_bytes, total_bytes));
}

// ---- additions beyond the reference shim ----------------------------------

extern "C" int mote_cuda_memcpy_host_to_device_async(void* destination, const void* source,
                                                     std::size_t bytes, void* stream) {
    return static_cast<int>(cudaMemcpyAsync(destination, source, bytes, cudaMemcpyHostToDevice,
                                            static_cast<cudaStream_t>(stream)));
}

extern "C" int mote_cuda_memcpy_device_to_host_async(void* destination, const void* source,
                                                     std::size_t bytes, void* stream) {
    return static_cast<int>(cudaMemcpyAsync(destination, source, bytes, cudaMemcpyDeviceToHost,
                                            static_cast<cudaStream_t>(stream)));
}

extern "C" int mote_cuda_memset_async(void* destination, int value, std::size_t bytes,
                                      void* stream) {
    return static_cast<int>(
        cudaMemsetAsync(destination, value, bytes, static_cast<cudaStream_t>(stream)));
}

extern "C" int mote_cuda_host_alloc(void** pointer, std::size_t bytes) {
    if (pointer == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaHostAlloc(pointer, bytes, cudaHostAllocDefault));
}

extern "C" int mote_cuda_host_free(void* pointer) {
    return static_cast<int>(cudaFreeHost(pointer));
}

extern "C" int mote_cuda_event_create(void** event) {
    if (event == nullptr) return mote::kInvalidValue;
    cudaEvent_t e = nullptr;
    const cudaError_t st = cudaEventCreate(&e);
    if (st == cudaSuccess) *event = e;
    return static_cast<int>(st);
}

extern "C" int mote_cuda_event_destroy(void* event) {
    return static_cast<int>(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
}

extern "C" int mote_cuda_event_record(void* event, void* stream) {
    return static_cast<int>(
        cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
}

// `stream` waits (on the device) for the work recorded in `event`: the
// ordering between a context's compute stream and its copy stream.
extern "C" int mote_cuda_stream_wait_event(void* stream, void* event) {
    if (stream == nullptr || event == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream),
                                                static_cast<cudaEvent_t>(event), 0));
}

extern "C" int mote_cuda_event_elapsed_ms(float* ms, void* start, void* end) {
    if (ms == nullptr) return mote::kInvalidValue;
    return static_cast<int>(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start),
                                                 static_cast<cudaEvent_t>(end)));
}

// Reads (and optionally clears) the current device's status word, where
// kernels record bounded-wait timeouts (bit 0) and out-of-range indices
// (bit 1).  Synchronizes with the device.
extern "C" int mote_cuda_device_status(unsigned* status, int clear) {
    if (status == nullptr) return mote::kInvalidValue;
    cudaError_t e = cudaMemcpyFromSymbol(status, mote::g_device_status, sizeof(unsigned));
    if (e != cudaSuccess) return static_cast<int>(e);
    if (clear) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(mote::g_device_status, &zero, sizeof(unsigned));
    }
    return static_cast<int>(e);
}

extern "C" const char* mote_cuda_status_string(int status) {
    if (status == mote::kInternalError) return "mote: invalid argument (internal error -1)";
    if (status == 10000) return "mote: NCCL library (libnccl.so.2) could not be loaded";
    if (status == 10001)
        return "mote: NCCL deadline passed (not every rank joined or completed in time); the "
               "communicator was aborted";
    if (status == 10200)
        return "mote: the request's K split needs more than the 8 MiB static scratch of "
               "mote_cuda_quantized_linear_q4_0_f16_noalloc (use the _ws entry point)";
    if (status > 10100 && status < 10200) return "mote: NCCL call failed (status - 10100 = ncclResult_t)";
    return cudaGetErrorString(static_cast<cudaError_t>(status));
}

extern "C" int mote_cuda_abi_version(void) { return 1; }
