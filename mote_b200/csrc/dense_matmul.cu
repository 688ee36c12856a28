// Dense row-major f16 x f16 -> f32 matmul through cuBLASLt: the CUDA
// counterpart of the HIP backend's hipBLASLt shim
// (crates/mote-backend-hip/src/hipblaslt_shim.cpp:326-408) and of its Rust
// wrapper matmul_f16_f32 (crates/mote-backend-hip/src/matmul.rs:11-53).  A
// plain library GEMM (no quantized weights): it keeps the reference's
// interface and behaviour --
// * an opaque context (handle, per-shape plans, the last error message);
// * row-major tensors: C^T = B^T A^T is evaluated on the column-major
//   library, so no transposes are needed;
// * f32 compute and output;
// * the first call for a new (M, N, K) asks the library's heuristic for up
//   to 8 algorithms that fit the caller's workspace, times each once on the
//   caller's stream and keeps the fastest; later calls only enqueue it.
//   The first call of a shape therefore synchronizes its stream and must
//   come before any stream capture;
// * null pointers (stream and workspace included) return -1 with a message;
//   library errors return the cuBLAS status; CUDA errors -1000 - code.
// cuBLASLt is loaded with dlopen on first use (the process's own copy when
// one is loaded, e.g. PyTorch's), so the library does not link it.

#include <cublasLt.h>
#include <dlfcn.h>

#include <array>
#include <limits>
#include <map>
#include <memory>
#include <mutex>
#include <string>

namespace mote {
namespace blaslt {

constexpr int kHeuristicCount = 8;

struct Api {
    decltype(&cublasLtCreate) create = nullptr;
    decltype(&cublasLtDestroy) destroy = nullptr;
    decltype(&cublasLtMatmulDescCreate) desc_create = nullptr;
    decltype(&cublasLtMatmulDescDestroy) desc_destroy = nullptr;
    decltype(&cublasLtMatrixLayoutCreate) layout_create = nullptr;
    decltype(&cublasLtMatrixLayoutDestroy) layout_destroy = nullptr;
    decltype(&cublasLtMatmulPreferenceCreate) pref_create = nullptr;
    decltype(&cublasLtMatmulPreferenceSetAttribute) pref_set = nullptr;
    decltype(&cublasLtMatmulPreferenceDestroy) pref_destroy = nullptr;
    decltype(&cublasLtMatmulAlgoGetHeuristic) heuristic = nullptr;
    decltype(&cublasLtMatmul) matmul = nullptr;
    bool ok = false;
};

inline const Api& api() {
    static Api a;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libcublasLt.so.12", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) h = dlopen("/usr/local/cuda/lib64/libcublasLt.so.12", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) h = dlopen("libcublasLt.so", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) return;
#define MOTE_LT(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, #name))
        MOTE_LT(create, cublasLtCreate);
        MOTE_LT(destroy, cublasLtDestroy);
        MOTE_LT(desc_create, cublasLtMatmulDescCreate);
        MOTE_LT(desc_destroy, cublasLtMatmulDescDestroy);
        MOTE_LT(layout_create, cublasLtMatrixLayoutCreate);
        MOTE_LT(layout_destroy, cublasLtMatrixLayoutDestroy);
        MOTE_LT(pref_create, cublasLtMatmulPreferenceCreate);
        MOTE_LT(pref_set, cublasLtMatmulPreferenceSetAttribute);
        MOTE_LT(pref_destroy, cublasLtMatmulPreferenceDestroy);
        MOTE_LT(heuristic, cublasLtMatmulAlgoGetHeuristic);
        MOTE_LT(matmul, cublasLtMatmul);
#undef MOTE_LT
        a.ok = a.create && a.destroy && a.desc_create && a.desc_destroy && a.layout_create &&
               a.layout_destroy && a.pref_create && a.pref_set && a.pref_destroy && a.heuristic &&
               a.matmul;
    });
    return a;
}

struct Plan {
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t rhs = nullptr, lhs = nullptr, out = nullptr;
    cublasLtMatmulAlgo_t algo{};
    std::size_t ws_need = 0;  // workspace the chosen algorithm needs
    ~Plan() {
        const Api& a = api();
        if (rhs) a.layout_destroy(rhs);
        if (lhs) a.layout_destroy(lhs);
        if (out) a.layout_destroy(out);
        if (op) a.desc_destroy(op);
    }
};

struct Context {
    cublasLtHandle_t handle = nullptr;
    // plans per (m, n, k, pointer alignment); a plan tuned under a larger
    // workspace limit than a later call offers is tuned again
    std::map<std::array<std::uint64_t, 4>, std::unique_ptr<Plan>> plans;
    std::string last_error;
    ~Context() {
        plans.clear();
        if (handle) api().destroy(handle);
    }
};

inline int fail(Context* c, int status, std::string message) {
    if (c != nullptr) c->last_error = std::move(message);
    return status == 0 ? kInternalError : status;
}
inline int fail_cuda(Context* c, cudaError_t e, const char* what) {
    return fail(c, -1000 - static_cast<int>(e),
                std::string(what) + " failed: " + cudaGetErrorString(e));
}

// D (n x m, column-major) = rhs (n x k) * lhs (k x m): row-major C = A B.
inline cublasStatus_t enqueue(const Context& c, const Plan& plan, const void* lhs, const void* rhs,
                              void* out, void* ws, std::size_t ws_bytes, cudaStream_t s) {
    const float alpha = 1.0f, beta = 0.0f;
    return api().matmul(c.handle, plan.op, &alpha, rhs, plan.rhs, lhs, plan.lhs, &beta, out,
                        plan.out, out, plan.out, &plan.algo, ws, ws_bytes, s);
}

// Largest power of two (at most 256) dividing every operand address.
inline std::uint64_t operand_alignment(const void* lhs, const void* rhs, const void* out) {
    const std::uintptr_t bits = reinterpret_cast<std::uintptr_t>(lhs) |
                                reinterpret_cast<std::uintptr_t>(rhs) |
                                reinterpret_cast<std::uintptr_t>(out) | 256u;
    return static_cast<std::uint64_t>(bits & (~bits + 1));
}

inline int make_plan(Context* c, std::uint64_t m, std::uint64_t n, std::uint64_t k,
                     const void* lhs, const void* rhs, void* out, void* ws, std::size_t ws_bytes,
                     cudaStream_t s, std::unique_ptr<Plan>& result) {
    const Api& a = api();
    auto plan = std::make_unique<Plan>();
    cublasStatus_t st = a.desc_create(&plan->op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
    if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatmulDescCreate failed");
    st = a.layout_create(&plan->rhs, CUDA_R_16F, n, k, static_cast<std::int64_t>(n));
    if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatrixLayoutCreate(rhs) failed");
    st = a.layout_create(&plan->lhs, CUDA_R_16F, k, m, static_cast<std::int64_t>(k));
    if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatrixLayoutCreate(lhs) failed");
    st = a.layout_create(&plan->out, CUDA_R_32F, n, m, static_cast<std::int64_t>(n));
    if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatrixLayoutCreate(output) failed");
    cublasLtMatmulPreference_t pref = nullptr;
    st = a.pref_create(&pref);
    if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatmulPreferenceCreate failed");
    const std::uint64_t limit = ws_bytes;
    st = a.pref_set(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &limit, sizeof(limit));
    // only algorithms valid for these operands' alignment
    const std::uint32_t align = static_cast<std::uint32_t>(operand_alignment(lhs, rhs, out));
    for (const auto attr : {CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_A_BYTES,
                            CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_B_BYTES,
                            CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_C_BYTES,
                            CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_D_BYTES})
        if (st == CUBLAS_STATUS_SUCCESS) st = a.pref_set(pref, attr, &align, sizeof(align));
    if (st != CUBLAS_STATUS_SUCCESS) {
        a.pref_destroy(pref);
        return fail(c, st, "cublasLtMatmulPreferenceSetAttribute failed");
    }
    std::array<cublasLtMatmulHeuristicResult_t, kHeuristicCount> cand{};
    int count = 0;
    st = a.heuristic(c->handle, plan->op, plan->rhs, plan->lhs, plan->out, plan->out, pref,
                     kHeuristicCount, cand.data(), &count);
    a.pref_destroy(pref);
    if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatmulAlgoGetHeuristic failed");
    if (count == 0) return fail(c, kInternalError, "cuBLASLt returned no algorithms");

    // time each candidate once (after one untimed launch) and keep the fastest
    cudaEvent_t start = nullptr, stop = nullptr;
    cudaError_t e = cudaEventCreate(&start);
    if (e != cudaSuccess) return fail_cuda(c, e, "cudaEventCreate(tuning start)");
    e = cudaEventCreate(&stop);
    if (e != cudaSuccess) {
        cudaEventDestroy(start);
        return fail_cuda(c, e, "cudaEventCreate(tuning stop)");
    }
    float best = std::numeric_limits<float>::infinity();
    bool found = false;
    cublasLtMatmulAlgo_t best_algo{};
    std::size_t best_ws = 0;
    for (int i = 0; i < count; ++i) {
        if (cand[i].state != CUBLAS_STATUS_SUCCESS || cand[i].workspaceSize > ws_bytes) continue;
        plan->algo = cand[i].algo;
        if (enqueue(*c, *plan, lhs, rhs, out, ws, ws_bytes, s) != CUBLAS_STATUS_SUCCESS) continue;
        if (cudaEventRecord(start, s) != cudaSuccess) continue;
        if (enqueue(*c, *plan, lhs, rhs, out, ws, ws_bytes, s) != CUBLAS_STATUS_SUCCESS) continue;
        if (cudaEventRecord(stop, s) != cudaSuccess) continue;
        if (cudaEventSynchronize(stop) != cudaSuccess) continue;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, start, stop) != cudaSuccess) continue;
        if (ms < best) {
            best = ms;
            best_algo = cand[i].algo;
            best_ws = cand[i].workspaceSize;
            found = true;
        }
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    if (!found) return fail(c, kInternalError, "no cuBLASLt algorithm ran for this shape");
    plan->algo = best_algo;
    plan->ws_need = best_ws;
    result = std::move(plan);
    return 0;
}

}  // namespace blaslt
}  // namespace mote

// mote_hipblaslt_create (hipblaslt_shim.cpp:326-341): a new context in
// *output; -1 for a null output, the library status if it fails to start.
extern "C" int mote_cuda_blaslt_create(void** output) {
    using namespace mote::blaslt;
    using mote::kInternalError;
    if (output == nullptr) return kInternalError;
    if (!api().ok) return kInternalError;
    try {
        auto c = std::make_unique<Context>();
        const cublasStatus_t st = api().create(&c->handle);
        if (st != CUBLAS_STATUS_SUCCESS) return static_cast<int>(st);
        *output = c.release();
        return 0;
    } catch (...) {
        return kInternalError;
    }
}

// mote_hipblaslt_destroy (:343-345); null is a no-op.
extern "C" void mote_cuda_blaslt_destroy(void* opaque) {
    delete static_cast<mote::blaslt::Context*>(opaque);
}

// mote_hipblaslt_last_error (:347-350): the message of the context's last
// failed call ("" after a success), null for a null context.
extern "C" const char* mote_cuda_blaslt_last_error(void* opaque) {
    const auto* c = static_cast<const mote::blaslt::Context*>(opaque);
    return c == nullptr ? nullptr : c->last_error.c_str();
}

// mote_hipblaslt_matmul_f16_f32 (:352-408): output[m, n] (f32) = lhs[m, k]
// (f16) x rhs[k, n] (f16), row-major, f32 accumulation, on `stream`, with
// `workspace_bytes` of caller workspace.  m == 0 or n == 0 succeeds without
// a launch; k == 0 writes zeros.
extern "C" int mote_cuda_blaslt_matmul_f16_f32(void* opaque, std::uint64_t m, std::uint64_t n,
                                               std::uint64_t k, const void* lhs, const void* rhs,
                                               void* output, void* workspace,
                                               std::size_t workspace_bytes, void* stream) {
    using namespace mote::blaslt;
    using mote::kInternalError;
    auto* c = static_cast<Context*>(opaque);
    if (c == nullptr || lhs == nullptr || rhs == nullptr || output == nullptr ||
        workspace == nullptr || stream == nullptr)
        return fail(c, kInternalError, "cuBLASLt matmul received a null handle");
    const auto s = static_cast<cudaStream_t>(stream);
    if (m == 0 || n == 0) {
        c->last_error.clear();
        return 0;
    }
    if (k == 0) {
        const cudaError_t e = cudaMemsetAsync(output, 0, m * n * sizeof(float), s);
        if (e != cudaSuccess) return fail_cuda(c, e, "cudaMemsetAsync");
        c->last_error.clear();
        return 0;
    }
    try {
        const std::array<std::uint64_t, 4> key{m, n, k, operand_alignment(lhs, rhs, output)};
        auto it = c->plans.find(key);
        if (it == c->plans.end() || it->second->ws_need > workspace_bytes) {
            // new shape, or a plan that needs more workspace than this call has
            std::unique_ptr<Plan> plan;
            const int st = make_plan(c, m, n, k, lhs, rhs, output, workspace, workspace_bytes, s,
                                     plan);
            if (st != 0) return st;
            if (it == c->plans.end())
                it = c->plans.emplace(key, std::move(plan)).first;
            else
                it->second = std::move(plan);
        }
        const cublasStatus_t st =
            enqueue(*c, *it->second, lhs, rhs, output, workspace, workspace_bytes, s);
        if (st != CUBLAS_STATUS_SUCCESS) return fail(c, st, "cublasLtMatmul failed");
        c->last_error.clear();
        return 0;
    } catch (const std::exception& err) {
        return fail(c, kInternalError, err.what());
    } catch (...) {
        return fail(c, kInternalError, "unknown C++ exception");
    }
}
