// cuBLAS backend — the engine's reference and the performance yardstick.
//
// Registered at priority 0 so the engine uses it as the reference
// (csrc/cublas_backends.cu:12-44 of VibeGEMM). The reference selects the operand
// order per target (:24-31); the B200 build uses the row-major-C order of its A100
// branch (:28-31): C^T = B^T·A in column-major terms, i.e.
//   cublasGemmEx(T, N, N, M, K, B, K, A, K, C, N), fp16 in/out, CUBLAS_COMPUTE_32F.
// Failures are reported instead of terminating the process (the reference exits),
// because this backend also lives inside a shared library loaded by test runners.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "backend.cuh"
#include "registry.cuh"
#include "utils.cuh"
#include "vibegemm_b200.h"

#if !defined(HAS_B200) && !defined(HAS_H100) && !defined(HAS_A100)
#error "Define one of HAS_B200, HAS_H100, HAS_A100"
#endif

namespace {

cublasStatus_t gemm_ex(cublasHandle_t h, const half *A, const half *B, half *C, int M, int N,
                       int K) {
    const float alpha = 1.f, beta = 0.f;
#if defined(HAS_H100) && !defined(HAS_B200)
    // Column-major C (the H100 family's layout).
    return cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, M, N, K, &alpha, A, CUDA_R_16F, K, B, CUDA_R_16F,
                        K, &beta, C, CUDA_R_16F, M, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
#else
    // Row-major C (A100 and B200 families).
    return cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &alpha, B, CUDA_R_16F, K, A, CUDA_R_16F,
                        K, &beta, C, CUDA_R_16F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
#endif
}

} // namespace

class CublasBackend : public GemmBackend {
  public:
    CublasBackend() {
        if (cublasCreate(&handle_) != CUBLAS_STATUS_SUCCESS) {
            std::fprintf(stderr, "cuBLAS: cublasCreate failed; backend unavailable\n");
            handle_ = nullptr;
        }
    }
    ~CublasBackend() override {
        if (handle_)
            cublasDestroy(handle_);
    }

    void run(half *A, half *B, half *C, int M, int N, int K) override {
        if (!handle_)
            return;
        const cublasStatus_t s = gemm_ex(handle_, A, B, C, M, N, K);
        if (s != CUBLAS_STATUS_SUCCESS)
            std::fprintf(stderr, "cuBLAS error: cublasGemmEx status=%d\n", (int)s);
    }

    std::string name() const override { return "cuBLAS"; }
    void teardown() override {}
    bool is_available() const override { return handle_ != nullptr; }

  private:
    cublasHandle_t handle_ = nullptr;
};

REGISTER_CUBLAS("cuBLAS", CublasBackend);

// C ABI: one cuBLAS handle per (thread, device), stream set per call.
// Returns 0, a cudaError_t code, or 1000 + cublasStatus_t for a cuBLAS failure.
namespace {

// One handle per (thread, device); 0 or the C-ABI error code in `code`.
cublasHandle_t thread_handle(int &code) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        code = (int)e;
        return nullptr;
    }
    constexpr int kMaxDev = 64;
    thread_local cublasHandle_t handles[kMaxDev] = {};
    if (dev < 0 || dev >= kMaxDev) {
        code = (int)cudaErrorInvalidDevice;
        return nullptr;
    }
    if (!handles[dev]) {
        const cublasStatus_t s = cublasCreate(&handles[dev]);
        if (s != CUBLAS_STATUS_SUCCESS) {
            handles[dev] = nullptr;
            code = 1000 + (int)s;
            return nullptr;
        }
    }
    code = 0;
    return handles[dev];
}

} // namespace

extern "C" int vg_cublas_gemm_f16(const void *A, const void *B, void *C, int M, int N, int K,
                                  vg_stream_t stream) {
    if (M < 0 || N < 0 || K < 0)
        return (int)cudaErrorInvalidValue;
    if (M == 0 || N == 0)
        return 0;
    int code = 0;
    cublasHandle_t h = thread_handle(code);
    if (!h)
        return code;
    cublasStatus_t s = cublasSetStream(h, (cudaStream_t)stream);
    if (s == CUBLAS_STATUS_SUCCESS)
        s = gemm_ex(h, static_cast<const half *>(A), static_cast<const half *>(B),
                    static_cast<half *>(C), M, N, K);
    return s == CUBLAS_STATUS_SUCCESS ? 0 : 1000 + (int)s;
}

// Validation twin of vg_cublas_gemm_f16: same operands and compute type, fp32 row-major C,
// so cuBLAS's accumulation can be compared with the B200 kernels' fp32-output build.
extern "C" int vg_cublas_gemm_f16_f32out(const void *A, const void *B, float *C, int M, int N,
                                         int K, vg_stream_t stream) {
    if (M < 0 || N < 0 || K < 0)
        return (int)cudaErrorInvalidValue;
    if (M == 0 || N == 0)
        return 0;
    int code = 0;
    cublasHandle_t h = thread_handle(code);
    if (!h)
        return code;
    const float alpha = 1.f, beta = 0.f;
    cublasStatus_t s = cublasSetStream(h, (cudaStream_t)stream);
    if (s == CUBLAS_STATUS_SUCCESS)
        s = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &alpha, B, CUDA_R_16F, K, A,
                         CUDA_R_16F, K, &beta, C, CUDA_R_32F, N, CUBLAS_COMPUTE_32F,
                         CUBLAS_GEMM_DEFAULT);
    return s == CUBLAS_STATUS_SUCCESS ? 0 : 1000 + (int)s;
}

// ── cuBLASLt heuristic sweep (a fairer "best cuBLAS" yardstick) ──────────────────────────
// Asks cuBLASLt for up to `max_algos` algorithms for the row-major problem (the same
// operand order as vg_cublas_gemm_f16: C^T = B^T·A in column-major terms, fp16 in/out,
// CUBLAS_COMPUTE_32F, 64 MiB workspace) and times each one on `stream`: `warmup` untimed
// launches, then `iters` launches between two events. ms_out[i] = mean ms of algorithm i
// (or -1 if it failed); *n_out = number of algorithms returned. C holds the result of the
// last algorithm timed.
#include <cublasLt.h>

extern "C" int vg_cublaslt_sweep(const void *A, const void *B, void *C, int M, int N, int K,
                                 int max_algos, int warmup, int iters, float *ms_out, int *n_out,
                                 vg_stream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || max_algos <= 0 || iters <= 0 || !ms_out || !n_out)
        return (int)cudaErrorInvalidValue;
    *n_out = 0;
    constexpr size_t kWorkspace = 64ull << 20;
    static thread_local void *workspace = nullptr;
    static thread_local int workspace_dev = -1;
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess)
        return (int)ce;
    if (!workspace || workspace_dev != dev) {
        if (workspace)
            (void)cudaFree(workspace); // the previous device's workspace (unified addressing)
        workspace = nullptr;
        ce = cudaMalloc(&workspace, kWorkspace);
        if (ce != cudaSuccess) {
            workspace = nullptr;
            return (int)ce;
        }
        workspace_dev = dev;
    }
    cublasLtHandle_t lt = nullptr;
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
    cublasLtMatmulPreference_t pref = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    auto st = [&](cublasStatus_t s) {
        if (s != CUBLAS_STATUS_SUCCESS && rc == 0)
            rc = 1000 + (int)s;
        return rc == 0;
    };
    const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
    const size_t ws = kWorkspace;
    if (st(cublasLtCreate(&lt)) && st(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F)) &&
        st(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta))) &&
        st(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb))) &&
        st(cublasLtMatrixLayoutCreate(&la, CUDA_R_16F, K, N, K)) &&   // B: N×K row-major
        st(cublasLtMatrixLayoutCreate(&lb, CUDA_R_16F, K, M, K)) &&   // A: M×K row-major
        st(cublasLtMatrixLayoutCreate(&lc, CUDA_R_16F, N, M, N)) &&   // C: M×N row-major
        st(cublasLtMatmulPreferenceCreate(&pref)) &&
        st(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws,
                                                sizeof(ws)))) {
        const int cap = max_algos < 64 ? max_algos : 64;
        cublasLtMatmulHeuristicResult_t res[64];
        int found = 0;
        if (st(cublasLtMatmulAlgoGetHeuristic(lt, op, la, lb, lc, lc, pref, cap, res, &found))) {
            ce = cudaEventCreate(&e0);
            if (ce == cudaSuccess)
                ce = cudaEventCreate(&e1);
            if (ce != cudaSuccess)
                rc = (int)ce;
            const float alpha = 1.f, beta = 0.f;
            cudaStream_t s = (cudaStream_t)stream;
            for (int i = 0; i < found && rc == 0; ++i) {
                auto run = [&]() {
                    return cublasLtMatmul(lt, op, &alpha, B, la, A, lb, &beta, C, lc, C, lc, &res[i].algo,
                                          workspace, kWorkspace, s);
                };
                bool ok = true;
                for (int w = 0; w < warmup && ok; ++w)
                    ok = run() == CUBLAS_STATUS_SUCCESS;
                if (ok && cudaEventRecord(e0, s) == cudaSuccess) {
                    for (int t = 0; t < iters && ok; ++t)
                        ok = run() == CUBLAS_STATUS_SUCCESS;
                    float ms = -1.f;
                    if (ok && cudaEventRecord(e1, s) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
                        cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess)
                        ms_out[i] = ms / iters;
                    else
                        ms_out[i] = -1.f;
                } else {
                    ms_out[i] = -1.f;
                }
                (void)cudaGetLastError();
            }
            *n_out = found;
        }
    }
    if (e0)
        cudaEventDestroy(e0);
    if (e1)
        cudaEventDestroy(e1);
    if (pref)
        cublasLtMatmulPreferenceDestroy(pref);
    if (lc)
        cublasLtMatrixLayoutDestroy(lc);
    if (lb)
        cublasLtMatrixLayoutDestroy(lb);
    if (la)
        cublasLtMatrixLayoutDestroy(la);
    if (op)
        cublasLtMatmulDescDestroy(op);
    if (lt)
        cublasLtDestroy(lt);
    return rc;
}
