// Derived from VibeGEMM's include/utils.cuh (AnonymousSC2026/VibeGEMM, licensed under the
// GNU General Public License v3.0): kept from it with the additive changes listed below, and
// distributed under the same licence (see NOTICE).
//
// Host helpers of the benchmark harness: error handling, input generation, the
// element-wise correctness check, CUDA-event timing and the TFLOPS formula.
//
// Behaviour matches the reference helpers (include/utils.cuh:1-150 of VibeGEMM):
//  * CUDA_TRY logs and returns false; cuda_check() synchronises and clears the error.
//  * fill_random_fp16: std::mt19937(seed) → std::uniform_real_distribution<float>(-1,1)
//    → round-to-nearest fp16, uploaded with one cudaMemcpy. Same engine, distribution
//    and conversion, so the same seed produces bit-identical matrices.
//  * check_error: per element |r - c| <= atol + rtol·|r| (atol 1e-3, rtol 1e-2), max
//    abs error and max rel error |r - c| / max(|r|, 1e-6), prints "(PASS)"/"(FAIL)".
//  * tflops = 2·M·N·K / (ms · 1e9).
// Additions: fill_normal_fp16 (N(mean, std) inputs for the LLM-projection shapes) and
// an optional ErrorStats out-parameter so callers can keep the numbers.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <random>
#include <string>
#include <vector>

inline bool cuda_report_error(cudaError_t err, const char *file, int line) {
    if (err == cudaSuccess)
        return true;
    std::fprintf(stderr, "CUDA error %s:%d  %s\n", file, line, cudaGetErrorString(err));
    return false;
}

#define CUDA_TRY(call) cuda_report_error((call), __FILE__, __LINE__)

// Synchronise the device; on failure report it under `context` and clear the sticky
// last-error state so later work can proceed.
inline bool cuda_check(const char *context) {
    const cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess)
        return true;
    std::fprintf(stderr, "[%s] %s\n", context, cudaGetErrorString(e));
    (void)cudaGetLastError();
    return false;
}

#define CUDA_CHECK(call)                                                                           \
    do {                                                                                           \
        cudaError_t vg_e_ = (call);                                                                \
        if (vg_e_ != cudaSuccess) {                                                                \
            std::fprintf(stderr, "CUDA error %s:%d  %s\n", __FILE__, __LINE__,                     \
                         cudaGetErrorString(vg_e_));                                               \
            std::exit(EXIT_FAILURE);                                                               \
        }                                                                                          \
    } while (0)

#define CUBLAS_CHECK(call)                                                                         \
    do {                                                                                           \
        cublasStatus_t vg_s_ = (call);                                                             \
        if (vg_s_ != CUBLAS_STATUS_SUCCESS) {                                                      \
            std::fprintf(stderr, "cuBLAS error %s:%d  status=%d\n", __FILE__, __LINE__,            \
                         (int)vg_s_);                                                              \
            std::exit(EXIT_FAILURE);                                                               \
        }                                                                                          \
    } while (0)

inline half *alloc_fp16(size_t elems) {
    half *p = nullptr;
    CUDA_CHECK(cudaMalloc(&p, elems * sizeof(half)));
    return p;
}

// Host-side generation of uniform[-1,1] fp16 values (the reference's input recipe).
inline void host_random_fp16(std::vector<half> &out, size_t elems, unsigned seed) {
    out.resize(elems);
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    for (size_t i = 0; i < elems; ++i)
        out[i] = __float2half(dist(rng));
}

inline bool fill_random_fp16(half *d_ptr, size_t elems, unsigned seed = 42) {
    std::vector<half> h;
    host_random_fp16(h, elems, seed);
    return CUDA_TRY(cudaMemcpy(d_ptr, h.data(), elems * sizeof(half), cudaMemcpyHostToDevice));
}

// N(mean, stddev) fp16 values from std::normal_distribution<float> on mt19937(seed).
inline bool fill_normal_fp16(half *d_ptr, size_t elems, unsigned seed, float mean = 0.0f,
                             float stddev = 0.02f) {
    std::vector<half> h(elems);
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (size_t i = 0; i < elems; ++i)
        h[i] = __float2half(dist(rng));
    return CUDA_TRY(cudaMemcpy(d_ptr, h.data(), elems * sizeof(half), cudaMemcpyHostToDevice));
}

struct ErrorStats {
    float max_abs_err = 0.f;
    float max_rel_err = 0.f;
    size_t max_abs_idx = 0;
    size_t max_rel_idx = 0;
    size_t mismatches = 0;
    bool passed = false;
};

inline bool check_error(half *ref, half *cmp, size_t elems, float atol = 1e-3f, float rtol = 1e-2f,
                        size_t print_first_n = 5, ErrorStats *stats = nullptr) {
    std::vector<half> hr(elems), hc(elems);
    if (!CUDA_TRY(cudaMemcpy(hr.data(), ref, elems * sizeof(half), cudaMemcpyDeviceToHost)))
        return false;
    if (!CUDA_TRY(cudaMemcpy(hc.data(), cmp, elems * sizeof(half), cudaMemcpyDeviceToHost)))
        return false;

    ErrorStats s;
    size_t printed = 0;
    for (size_t i = 0; i < elems; ++i) {
        const float r = __half2float(hr[i]);
        const float c = __half2float(hc[i]);
        const float abs_err = std::fabs(r - c);
        const float rel_err = abs_err / std::max(std::fabs(r), 1e-6f);
        if (abs_err > s.max_abs_err) {
            s.max_abs_err = abs_err;
            s.max_abs_idx = i;
        }
        if (rel_err > s.max_rel_err) {
            s.max_rel_err = rel_err;
            s.max_rel_idx = i;
        }
        // NaN-safe: a NaN on either side fails the comparison.
        if (!(abs_err <= atol + rtol * std::fabs(r))) {
            ++s.mismatches;
            if (printed < print_first_n) {
                std::fprintf(stdout, "  mismatch[%zu]: ref=%.6f  cmp=%.6f  abs=%.6e  rel=%.6e\n", i,
                             r, c, abs_err, rel_err);
                ++printed;
            }
        }
    }
    s.passed = (s.mismatches == 0);
    std::fprintf(stdout, "  max absolute error = %e at [%zu]\n", s.max_abs_err, s.max_abs_idx);
    std::fprintf(stdout, "  max relative error = %e at [%zu]  (%s)\n", s.max_rel_err, s.max_rel_idx,
                 s.passed ? "PASS" : "FAIL");
    if (stats)
        *stats = s;
    return s.passed;
}

// CUDA events recorded on the legacy default stream (where backends launch).
struct CudaTimer {
    cudaEvent_t start_{}, stop_{};
    CudaTimer() {
        CUDA_CHECK(cudaEventCreate(&start_));
        CUDA_CHECK(cudaEventCreate(&stop_));
    }
    ~CudaTimer() {
        cudaEventDestroy(start_);
        cudaEventDestroy(stop_);
    }
    CudaTimer(const CudaTimer &) = delete;
    CudaTimer &operator=(const CudaTimer &) = delete;

    void start() { (void)CUDA_TRY(cudaEventRecord(start_)); }
    // Elapsed milliseconds, or a negative value when timing failed.
    float stop() {
        float ms = -1.f;
        if (!CUDA_TRY(cudaEventRecord(stop_)))
            return ms;
        if (!CUDA_TRY(cudaEventSynchronize(stop_)))
            return ms;
        if (!CUDA_TRY(cudaEventElapsedTime(&ms, start_, stop_)))
            return -1.f;
        return ms;
    }
};

inline double tflops(int m, int n, int k, double ms) { return 2.0 * m * n * k / (ms * 1e9); }
