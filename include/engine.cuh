// Derived from VibeGEMM's include/engine.cuh (AnonymousSC2026/VibeGEMM, licensed under the
// GNU General Public License v3.0): kept from it with the additive changes listed below, and
// distributed under the same licence (see NOTICE).
//
// BenchmarkEngine — validates and times every registered backend on one shape.
//
// Same procedure as the reference engine (include/engine.cuh:11-143 of VibeGEMM):
// grow-only device buffers; A from seed 42 and B from seed 77; backends_[0] (cuBLAS,
// priority 0) computes the reference C; for each backend: [SKIP] if unavailable,
// 10 warm-up launches, 30 launches between two events on the default stream
// (avg = total/30, launch cost included, no L2 flush), then C_test is zeroed, the
// backend runs once more and check_error compares it to the reference.
// Additions: per-backend results are kept (results()) instead of only printed, and
// the input distribution can be switched to N(0, 0.02) for the LLM-projection shapes.
#pragma once

#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <memory>
#include <string>
#include <vector>

#include "backend.cuh"
#include "utils.cuh"

struct EngineResult {
    std::string name;
    double avg_ms = -1.0;
    double tflops = 0.0;
    ErrorStats err;
    bool skipped = false;
    bool ran = false;
};

class BenchmarkEngine {
  public:
    static constexpr int kWarmup = 10;
    static constexpr int kBenchmark = 30;

    enum class Inputs { Uniform, Normal002 };

    ~BenchmarkEngine() {
        for (half *p : {d_A_, d_B_, d_C_ref_, d_C_test_})
            if (p)
                cudaFree(p);
    }

    void set_log_file(FILE *fp) { fp_ = fp; }
    void set_inputs(Inputs kind) { inputs_ = kind; }
    void add_backend(std::shared_ptr<GemmBackend> b) { backends_.push_back(std::move(b)); }
    const std::vector<EngineResult> &results() const { return results_; }

    void execute(int M, int N, int K) {
        results_.clear();
        log_print("\n=== GEMM  M=%d  N=%d  K=%d ===\n", M, N, K);

        if (!alloc_buffers(M, N, K)) {
            log_print("  [ERROR] device buffer allocation failed; skipping shape.\n");
            return;
        }
        const bool filled =
            (inputs_ == Inputs::Uniform)
                ? (fill_random_fp16(d_A_, (size_t)M * K, 42) && fill_random_fp16(d_B_, (size_t)K * N, 77))
                : (fill_normal_fp16(d_A_, (size_t)M * K, 42) && fill_normal_fp16(d_B_, (size_t)K * N, 77));
        if (!filled) {
            log_print("  [ERROR] failed to upload random A/B; skipping shape.\n");
            return;
        }
        if (backends_.empty())
            return;

        auto &reference = backends_[0];
        reference->run(d_A_, d_B_, d_C_ref_, M, N, K);
        if (!cuda_check("reference")) {
            log_print("  [ERROR] reference backend failed; skipping shape.\n");
            reference->teardown();
            return;
        }

        for (auto &b : backends_) {
            EngineResult res;
            res.name = b->name();
            log_print("\n[%s]\n", res.name.c_str());
            if (!b->is_available()) {
                log_print("  [SKIP] backend not available\n");
                res.skipped = true;
                results_.push_back(res);
                b->teardown();
                continue;
            }

            for (int i = 0; i < kWarmup; ++i)
                b->run(d_A_, d_B_, d_C_test_, M, N, K);

            CudaTimer timer;
            timer.start();
            for (int i = 0; i < kBenchmark; ++i)
                b->run(d_A_, d_B_, d_C_test_, M, N, K);
            const float total_ms = timer.stop();
            if (total_ms < 0.f) {
                log_print("  [ERROR] CUDA timer failed; skipping backend.\n");
                (void)cudaGetLastError();
                results_.push_back(res);
                b->teardown();
                continue;
            }
            res.avg_ms = total_ms / kBenchmark;
            res.tflops = tflops(M, N, K, res.avg_ms);
            log_print("  avg latency = %.3f ms   %.2f TFLOPS\n", res.avg_ms, res.tflops);

            if (!CUDA_TRY(cudaMemset(d_C_test_, 0, (size_t)M * N * sizeof(half)))) {
                log_print("  [WARN] cudaMemset failed; skipping correctness check.\n");
                results_.push_back(res);
                b->teardown();
                continue;
            }
            b->run(d_A_, d_B_, d_C_test_, M, N, K);
            if (!cuda_check(res.name.c_str())) {
                log_print("  [WARN] CUDA failure on correctness run.\n");
                results_.push_back(res);
                b->teardown();
                continue;
            }
            check_error(d_C_ref_, d_C_test_, (size_t)M * N, 1e-3f, 1e-2f, 5, &res.err);
            log_print("  check: max_abs=%e max_rel=%e (%s)\n", res.err.max_abs_err,
                      res.err.max_rel_err, res.err.passed ? "PASS" : "FAIL");
            res.ran = true;
            results_.push_back(res);
            b->teardown();
        }
    }

  private:
    FILE *fp_ = nullptr;
    Inputs inputs_ = Inputs::Uniform;
    std::vector<std::shared_ptr<GemmBackend>> backends_;
    std::vector<EngineResult> results_;

    half *d_A_ = nullptr;
    half *d_B_ = nullptr;
    half *d_C_ref_ = nullptr;
    half *d_C_test_ = nullptr;
    size_t cap_A_ = 0, cap_B_ = 0, cap_C_ref_ = 0, cap_C_test_ = 0;

    // stdout and, when set, the log file.
    void log_print(const char *fmt, ...) {
        va_list args;
        va_start(args, fmt);
        std::vprintf(fmt, args);
        va_end(args);
        if (fp_) {
            va_start(args, fmt);
            std::vfprintf(fp_, fmt, args);
            va_end(args);
            std::fflush(fp_);
        }
        std::fflush(stdout);
    }

    static bool grow(half *&p, size_t &cap, size_t need) {
        if (need <= cap)
            return true;
        if (p) {
            if (!CUDA_TRY(cudaFree(p)))
                return false;
            p = nullptr;
            cap = 0;
        }
        void *raw = nullptr;
        if (!CUDA_TRY(cudaMalloc(&raw, need)))
            return false;
        p = static_cast<half *>(raw);
        cap = need;
        return true;
    }

    bool alloc_buffers(int M, int N, int K) {
        const size_t a = (size_t)M * K * sizeof(half), b = (size_t)K * N * sizeof(half),
                     c = (size_t)M * N * sizeof(half);
        if (!grow(d_A_, cap_A_, a) || !grow(d_B_, cap_B_, b) || !grow(d_C_ref_, cap_C_ref_, c) ||
            !grow(d_C_test_, cap_C_test_, c)) {
            std::fprintf(stderr, "BenchmarkEngine: buffer allocation failed; skipping shape.\n");
            return false;
        }
        return true;
    }
};
