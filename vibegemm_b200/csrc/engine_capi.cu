// C ABI over the reference-facing plugin layer: the registry (GemmBackend::run by
// name) and the benchmark engine. Lets the Python tests and the bench drive exactly
// the path a VibeGEMM user drives (registry → backend → launchKernel) through plain
// C calls.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "engine.cuh"
#include "registry.cuh"
#include "vibegemm_b200.h"

namespace {

std::mutex g_mu;
std::vector<std::string> g_names;
std::vector<std::shared_ptr<GemmBackend>> g_backends;
std::vector<EngineResult> g_results;

void ensure_backends() {
    if (!g_backends.empty())
        return;
    g_backends = KernelRegistry::instance().make_all();
    g_names.clear();
    for (auto &b : g_backends)
        g_names.push_back(b->name());
}

} // namespace

extern "C" {

int vg_backend_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return (int)KernelRegistry::instance().names().size();
}

const char *vg_backend_name(int i) {
    std::lock_guard<std::mutex> lk(g_mu);
    static thread_local std::vector<std::string> names;
    names = KernelRegistry::instance().names();
    if (i < 0 || i >= (int)names.size())
        return nullptr;
    return names[i].c_str();
}

int vg_backend_run(const char *name, void *A, void *B, void *C, int M, int N, int K) {
    if (!name)
        return (int)cudaErrorInvalidValue;
    std::shared_ptr<GemmBackend> b;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        ensure_backends();
        for (size_t i = 0; i < g_backends.size(); ++i)
            if (g_names[i] == name)
                b = g_backends[i];
    }
    if (!b)
        return (int)cudaErrorInvalidValue;
    if (!b->is_available())
        return (int)cudaErrorNoKernelImageForDevice;
    b->run(static_cast<half *>(A), static_cast<half *>(B), static_cast<half *>(C), M, N, K);
    return (int)cudaGetLastError();
}

int vg_engine_execute(int M, int N, int K, int inputs, const char *log_path) {
    if (M <= 0 || N <= 0 || K <= 0)
        return (int)cudaErrorInvalidValue;
    FILE *fp = nullptr;
    if (log_path && *log_path) {
        fp = std::fopen(log_path, "a");
        if (!fp)
            return (int)cudaErrorInvalidValue;
    }
    BenchmarkEngine engine;
    engine.set_log_file(fp);
    engine.set_inputs(inputs == 1 ? BenchmarkEngine::Inputs::Normal002
                                  : BenchmarkEngine::Inputs::Uniform);
    for (auto &b : KernelRegistry::instance().make_all()) {
        const std::string n = b->name();
        if (n.find("A100") != std::string::npos || n.find("H100") != std::string::npos)
            continue;
        engine.add_backend(b);
    }
    engine.execute(M, N, K);
    if (fp)
        std::fclose(fp);
    std::lock_guard<std::mutex> lk(g_mu);
    g_results = engine.results();
    return 0;
}

int vg_engine_result_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return (int)g_results.size();
}

int vg_engine_result(int i, char *name_buf, int name_len, double *out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (i < 0 || i >= (int)g_results.size())
        return (int)cudaErrorInvalidValue;
    const EngineResult &r = g_results[i];
    if (name_buf && name_len > 0) {
        std::strncpy(name_buf, r.name.c_str(), (size_t)name_len - 1);
        name_buf[name_len - 1] = '\0';
    }
    if (out) {
        out[0] = r.avg_ms;
        out[1] = r.tflops;
        out[2] = r.err.max_abs_err;
        out[3] = r.err.max_rel_err;
        out[4] = (r.ran && r.err.passed) ? 1.0 : 0.0;
        out[5] = r.skipped ? 1.0 : 0.0;
    }
    return 0;
}

} // extern "C"
