// VibeGEMM driver: runs every registered backend of this build through the engine.
//
// Mirrors the reference driver (main.cu:68-109 of VibeGEMM): query device 0, open
// the per-architecture log, take KernelRegistry::make_all(), keep the backends of
// this architecture, run each problem size. The B200 arm (sm >= 100) keeps
// "B200" backends and cuBLAS, drops "A100"/"H100" names and logs to
// results/perf_b200.txt. The default problem list is the reference's (8192³);
// shapes can be given as arguments: `VibeGEMM [--normal] [--only SUBSTR] MxNxK ...`
// (--normal = N(0, 0.02) inputs instead of uniform[-1,1]; --only keeps cuBLAS, the engine's
// reference, and the backends whose names contain SUBSTR).
// Besides the reference's text log, one JSON line per (backend, shape) goes to
// results/perf_<arch>.jsonl: TFLOP/s, % of cuBLAS, % of the dense fp16 peak
// (VG_PEAK_TFLOPS, else the nominal 2250 of B200), the check_error figures and the
// host's core count.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <sys/stat.h>
#include <thread>
#include <vector>

#include "engine.cuh"
#include "registry.cuh"

static FILE *g_fp = nullptr;

static void log_print(const char *fmt, ...) {
    va_list args;
    va_start(args, fmt);
    std::vprintf(fmt, args);
    va_end(args);
    if (g_fp) {
        va_start(args, fmt);
        std::vfprintf(g_fp, fmt, args);
        va_end(args);
    }
}

static void json_string(FILE *fp, const std::string &v) {
    std::fputc('"', fp);
    for (char ch : v) {
        if (ch == '"' || ch == '\\')
            std::fputc('\\', fp);
        if (static_cast<unsigned char>(ch) >= 0x20)
            std::fputc(ch, fp);
    }
    std::fputc('"', fp);
}

// JSON has no inf / nan: non-finite error figures are written as null.
static void json_number(FILE *fp, double v) {
    if (std::isfinite(v))
        std::fprintf(fp, "%.6g", v);
    else
        std::fputs("null", fp);
}

// One JSON object per backend result of the last engine.execute().
static void write_json_results(FILE *fp, const cudaDeviceProp &prop, int sm, int M, int N, int K,
                               bool normal, const std::vector<EngineResult> &results) {
    double peak = 2250.0;
    const char *peak_kind = "nominal";
    if (const char *env = std::getenv("VG_PEAK_TFLOPS")) {
        const double v = std::atof(env);
        if (v > 0) {
            peak = v;
            peak_kind = "env";
        }
    }
    double cublas = 0.0;
    for (const auto &r : results)
        if (r.ran && r.name.find("cuBLAS") != std::string::npos)
            cublas = r.tflops;
    for (const auto &r : results) {
        std::fprintf(fp, "{\"gpu\": ");
        json_string(fp, prop.name);
        std::fprintf(fp, ", \"sm\": %d, \"ngpu\": 1, \"backend\": ", sm);
        json_string(fp, r.name);
        std::fprintf(fp, ", \"M\": %d, \"N\": %d, \"K\": %d, \"inputs\": \"%s\"", M, N, K,
                     normal ? "normal(0,0.02)" : "uniform(-1,1)");
        if (r.skipped || !r.ran) {
            std::fprintf(fp, ", \"skipped\": %s, \"ran\": %s}\n", r.skipped ? "true" : "false",
                         r.ran ? "true" : "false");
            continue;
        }
        std::fprintf(fp,
                     ", \"avg_ms\": %.6f, \"tflops\": %.2f, \"pct_cublas\": %.2f, \"pct_peak\": %.2f,"
                     " \"peak_tflops\": %.1f, \"peak_kind\": \"%s\", \"max_abs_err\": ",
                     r.avg_ms, r.tflops, cublas > 0 ? 100.0 * r.tflops / cublas : 0.0,
                     100.0 * r.tflops / peak, peak, peak_kind);
        json_number(fp, r.err.max_abs_err);
        std::fprintf(fp, ", \"max_rel_err\": ");
        json_number(fp, r.err.max_rel_err);
        std::fprintf(fp, ", \"mismatches\": %zu, \"passed\": %s, \"cpu_cores\": %u}\n",
                     r.err.mismatches, r.err.passed ? "true" : "false",
                     std::thread::hardware_concurrency());
    }
    std::fflush(fp);
}

struct GemmProblem {
    const char *label;
    int m, n, k;
};

static const GemmProblem kDefaultSizes[] = {
    {nullptr, 8192, 8192, 8192},
};

int main(int argc, char **argv) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, 0) != cudaSuccess) {
        std::fprintf(stderr, "no CUDA device\n");
        return 1;
    }
    const int sm = prop.major * 10 + prop.minor;

    std::vector<GemmProblem> sizes;
    bool normal = false;
    std::string only;
    for (int i = 1; i < argc; ++i) {
        if (std::strcmp(argv[i], "--normal") == 0) {
            normal = true;
            continue;
        }
        if (std::strcmp(argv[i], "--only") == 0 && i + 1 < argc) {
            only = argv[++i];
            continue;
        }
        int m = 0, n = 0, k = 0;
        if (std::sscanf(argv[i], "%dx%dx%d", &m, &n, &k) == 3 && m > 0 && n > 0 && k > 0)
            sizes.push_back({nullptr, m, n, k});
        else {
            std::fprintf(stderr, "bad shape '%s' (expected MxNxK)\n", argv[i]);
            return 2;
        }
    }
    if (sizes.empty())
        sizes.assign(std::begin(kDefaultSizes), std::end(kDefaultSizes));

    mkdir("results", 0755);
    const std::string log_file = (sm >= 100)  ? "results/perf_b200.txt"
                                 : (sm >= 90) ? "results/perf_h100.txt"
                                              : "results/perf_a100.txt";
    g_fp = std::fopen(log_file.c_str(), "w");
    if (!g_fp) {
        std::fprintf(stderr, "Failed to open %s for writing!\n", log_file.c_str());
        return 1;
    }
    log_print("=== Device: %s (SM: %d) ===\n", prop.name, sm);
    const std::string json_file = log_file.substr(0, log_file.size() - 4) + ".jsonl";
    FILE *jfp = std::fopen(json_file.c_str(), "w");
    if (!jfp) {
        std::fprintf(stderr, "Failed to open %s for writing!\n", json_file.c_str());
        return 1;
    }

    BenchmarkEngine engine;
    engine.set_log_file(g_fp);
    if (normal)
        engine.set_inputs(BenchmarkEngine::Inputs::Normal002);

    for (auto &b : KernelRegistry::instance().make_all()) {
        const std::string name = b->name();
        const bool is_a100 = name.find("A100") != std::string::npos;
        const bool is_h100 = name.find("H100") != std::string::npos;
        const bool is_b200 = name.find("B200") != std::string::npos;
        if (sm >= 100 && (is_a100 || is_h100))
            continue;
        if (sm >= 90 && sm < 100 && (is_a100 || is_b200))
            continue;
        if (sm < 90 && (is_h100 || is_b200))
            continue;
        if (!only.empty() && name != "cuBLAS" && name.find(only) == std::string::npos)
            continue;
        engine.add_backend(b);
    }

    int failures = 0;
    for (const auto &c : sizes) {
        if (c.label)
            log_print("\n>>> %s\n", c.label);
        engine.execute(c.m, c.n, c.k);
        write_json_results(jfp, prop, sm, c.m, c.n, c.k, normal, engine.results());
        for (const auto &r : engine.results())
            if (!r.skipped && (!r.ran || !r.err.passed))
                ++failures;
    }
    log_print("\nDone.\n");
    std::fflush(g_fp);
    std::fclose(g_fp);
    g_fp = nullptr;
    std::fclose(jfp);
    return failures == 0 ? 0 : 3;
}
