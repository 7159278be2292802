// ORACLE — CPU restatement of the reference's FP16 GEMM path. TEST INFRASTRUCTURE ONLY.
//
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference-arm
// leg may load this library, and only as the checker or the timed CPU baseline —
// never as the product path. The product (vibegemm_b200/libvibegemm_b200.so) never
// links, loads or calls it.
//
// What it restates (reference = AnonymousSC2026/VibeGEMM):
//  * oracle_fill_uniform_f16: include/utils.cuh:59-66 — std::mt19937(seed),
//    std::uniform_real_distribution<float>(-1, 1), __float2half (round to nearest
//    even). Same libstdc++ engine and distribution, so bit-identical.
//  * oracle_fill_normal_f16: N(mean, std) via std::normal_distribution<float> on
//    mt19937(seed) (the LLM-projection configs; the reference has no normal fill).
//  * oracle_gemm_*: the naive kernels csrc/a100/gemm_8192x8192_v0.cuh:23-74 and
//    csrc/h100/gemm_8192x8192_v8.cuh:347-358:
//        float acc = 0; for k in 0..K-1: acc += float(A[m*K+k]) * float(B[n*K+k]);
//        C[m*N+n] = __float2half(acc)
//    nvcc contracts `acc += a*b` into one fused multiply-add, so the restatement uses
//    fmaf in the same k order and is bit-identical to those kernels (pinned by the
//    golden fixtures produced from the reference's own v0 kernel).
//  * oracle_check_error: include/utils.cuh:70-118 — |r-c| <= atol + rtol*|r|,
//    max abs error, max rel error |r-c| / max(|r|, 1e-6).
//
// Parallelised with std::thread over row blocks; the vector loop runs across output
// columns so every output keeps its own strictly sequential k order.
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <random>
#include <thread>
#include <vector>

namespace {

// IEEE binary32 -> binary16, round to nearest even; overflow to inf, NaN kept quiet.
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) // inf / NaN
        return static_cast<uint16_t>(sign | 0x7c00u | (ax > 0x7f800000u ? (0x200u | ((ax >> 13) & 0x3ffu)) : 0u));
    if (ax >= 0x477ff000u) // >= 65520 rounds to inf
        return static_cast<uint16_t>(sign | 0x7c00u);
    if (ax < 0x38800000u) { // below 2^-14: subnormal half (or zero)
        float v;
        std::memcpy(&v, &ax, 4);
        const float scaled = v * 16777216.0f; // exact: multiply by 2^24
        const uint32_t m = static_cast<uint32_t>(std::nearbyint(scaled)); // ties to even
        return static_cast<uint16_t>(sign | m);
    }
    const uint32_t e = (ax >> 23) - 127u + 15u;
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
        h += 1u;
    return static_cast<uint16_t>(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            const float v = static_cast<float>(m) * (1.0f / 16777216.0f);
            std::memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e - 15u + 127u) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

int threads_or_default(int threads) {
    if (threads > 0)
        return threads;
    const unsigned hc = std::thread::hardware_concurrency();
    return hc > 0 ? static_cast<int>(hc) : 1;
}

// Runs body(i) for i in [0, n) on `nt` threads, handing out indices dynamically.
template <typename Body> void parallel_for(long n, int nt, Body body) {
    if (nt <= 1 || n <= 1) {
        for (long i = 0; i < n; ++i)
            body(i);
        return;
    }
    std::atomic<long> next{0};
    auto worker = [&] {
        for (long i = next.fetch_add(1); i < n; i = next.fetch_add(1))
            body(i);
    };
    std::vector<std::thread> pool;
    const long workers = n < nt ? n : nt;
    for (long t = 1; t < workers; ++t)
        pool.emplace_back(worker);
    worker();
    for (auto &th : pool)
        th.join();
}

constexpr long kRowBlock = 8;   // output rows sharing one streamed B^T row
constexpr long kColBlock = 256; // output columns per accumulator block

// out[r, n] for rows [row0, row0+rows): sequential-k fused multiply-add in fp32
// (or fp64 when Acc = double). Emit(m, n, acc) stores one result.
template <typename Acc, typename Emit>
void gemm_rows(const uint16_t *A, const uint16_t *B, long N, long K, long row0, long rows,
               int threads, Emit emit) {
    const int nt = threads_or_default(threads);
    std::vector<float> bt(static_cast<size_t>(K) * kColBlock);
    for (long nb = 0; nb < N; nb += kColBlock) {
        const long nlen = (N - nb) < kColBlock ? (N - nb) : kColBlock;
        // B^T block: bt[k*kColBlock + j] = float(B[(nb+j)*K + k]).
        const long kchunks = (K + 255) / 256;
        parallel_for(kchunks, nt, [&](long kc) {
            const long k1 = (kc + 1) * 256 < K ? (kc + 1) * 256 : K;
            for (long k = kc * 256; k < k1; ++k) {
                float *dst = bt.data() + static_cast<size_t>(k) * kColBlock;
                for (long j = 0; j < nlen; ++j)
                    dst[j] = f16_to_f32(B[static_cast<size_t>(nb + j) * K + k]);
                for (long j = nlen; j < kColBlock; ++j)
                    dst[j] = 0.0f;
            }
        });
        const long nblocks = (rows + kRowBlock - 1) / kRowBlock;
        parallel_for(nblocks, nt, [&](long rb) {
            const long r0 = row0 + rb * kRowBlock;
            const long rl = (row0 + rows - r0) < kRowBlock ? (row0 + rows - r0) : kRowBlock;
            alignas(64) Acc acc[kRowBlock][kColBlock];
            for (long r = 0; r < kRowBlock; ++r)
                for (long j = 0; j < kColBlock; ++j)
                    acc[r][j] = Acc(0);
            for (long k = 0; k < K; ++k) {
                const float *brow = bt.data() + static_cast<size_t>(k) * kColBlock;
                for (long r = 0; r < rl; ++r) {
                    const Acc a = static_cast<Acc>(f16_to_f32(A[static_cast<size_t>(r0 + r) * K + k]));
                    Acc *ar = acc[r];
                    if constexpr (sizeof(Acc) == 4) {
#pragma omp simd
                        for (long j = 0; j < kColBlock; ++j)
                            ar[j] = std::fmaf(a, brow[j], ar[j]);
                    } else {
#pragma omp simd
                        for (long j = 0; j < kColBlock; ++j)
                            ar[j] = std::fma(a, static_cast<Acc>(brow[j]), ar[j]);
                    }
                }
            }
            for (long r = 0; r < rl; ++r)
                for (long j = 0; j < nlen; ++j)
                    emit(r0 + r, nb + j, acc[r][j]);
        });
    }
}

} // namespace

extern "C" {

uint16_t oracle_f32_to_f16(float x) { return f32_to_f16(x); }
float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

void oracle_f32_to_f16_array(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i)
        out[i] = f32_to_f16(in[i]);
}

// include/utils.cuh:59-66 (uniform[-1,1], mt19937(seed)).
void oracle_fill_uniform_f16(uint16_t *out, size_t n, unsigned seed) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    for (size_t i = 0; i < n; ++i)
        out[i] = f32_to_f16(dist(rng));
}

void oracle_fill_normal_f16(uint16_t *out, size_t n, unsigned seed, float mean, float stddev) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (size_t i = 0; i < n; ++i)
        out[i] = f32_to_f16(dist(rng));
}

// Rows [row0, row0+rows) of the M×N product; C holds just those rows (rows × N).
// A points at row 0 of the full M×K operand.
void oracle_gemm_f16(const uint16_t *A, const uint16_t *B, uint16_t *C, long M, long N, long K,
                     long row0, long rows, int threads) {
    (void)M;
    gemm_rows<float>(A, B, N, K, row0, rows, threads, [&](long m, long n, float acc) {
        C[static_cast<size_t>(m - row0) * N + n] = f32_to_f16(acc);
    });
}

void oracle_gemm_f32(const uint16_t *A, const uint16_t *B, float *C, long M, long N, long K,
                     long row0, long rows, int threads) {
    (void)M;
    gemm_rows<float>(A, B, N, K, row0, rows, threads,
                     [&](long m, long n, float acc) { C[static_cast<size_t>(m - row0) * N + n] = acc; });
}

// fp64 accumulation: the "exact" reference for judging accumulation error.
void oracle_gemm_f64(const uint16_t *A, const uint16_t *B, double *C, long M, long N, long K,
                     long row0, long rows, int threads) {
    (void)M;
    gemm_rows<double>(A, B, N, K, row0, rows, threads,
                      [&](long m, long n, double acc) { C[static_cast<size_t>(m - row0) * N + n] = acc; });
}

// include/utils.cuh:70-118. stats: [max_abs, max_rel, max_abs_idx, max_rel_idx, mismatches].
int oracle_check_error(const uint16_t *ref, const uint16_t *cmp, size_t n, float atol, float rtol,
                       double *stats) {
    float max_abs = 0.f, max_rel = 0.f;
    size_t abs_idx = 0, rel_idx = 0, bad = 0;
    for (size_t i = 0; i < n; ++i) {
        const float r = f16_to_f32(ref[i]);
        const float c = f16_to_f32(cmp[i]);
        const float abs_err = std::fabs(r - c);
        const float rel_err = abs_err / std::fmax(std::fabs(r), 1e-6f);
        if (abs_err > max_abs) {
            max_abs = abs_err;
            abs_idx = i;
        }
        if (rel_err > max_rel) {
            max_rel = rel_err;
            rel_idx = i;
        }
        if (!(abs_err <= atol + rtol * std::fabs(r)))
            ++bad;
    }
    if (stats) {
        stats[0] = max_abs;
        stats[1] = max_rel;
        stats[2] = static_cast<double>(abs_idx);
        stats[3] = static_cast<double>(rel_idx);
        stats[4] = static_cast<double>(bad);
    }
    return bad == 0 ? 1 : 0;
}

int oracle_max_threads(void) { return threads_or_default(0); }

} // extern "C"
