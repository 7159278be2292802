// GEMM on host-resident operands with copy/compute overlap.
//
// One call computes C_host = A_host · B_host^T through caller-owned device buffers. A and
// C are split into `chunks` contiguous row blocks; the work is spread over three streams
// owned by the pipeline:
//   h2d      B, then A row block j, host → device (waits until the previous call's
//            GEMMs no longer read dB / dA_j)
//   compute  GEMM of row block j once B and A_j have landed (waits until the previous
//            call's copy-out of dC_j has finished)
//   d2h      C row block j, device → host, as soon as its GEMM is done
// and the caller's stream waits for the last copy-out. Consecutive calls therefore
// overlap: call i+1 uploads while call i's results download on the other copy engine.
// Host buffers must be pinned (cudaHostAlloc / cudaHostRegister) for the copies to be
// asynchronous. No reference counterpart: the reference engine uploads once and times
// device-resident launches only (include/engine.cuh:28-32).
#include <cuda_runtime.h>

#include <algorithm>
#include <new>
#include <vector>

#include "vibegemm_b200.h"

namespace {

constexpr int kMaxChunks = 64;

struct Pipeline {
    int device = 0;
    cudaStream_t h2d = nullptr, compute = nullptr, d2h = nullptr;
    cudaEvent_t b_ready = nullptr;                // B uploaded
    cudaEvent_t gemm_all = nullptr;               // every GEMM of the last call done
    cudaEvent_t a_ready[kMaxChunks] = {};         // A row block j uploaded
    cudaEvent_t gemm_done[kMaxChunks] = {};       // GEMM of row block j done
    cudaEvent_t d2h_done[kMaxChunks] = {};        // C row block j downloaded
    bool has_prev = false;
    int prev_chunks = 0;
};

cudaError_t make_event(cudaEvent_t *e) { return cudaEventCreateWithFlags(e, cudaEventDisableTiming); }

void destroy(Pipeline *p) {
    if (!p)
        return;
    int prev = 0;
    const bool switch_dev = cudaGetDevice(&prev) == cudaSuccess && prev != p->device;
    if (switch_dev)
        cudaSetDevice(p->device);
    for (cudaStream_t s : {p->h2d, p->compute, p->d2h})
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    for (cudaEvent_t e : {p->b_ready, p->gemm_all})
        if (e)
            cudaEventDestroy(e);
    for (int j = 0; j < kMaxChunks; ++j)
        for (cudaEvent_t e : {p->a_ready[j], p->gemm_done[j], p->d2h_done[j]})
            if (e)
                cudaEventDestroy(e);
    if (switch_dev)
        cudaSetDevice(prev);
    delete p;
}

} // namespace

extern "C" {

vg_host_pipeline_t vg_host_pipeline_create(int device) {
    Pipeline *p = new (std::nothrow) Pipeline();
    if (!p)
        return nullptr;
    p->device = device;
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) {
        (void)cudaGetLastError();
        delete p;
        return nullptr;
    }
    bool ok = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->compute, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking) == cudaSuccess &&
              make_event(&p->b_ready) == cudaSuccess && make_event(&p->gemm_all) == cudaSuccess;
    for (int j = 0; ok && j < kMaxChunks; ++j)
        ok = make_event(&p->a_ready[j]) == cudaSuccess && make_event(&p->gemm_done[j]) == cudaSuccess &&
             make_event(&p->d2h_done[j]) == cudaSuccess;
    cudaSetDevice(prev);
    if (!ok) {
        (void)cudaGetLastError();
        destroy(p);
        return nullptr;
    }
    return reinterpret_cast<vg_host_pipeline_t>(p);
}

void vg_host_pipeline_destroy(vg_host_pipeline_t handle) { destroy(reinterpret_cast<Pipeline *>(handle)); }

int vg_host_pipeline_gemm_f16(vg_host_pipeline_t handle, const void *hA, const void *hB, void *hC,
                              void *dA, void *dB, void *dC, int M, int N, int K, int chunks,
                              vg_stream_t done_stream) {
    Pipeline *p = reinterpret_cast<Pipeline *>(handle);
    if (!p || M < 0 || N < 0 || K < 0 || chunks < 1 || chunks > kMaxChunks)
        return (int)cudaErrorInvalidValue;
    if (M == 0 || N == 0)
        return 0;
    if (!hA || !hB || !hC || !dA || !dB || !dC)
        return (int)cudaErrorInvalidValue;
    int cur = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess)
        return (int)e;
    if (cur != p->device)
        return (int)cudaErrorInvalidDevice;

    const size_t esz = 2; // fp16
    const int nchunk = std::min(chunks, M);
    const int rows_per = (M + nchunk - 1) / nchunk;
    const char *ha = static_cast<const char *>(hA);
    char *hc = static_cast<char *>(hC);
    char *da = static_cast<char *>(dA);
    char *dc = static_cast<char *>(dC);

#define VG_TRY(x)                                                                                  \
    do {                                                                                           \
        e = (x);                                                                                   \
        if (e != cudaSuccess)                                                                      \
            return (int)e;                                                                         \
    } while (0)

    // dB (and every dA block) must no longer be read by the previous call's GEMMs.
    if (p->has_prev)
        VG_TRY(cudaStreamWaitEvent(p->h2d, p->gemm_all, 0));
    VG_TRY(cudaMemcpyAsync(dB, hB, (size_t)N * K * esz, cudaMemcpyHostToDevice, p->h2d));
    VG_TRY(cudaEventRecord(p->b_ready, p->h2d));
    for (int j = 0; j < nchunk; ++j) {
        const int r0 = j * rows_per;
        const int rows = std::min(rows_per, M - r0);
        if (rows <= 0)
            break;
        VG_TRY(cudaMemcpyAsync(da + (size_t)r0 * K * esz, ha + (size_t)r0 * K * esz,
                               (size_t)rows * K * esz, cudaMemcpyHostToDevice, p->h2d));
        VG_TRY(cudaEventRecord(p->a_ready[j], p->h2d));
    }
    VG_TRY(cudaStreamWaitEvent(p->compute, p->b_ready, 0));
    // dC must have been copied out by the previous call before it is overwritten (those
    // copies overlap this call's uploads, so this rarely waits).
    if (p->has_prev)
        for (int q = 0; q < p->prev_chunks; ++q)
            VG_TRY(cudaStreamWaitEvent(p->compute, p->d2h_done[q], 0));
    int last = 0;
    for (int j = 0; j < nchunk; ++j) {
        const int r0 = j * rows_per;
        const int rows = std::min(rows_per, M - r0);
        if (rows <= 0)
            break;
        VG_TRY(cudaStreamWaitEvent(p->compute, p->a_ready[j], 0));
        const int ge = vg_b200_gemm_f16(da + (size_t)r0 * K * esz, dB, dc + (size_t)r0 * N * esz,
                                        rows, N, K, reinterpret_cast<vg_stream_t>(p->compute));
        if (ge != 0)
            return ge;
        VG_TRY(cudaEventRecord(p->gemm_done[j], p->compute));
        VG_TRY(cudaStreamWaitEvent(p->d2h, p->gemm_done[j], 0));
        VG_TRY(cudaMemcpyAsync(hc + (size_t)r0 * N * esz, dc + (size_t)r0 * N * esz,
                               (size_t)rows * N * esz, cudaMemcpyDeviceToHost, p->d2h));
        VG_TRY(cudaEventRecord(p->d2h_done[j], p->d2h));
        last = j;
    }
    VG_TRY(cudaEventRecord(p->gemm_all, p->compute));
    VG_TRY(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(done_stream), p->d2h_done[last], 0));
#undef VG_TRY
    p->has_prev = true;
    p->prev_chunks = last + 1;
    return 0;
}

} // extern "C"
