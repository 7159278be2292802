/*
 * vibegemm_b200.h — C ABI of the B200 (sm_100a) FP16 GEMM backend.
 *
 * Semantics of every GEMM entry point (identical to the reference backends):
 *   C[m*N + n] = fp16_rn( sum_k float(A[m*K + k]) * float(B[n*K + k]) )
 *   A: M×K fp16 row-major; B: N×K fp16 (K contiguous, i.e. "K×N column-major");
 *   C: M×N row-major; alpha = 1, beta = 0; C is fully overwritten; fp32 accumulate.
 *   All pointers are device pointers owned by the caller.
 *
 * Return values are cudaError_t codes (0 = cudaSuccess). Launches are asynchronous
 * on `stream` (NULL = the legacy default stream, which is where the reference
 * engine records its timing events). Asynchronous device faults surface at the
 * caller's next synchronisation, as with the reference's cuda_check().
 *
 * Plain C types only: pointers, ints and an opaque stream handle that is
 * ABI-identical to cudaStream_t.
 */
#ifndef VIBEGEMM_B200_H
#define VIBEGEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *vg_stream_t;

/* Default B200 kernel: the version chosen per shape ("VibeGEMM B200 auto", version -1).
 * Replaces GemmBackend::run (include/backend.cuh:13) of a registered backend and the
 * per-version free function launchKernel(half*,half*,half*,int,int,int)
 * (csrc/h100/gemm_8192x8192_v18.cuh:545, bound through csrc/gemm_h100_backends.cu:41). */
int vg_b200_gemm_f16(const void *A, const void *B, void *C, int M, int N, int K,
                     vg_stream_t stream);

/* One specific kernel version of the B200 ladder, 0 <= version < vg_b200_num_versions(),
 * or -1 for the per-shape choice of vg_b200_gemm_f16.
 * Replaces gemm_8192x8192_vN::launchKernel (csrc/h100/gemm_8192x8192_v*.cuh), one per
 * registered "VibeGEMM B200 vN" backend (registry.cuh:68-70 pattern). */
int vg_b200_gemm_f16_version(int version, const void *A, const void *B, void *C, int M, int N,
                             int K, vg_stream_t stream);

/* Allocation-free form of vg_b200_gemm_f16 (no counterpart in the reference).
 *
 * For callers that must not allocate device memory: programs that hand the whole GPU to
 * their own memory pool and forbid side allocations, latency-critical loops where an
 * allocation could stall or fail under memory pressure, and hosts with a device-memory
 * budget fixed at start-up. vg_b200_gemm_f16 takes the buffer for its K-padding pre-pass
 * (needed when K % 8 != 0 or A/B is not 16-byte aligned) from the CUDA stream-ordered
 * pool; this entry point uses a fixed 32 MiB array in the library's device memory
 * instead and never calls cudaMalloc, cudaMallocAsync, cudaFree or an allocating library.
 *   - Limit: the call's workspace must fit in 32 MiB: a padded copy of each operand that
 *     needs one (M * roundup(K, 8) * 2 bytes for A, N * roundup(K, 8) * 2 bytes for B), plus
 *     for small grids whose K range is split the fp32 partials of every split (splits *
 *     M * N * 4 bytes; about 19 MiB at most for the grids the per-shape choice splits), plus
 *     256 bytes for the tile counter of the versions that claim tiles at run time. Larger workspaces return
 *     VG_ERROR_NOALLOC_SCRATCH_LIMIT and launch nothing. Problems that need none of these
 *     have no size limit.
 *   - The 32 MiB belong to the library's device code. With CUDA's lazy module loading
 *     (the default) a GPU reserves them when that code is first loaded on it, i.e. at the
 *     first GEMM call of any entry point on that device, and holds them until the process
 *     exits. A host that gives all of a GPU's memory to its own pool must make one call on
 *     that device first.
 *   - The first call of this entry point on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture. A failed
 *     lookup is returned as that call's error and retried by the next call.
 *   - All calls share the array: calls that overlap on the GPU (different streams, or
 *     different host threads on one device) race on it; serialise them. Each call
 *     rewrites every scratch byte it reads and zeroes its stream-K flags and tile counter
 *     itself (cudaMemsetAsync), so nothing needs clearing between calls.
 * Same semantics, arguments and return codes as vg_b200_gemm_f16 otherwise. */
#define VG_ERROR_NOALLOC_SCRATCH_LIMIT 2001
int vg_b200_gemm_f16_noalloc(const void *A, const void *B, void *C, int M, int N, int K,
                             vg_stream_t stream);

/* GEMM on host-resident (pinned) operands with copy/compute overlap; no reference
 * counterpart (the reference engine uploads once and times device-resident launches,
 * include/engine.cuh:28-32). A pipeline owns three streams (upload, compute, download)
 * and per-row-block events. vg_host_pipeline_gemm_f16 uploads B and then A in `chunks`
 * row blocks into the caller's device buffers dA (M×K), dB (N×K), dC (M×N), runs the
 * B200 GEMM per row block as soon as it has landed, downloads each C row block as soon
 * as it is done, and makes `done_stream` wait for the last download. Consecutive calls
 * overlap (uploads of call i+1 with downloads of call i). Host buffers must be pinned and
 * are accessed asynchronously: leave hA/hB unmodified and do not read hC until
 * `done_stream` has passed the call (e.g. cudaStreamSynchronize). The calling thread's
 * current device must be the pipeline's device. Returns 0 or a cudaError_t code. */
typedef struct vg_host_pipeline *vg_host_pipeline_t;
vg_host_pipeline_t vg_host_pipeline_create(int device);
void vg_host_pipeline_destroy(vg_host_pipeline_t pipeline);
int vg_host_pipeline_gemm_f16(vg_host_pipeline_t pipeline, const void *hA, const void *hB, void *hC,
                              void *dA, void *dB, void *dC, int M, int N, int K, int chunks,
                              vg_stream_t done_stream);

/* Validation build: the same main loop as `version`, fp32 C (no fp16 rounding), so
 * accumulation error can be measured separately from output quantisation. No
 * counterpart in the reference (its only check is fp16-vs-cuBLAS,
 * include/utils.cuh:70-118). */
int vg_b200_gemm_f16_f32out(int version, const void *A, const void *B, float *C, int M, int N,
                            int K, vg_stream_t stream);

/* cuBLAS yardstick with the row-major-C operand order.
 * Replaces CublasBackend::run (csrc/cublas_backends.cu:21-35, the HAS_A100 branch
 * :28-31, which writes row-major C) — the reference engine's arbiter of correctness. */
int vg_cublas_gemm_f16(const void *A, const void *B, void *C, int M, int N, int K,
                       vg_stream_t stream);

/* Validation twin of vg_cublas_gemm_f16 with fp32 C (cublasGemmEx, C type CUDA_R_32F,
 * same compute type): cuBLAS's accumulation error next to vg_b200_gemm_f16_f32out's.
 * No reference counterpart (the reference compares fp16 outputs only,
 * include/utils.cuh:70-118). */
int vg_cublas_gemm_f16_f32out(const void *A, const void *B, float *C, int M, int N, int K,
                              vg_stream_t stream);

/* cuBLASLt heuristic sweep, the "best cuBLAS" yardstick: up to `max_algos` algorithms that
 * cublasLtMatmulAlgoGetHeuristic returns for this row-major problem (same operand order and
 * compute type as vg_cublas_gemm_f16, 64 MiB workspace), each timed on `stream` after
 * `warmup` launches over `iters` launches. ms_out[i] = mean ms per launch of algorithm i
 * (-1 if it failed), *n_out = algorithms returned. Extends the reference's cuBLAS
 * backend (csrc/cublas_backends.cu:21-35), which runs only cublasGemmEx's default choice. */
int vg_cublaslt_sweep(const void *A, const void *B, void *C, int M, int N, int K, int max_algos,
                      int warmup, int iters, float *ms_out, int *n_out, vg_stream_t stream);

/* Registry listing: replaces KernelRegistry::make_all / GemmBackend::name
 * (include/registry.cuh:23-32, include/backend.cuh:16). vg_b200_default_version() is -1
 * (per-shape choice); vg_b200_version_name(-1) is "VibeGEMM B200 auto". */
int vg_b200_num_versions(void);
const char *vg_b200_version_name(int version);
int vg_b200_default_version(void);

/* Tuning: height (in M tiles) of the grouped raster the persistent kernels walk;
 * 0 restores each version's default. The VG_RASTER_GROUP_M environment variable sets
 * the initial value. Replaces the compile-time group constants of the reference's
 * schedulers (csrc/h100/gemm_8192x8192_v18.cuh:207, TM=16). */
int vg_b200_set_raster_group(int group_m);

/* Replaces GemmBackend::is_available (include/backend.cuh:24): 1 if `device` is an
 * sm_100 part this library was built for, 0 otherwise (never throws). */
int vg_b200_is_available(int device);

/* Replaces GemmBackend::teardown (include/backend.cuh:20): drops cached tensor maps
 * and launch configuration of the calling thread. */
void vg_b200_teardown(void);

/* Failure detection (no reference counterpart; the reference only has the
 * non-fatal CUDA_TRY / cuda_check, include/utils.cuh:13-30). Every device wait in the
 * kernels is bounded by the timeout below; a wait that runs out records a nonzero
 * status word on the device and the kernel unwinds instead of hanging. */
unsigned vg_b200_device_status(int reset); /* synchronous read of the status word */
int vg_b200_set_wait_timeout_ns(unsigned long long ns); /* 0 restores the default (2 s) */
/* Launches a kernel that waits on a barrier nothing arrives on, bounded by
 * `timeout_ns`; returns 1 if the wait correctly gave up and recorded its status. */
int vg_b200_selftest_wait_timeout(unsigned long long timeout_ns);

/* Row-sharded GEMM fused with the all-gather of C (no reference counterpart; the
 * reference is single-GPU). Rank `rank` of `world` (<= 8 GPUs of one NVLink domain)
 * computes rows [row0, row0 + M_local) of C = A · B^T from its A rows (A_local, M_local×K)
 * and the replicated B, and its epilogue writes every finished C tile both into its own
 * full-size C (C_ranks[rank]) and, over NVLink, into every other rank's full-size C:
 * C_ranks[r] must be rank r's M×N C buffer mapped into this process (peer pointers, e.g.
 * from symmetric memory), N % 8 == 0 and 16-B aligned rows. If C_multicast is not NULL it
 * is the NVLink-multicast (NVLS) address of the same M×N buffers: each tile is then sent
 * once with multimem stores and the switch delivers it to every rank; otherwise one store
 * per peer. The all-gather's traffic overlaps the math tile by tile. No kernel waits on
 * another GPU: after the call, the ranks must synchronise (e.g. a barrier) before reading
 * rows written by peers. K must be positive (K == 0, an all-zero C, is rejected with
 * cudaErrorInvalidValue rather than leaving the peers' rows stale). Returns 0 or a
 * cudaError_t code. */
int vg_b200_gemm_f16_allgather(const void *A_local, const void *B, void *const *C_ranks,
                               void *C_multicast, int world, int rank, long long row0, int M_local,
                               int N, int K, vg_stream_t stream);

/* Contiguous row-block sharding used by the multi-GPU driver (A and C split by rows,
 * B replicated): rank r of `world` owns rows [row0, row0 + rows). No reference
 * counterpart (the reference is single-device, main.cu:70). */
void vg_shard_rows(long long M, int world, int rank, long long *row0, long long *rows);

/* Grouped-raster tile order used by the persistent kernels: linear tile index t ->
 * (tile_m, tile_n). Replaces Schedule::next (csrc/h100/gemm_8192x8192_v18.cuh:207-260). */
void vg_raster_tile(int t, int num_m, int num_n, int group_m, int *tile_m, int *tile_n);

/* Work units persistent worker `worker` of `workers` processes (host copy of the device
 * schedule, for tests): data-parallel (stream_k = 0: whole tiles in grouped-raster order;
 * with splits > 1, split-K: tile × K-split units, unit u = tile u % T over the K range of
 * split u / T), stream-K (stream_k = 1: an equal share of the (tile, k-block)
 * iterations) or contiguous runs (stream_k = 2, the A-resident kernel: tiles
 * [w·T/P, (w+1)·T/P) in row-major order). Writes up to max_units records of 8 ints {tile_m, tile_n, kb0, kb1, kind (0
 * whole tile or split, 1 partial written to the workspace, 2 owner that adds the partials
 * of workers first..last), first_contrib, last_contrib, split} and returns the number of
 * units (-1 on bad input). Replaces the tile walk of Schedule::next
 * (csrc/h100/gemm_8192x8192_v18.cuh:207-260). */
int vg_work_units(int stream_k, int worker, int workers, int num_m, int num_n, int group_m,
                  int num_kb, int splits, int *out, int max_units);

/* Host-side launch plan for a problem, as the launcher would build it for a device
 * with `num_sms` SMs (exposed so the planner can be tested without a GPU).
 * `version` may be -1 (per-shape choice). `mode`: 0 = fp16 C (vg_b200_gemm_f16),
 * 1 = fp32 C (vg_b200_gemm_f16_f32out), 2 = fp16 C with the fused all-gather
 * (vg_b200_gemm_f16_allgather, whose per-shape choice excludes stream-K).
 * Fields of `out` (int[20]): cta_group, stages, epilogue kind (0 TMA fp16, 1 direct fp16,
 * 2 direct fp32, 3 TMA fp16 + peer stores, 4 staged fp16 with coalesced row stores for C
 * rows TMA cannot describe, 5 split-K: fp32 partials then a reduction kernel writing fp16
 * C), pad_a, pad_b, padded K, num_m_tiles, num_n_tiles, num_kb, group_m, grid (CTAs),
 * persistent, tile columns, resolved version, stream-K, promote (chunked accumulation
 * with an fp32 running sum), dyn (tiles claimed at run time), k-blocks of 64 per
 * accumulation chunk (num_kb: one chunk), split-K parts (1: none), A resident in shared
 * memory over contiguous tile runs (v12 with K <= 256; then `stages` counts B stages).
 * Returns 0 or a cudaError_t code. */
int vg_b200_plan(int version, int M, int N, int K, uintptr_t A, uintptr_t B, uintptr_t C,
                 int mode, int num_sms, int *out);

/* Reference-facing plugin path: runs registered backend `name` (e.g. "cuBLAS",
 * "VibeGEMM B200 v2") through GemmBackend::run on the legacy default stream.
 * Returns cudaErrorInvalidValue if no backend has that name. */
int vg_backend_count(void);
const char *vg_backend_name(int i);
int vg_backend_run(const char *name, void *A, void *B, void *C, int M, int N, int K);

/* The reference engine (include/engine.cuh) run over every registered backend for
 * one shape: reference = cuBLAS, 10 warm-up + 30 timed launches, then the
 * element-wise check (replaces BenchmarkEngine::execute, include/engine.cuh:20-86).
 * `inputs`: 0 = uniform[-1,1] (seeds 42/77, the reference's), 1 = N(0, 0.02).
 * `log_path` may be NULL. Results of the last call are readable per backend. */
int vg_engine_execute(int M, int N, int K, int inputs, const char *log_path);
int vg_engine_result_count(void);
/* out: [avg_ms, tflops, max_abs_err, max_rel_err, passed(0/1), skipped(0/1)] */
int vg_engine_result(int i, char *name_buf, int name_len, double *out);

#ifdef __cplusplus
}
#endif

#endif /* VIBEGEMM_B200_H */
