// ORACLE pinning shim (test infrastructure only): compiles the reference's own GPU
// pieces for sm_100a into oracle/_ref/libvgref_gpu.so so that tests (and the
// golden-fixture generator) can run them on a B200 beside the product kernels:
//  * the naive scalar kernel csrc/a100/gemm_8192x8192_v0.cuh:23-82 (plain CUDA, no
//    mma.sync) — sequential-k fp32 accumulation, the semantics the oracle restates;
//  * CublasBackend from csrc/cublas_backends.cu:12-44 with HAS_A100 (the row-major-C
//    operand order, :28-31) — the reference engine's arbiter of correctness;
//  * fill_random_fp16 from include/utils.cuh:59-66 on a real device buffer.
// The reference files are included from the reference tree at build time; nothing
// is copied into this repository.
#include "include/utils.cuh"
#include "csrc/a100/gemm_8192x8192_v0.cuh"

#ifndef HAS_A100
#define HAS_A100
#endif
#include "csrc/cublas_backends.cu"

extern "C" int vgref_naive_gemm(void *A, void *B, void *C, int M, int N, int K) {
    gemm_8192x8192_v0::launchKernel(static_cast<half *>(A), static_cast<half *>(B),
                                    static_cast<half *>(C), M, N, K);
    return (int)cudaDeviceSynchronize();
}

extern "C" int vgref_cublas_gemm(void *A, void *B, void *C, int M, int N, int K) {
    static CublasBackend *backend = new CublasBackend();
    backend->run(static_cast<half *>(A), static_cast<half *>(B), static_cast<half *>(C), M, N, K);
    return (int)cudaDeviceSynchronize();
}

extern "C" int vgref_fill_random_fp16_device(void *d_ptr, size_t n, unsigned seed) {
    return fill_random_fp16(static_cast<half *>(d_ptr), n, seed) ? 0 : 1;
}
