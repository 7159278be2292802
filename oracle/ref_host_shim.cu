// ORACLE pinning shim (test infrastructure only): compiles the reference's own host
// helpers — fill_random_fp16 and check_error from include/utils.cuh:59-118 of VibeGEMM —
// straight from the reference source tree into oracle/_ref/libvgref_host.so.
//
// Those helpers move data with cudaMemcpy (H2D in fill_random_fp16, D2H in
// check_error). Here cudaMemcpy is redirected to a host memcpy for the duration of
// the #include, so the reference's generator and checker run unmodified on host
// buffers and need no GPU. The resulting outputs pin the oracle's restatement.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

static cudaError_t vgref_host_copy(void *dst, const void *src, size_t n, cudaMemcpyKind) {
    std::memcpy(dst, src, n);
    return cudaSuccess;
}

#define cudaMemcpy vgref_host_copy
#include "include/utils.cuh"
#undef cudaMemcpy

extern "C" int vgref_fill_random_fp16(uint16_t *out, size_t n, unsigned seed) {
    return fill_random_fp16(reinterpret_cast<half *>(out), n, seed) ? 0 : 1;
}

extern "C" int vgref_check_error(const uint16_t *ref, const uint16_t *cmp, size_t n, float atol,
                                 float rtol) {
    return check_error(reinterpret_cast<half *>(const_cast<uint16_t *>(ref)),
                       reinterpret_cast<half *>(const_cast<uint16_t *>(cmp)), n, atol, rtol, 0)
               ? 1
               : 0;
}
