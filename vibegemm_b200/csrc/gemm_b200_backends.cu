// B200 backend family: adapts each kernel version's launchKernel to GemmBackend and
// registers it, exactly as the reference wires its H100 family
// (csrc/gemm_h100_backends.cu:34-57): a template adapter over a free function
// void launchKernel(half*, half*, half*, int, int, int), one registration per
// version, display names "VibeGEMM B200 vN".
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <string>

#include "backend.cuh"
#include "registry.cuh"
#include "vibegemm_b200.h"

namespace {

// Launch on the legacy default stream, where the engine records its events
// (include/engine.cuh timing, include/utils.cuh CudaTimer). Host-side errors
// (unsupported device, bad sizes) are reported on stderr; device-side errors surface
// at the engine's next cuda_check().
template <int V> void launch_version(half *A, half *B, half *C, int M, int N, int K) {
    const int e = vg_b200_gemm_f16_version(V, A, B, C, M, N, K, nullptr);
    if (e != 0)
        std::fprintf(stderr, "%s: launch failed: %s\n", vg_b200_version_name(V),
                     cudaGetErrorString((cudaError_t)e));
}

} // namespace

namespace gemm_b200_v0 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<0>(A, B, C, M, N, K); }
} // namespace gemm_b200_v0
namespace gemm_b200_v1 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<1>(A, B, C, M, N, K); }
} // namespace gemm_b200_v1
namespace gemm_b200_v2 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<2>(A, B, C, M, N, K); }
} // namespace gemm_b200_v2
namespace gemm_b200_v3 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<3>(A, B, C, M, N, K); }
} // namespace gemm_b200_v3
namespace gemm_b200_v4 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<4>(A, B, C, M, N, K); }
} // namespace gemm_b200_v4
namespace gemm_b200_v5 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<5>(A, B, C, M, N, K); }
} // namespace gemm_b200_v5
namespace gemm_b200_v6 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<6>(A, B, C, M, N, K); }
} // namespace gemm_b200_v6
namespace gemm_b200_v7 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<7>(A, B, C, M, N, K); }
} // namespace gemm_b200_v7
namespace gemm_b200_v8 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<8>(A, B, C, M, N, K); }
} // namespace gemm_b200_v8
namespace gemm_b200_v9 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<9>(A, B, C, M, N, K); }
} // namespace gemm_b200_v9
namespace gemm_b200_v10 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<10>(A, B, C, M, N, K); }
} // namespace gemm_b200_v10
namespace gemm_b200_v11 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<11>(A, B, C, M, N, K); }
} // namespace gemm_b200_v11
namespace gemm_b200_v12 {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<12>(A, B, C, M, N, K); }
} // namespace gemm_b200_v12
// The default entry point: one of the versions above, chosen per shape.
namespace gemm_b200_auto {
void launchKernel(half *A, half *B, half *C, int M, int N, int K) { launch_version<-1>(A, B, C, M, N, K); }
} // namespace gemm_b200_auto

using KernelFn = void (*)(half *, half *, half *, int, int, int);

template <KernelFn Fn> class GeneratedB200KernelBackend : public GemmBackend {
  public:
    explicit GeneratedB200KernelBackend(std::string backend_name)
        : backend_name_(std::move(backend_name)) {}

    void run(half *A, half *B, half *C, int M, int N, int K) override { Fn(A, B, C, M, N, K); }
    std::string name() const override { return backend_name_; }
    void teardown() override { vg_b200_teardown(); }
    bool is_available() const override {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) {
            (void)cudaGetLastError();
            return false;
        }
        return vg_b200_is_available(dev) != 0;
    }

  private:
    std::string backend_name_;
};

REGISTER_B200_KERNEL("VibeGEMM B200 v0", GeneratedB200KernelBackend<gemm_b200_v0::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v1", GeneratedB200KernelBackend<gemm_b200_v1::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v2", GeneratedB200KernelBackend<gemm_b200_v2::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v3", GeneratedB200KernelBackend<gemm_b200_v3::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v4", GeneratedB200KernelBackend<gemm_b200_v4::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v5", GeneratedB200KernelBackend<gemm_b200_v5::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v6", GeneratedB200KernelBackend<gemm_b200_v6::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v7", GeneratedB200KernelBackend<gemm_b200_v7::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v8", GeneratedB200KernelBackend<gemm_b200_v8::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v9", GeneratedB200KernelBackend<gemm_b200_v9::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v10", GeneratedB200KernelBackend<gemm_b200_v10::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v11", GeneratedB200KernelBackend<gemm_b200_v11::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 v12", GeneratedB200KernelBackend<gemm_b200_v12::launchKernel>);
REGISTER_B200_KERNEL("VibeGEMM B200 auto", GeneratedB200KernelBackend<gemm_b200_auto::launchKernel>);
