// Interface of VibeGEMM's include/backend.cuh (AnonymousSC2026/VibeGEMM, GNU General Public
// License v3.0), kept identical so backends drop in; see NOTICE.
//
// GemmBackend — the plugin interface every GEMM implementation is registered behind.
//
// Kept interface-identical to the reference (include/backend.cuh:7-25 of VibeGEMM) so
// that a B200 backend is a drop-in registration: same virtual methods, same argument
// meaning, same ownership rules. Only the comments and this file's code are new.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <string>

class GemmBackend {
  public:
    virtual ~GemmBackend() = default;

    // C = A · B^T for A M×K row-major, B stored N×K (K contiguous), C M×N row-major,
    // fp32 accumulation, fp16 output (alpha = 1, beta = 0). The caller owns all three
    // device buffers; the backend launches asynchronously on the legacy default stream.
    virtual void run(half *A, half *B, half *C, int M, int N, int K) = 0;

    // Display name used in the benchmark report.
    virtual std::string name() const = 0;

    // Release per-shape resources (cached descriptors, workspaces). Called by the
    // engine after each backend finishes a problem size.
    virtual void teardown() {}

    // false → the engine prints [SKIP] and does not run this backend.
    virtual bool is_available() const { return true; }
};
