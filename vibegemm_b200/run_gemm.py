"""Run one GEMM shape on one GPU: a few timed launches plus a check against cuBLAS.

    python -m vibegemm_b200.run_gemm --M 8192 --N 8192 --K 8192 [--version 2] [--iters 3]
                                     [--warmup 2] [--dist uniform|normal] [--backend b200|cublas]

Used to profile a single kernel (e.g. under ncu with -k/-c) and to spot-check shapes.
Prints one JSON line: ms per launch (CUDA events), TFLOP/s, max |C - C_cuBLAS|.
"""
from __future__ import annotations

import argparse
import json


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=8192)
    ap.add_argument("--N", type=int, default=8192)
    ap.add_argument("--K", type=int, default=8192)
    ap.add_argument("--version", type=int, default=None)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--dist", choices=["uniform", "normal"], default="uniform")
    ap.add_argument("--backend", choices=["b200", "cublas"], default="b200")
    ap.add_argument("--no-check", action="store_true")
    a = ap.parse_args()

    import torch

    import vibegemm_b200 as vg

    g = torch.Generator(device="cuda")
    g.manual_seed(42)
    A = torch.empty((a.M, a.K), dtype=torch.float16, device="cuda")
    B = torch.empty((a.N, a.K), dtype=torch.float16, device="cuda")
    if a.dist == "uniform":
        A.uniform_(-1, 1, generator=g)
        B.uniform_(-1, 1, generator=g)
    else:
        A.normal_(0, 0.02, generator=g)
        B.normal_(0, 0.02, generator=g)
    C = torch.empty((a.M, a.N), dtype=torch.float16, device="cuda")

    def launch():
        if a.backend == "b200":
            vg.gemm(A, B, out=C, version=a.version)
        else:
            vg.cublas_gemm(A, B, out=C)

    for _ in range(a.warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        launch()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / max(1, a.iters)
    out = {"M": a.M, "N": a.N, "K": a.K, "backend": a.backend,
           "version": vg.default_version() if a.version is None else a.version,
           "ms": ms, "tflops": 2.0 * a.M * a.N * a.K / (ms * 1e-3) / 1e12,
           "device_status": vg.device_status()}
    if not a.no_check and a.backend == "b200":
        R = vg.cublas_gemm(A, B)
        torch.cuda.synchronize()
        d = (C.float() - R.float()).abs()
        out["max_abs_vs_cublas"] = float(d.max())
        out["mismatches_vs_cublas"] = int((d > 1e-3 + 1e-2 * R.float().abs()).sum())
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
