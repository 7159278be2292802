"""Sustained throughput under the power cap: one shape, several kernels, seconds each.

    python -m vibegemm_b200.sustained --shape 8192x8192x8192 --seconds 2 \\
        --kernels cublas,v3,v2,v6,auto,cublas [--raster-group 16]

Each kernel runs back to back for about `--seconds` after 3 s of idle (so every kernel starts
from a similar thermal state), with CUDA events every tenth of the run and NVML samples of
board power, SM clock and the active clock-event reasons every 10 ms. "steady" is the mean
TFLOP/s over the second half of the run. One JSON line per kernel. Kernel names: `cublas`,
`auto` (the default entry point's per-shape choice) or `vN` (ladder version N).
"""
from __future__ import annotations

import argparse
import json
import statistics
import threading
import time


def _sampler(handle, nvml, stop, out):
    while not stop.is_set():
        reasons = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
        out.append((nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0,
                    nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM), reasons))
        time.sleep(0.01)


def _reason_names(mask: int, nvml) -> list[str]:
    names = {"sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
             "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
             "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
             "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown"}
    return [k for k, attr in names.items() if mask & getattr(nvml, attr, 0)]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="8192x8192x8192")
    ap.add_argument("--seconds", type=float, default=2.0)
    ap.add_argument("--kernels", default="cublas,auto,cublas")
    ap.add_argument("--raster-group", type=int, default=0, help="0 = each version's default")
    a = ap.parse_args()

    import pynvml as nvml
    import torch

    import vibegemm_b200 as vg

    M, N, K = map(int, a.shape.split("x"))
    nvml.nvmlInit()
    dev = torch.cuda.current_device()
    # NVML numbers devices physically; match this CUDA device by UUID.
    uuid = str(torch.cuda.get_device_properties(dev).uuid).replace("GPU-", "")
    handle = None
    for i in range(nvml.nvmlDeviceGetCount()):
        h = nvml.nvmlDeviceGetHandleByIndex(i)
        u = nvml.nvmlDeviceGetUUID(h)
        if uuid in (u.decode() if isinstance(u, bytes) else u):
            handle = h
    if handle is None:
        raise RuntimeError("no NVML device matches the CUDA device")
    g = torch.Generator(device="cuda")
    g.manual_seed(42)
    A = torch.empty((M, K), dtype=torch.float16, device="cuda").uniform_(-1, 1, generator=g)
    B = torch.empty((N, K), dtype=torch.float16, device="cuda").uniform_(-1, 1, generator=g)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    vg.set_raster_group(a.raster_group)

    def kernel(name: str):
        if name == "cublas":
            return lambda: vg.cublas_gemm(A, B, out=C)
        version = None if name == "auto" else int(name.lstrip("v"))
        return lambda: vg.gemm(A, B, out=C, version=version)

    for name in a.kernels.split(","):
        fn = kernel(name)
        torch.cuda.synchronize()
        time.sleep(3.0)
        fn()
        torch.cuda.synchronize()
        t0 = time.time()
        fn()
        torch.cuda.synchronize()
        one = time.time() - t0
        iters = max(10, int(a.seconds / max(one, 1e-4)))
        window = max(1, iters // 10)
        events = [torch.cuda.Event(enable_timing=True) for _ in range(iters // window + 1)]
        stop, samples = threading.Event(), []
        th = threading.Thread(target=_sampler, args=(handle, nvml, stop, samples))
        th.start()
        events[0].record()
        for i in range(iters):
            fn()
            if (i + 1) % window == 0:
                events[(i + 1) // window].record()
        torch.cuda.synchronize()
        stop.set()
        th.join()
        ms = [events[j].elapsed_time(events[j + 1]) / window for j in range(len(events) - 1)]
        tf = [2.0 * M * N * K / (x * 1e-3) / 1e12 for x in ms]
        reasons = set()
        for s in samples:
            reasons.update(_reason_names(s[2], nvml))
        print(json.dumps({
            "shape": a.shape, "kernel": name, "iters": iters,
            "version": None if name == "cublas" else vg.plan(-1 if name == "auto" else int(name.lstrip("v")),
                                                              M, N, K, 256, 256, 256)["version"],
            "first_tflops": round(tf[0], 1), "steady_tflops": round(statistics.mean(tf[len(tf) // 2:]), 1),
            "sm_mhz_median": statistics.median(s[1] for s in samples),
            "power_w_mean": round(statistics.mean(s[0] for s in samples), 1),
            "reasons": sorted(reasons)}), flush=True)
    vg.set_raster_group(0)


if __name__ == "__main__":
    main()
