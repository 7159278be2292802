"""VibeGEMM-B200: FP16 GEMM (fp32 accumulate, fp16 out) for NVIDIA B200 (sm_100a).

Python bindings over the C ABI in ``include/vibegemm_b200.h`` (``libvibegemm_b200.so``,
built in-tree by :mod:`vibegemm_b200.build`). Device buffers are torch tensors; the
kernels themselves are the hand-written tcgen05/TMA kernels of the library. There is no
fallback: if the library is missing, :func:`lib` raises, and every GEMM entry point
requires CUDA tensors.

Layout convention (the reference's): ``A`` is M×K row-major, ``B`` is stored N×K
(K contiguous), ``C = A @ B.T`` is M×N row-major.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libvibegemm_b200.so"
_lib: Optional[ctypes.CDLL] = None

# Names exported by the C ABI (include/vibegemm_b200.h), with their signatures.
_SIGS = {
    "vg_b200_gemm_f16": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]),
    "vg_b200_gemm_f16_version": (ctypes.c_int, [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]),
    "vg_b200_gemm_f16_f32out": (ctypes.c_int, [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]),
    "vg_b200_gemm_f16_noalloc": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]),
    "vg_cublas_gemm_f16": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]),
    "vg_cublas_gemm_f16_f32out": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]),
    "vg_cublaslt_sweep": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 6
                          + [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]),
    "vg_b200_num_versions": (ctypes.c_int, []),
    "vg_b200_version_name": (ctypes.c_char_p, [ctypes.c_int]),
    "vg_b200_default_version": (ctypes.c_int, []),
    "vg_b200_is_available": (ctypes.c_int, [ctypes.c_int]),
    "vg_b200_teardown": (None, []),
    "vg_b200_device_status": (ctypes.c_uint, [ctypes.c_int]),
    "vg_b200_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_ulonglong]),
    "vg_b200_set_raster_group": (ctypes.c_int, [ctypes.c_int]),
    "vg_b200_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_ulonglong]),
    "vg_shard_rows": (None, [ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                             ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong)]),
    "vg_raster_tile": (None, [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int)] * 2),
    "vg_work_units": (ctypes.c_int, [ctypes.c_int] * 8 + [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "vg_b200_plan": (ctypes.c_int, [ctypes.c_int] * 4 + [ctypes.c_size_t] * 3 + [ctypes.c_int] * 2
                     + [ctypes.POINTER(ctypes.c_int)]),
    "vg_b200_gemm_f16_allgather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                   ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_longlong,
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_void_p]),
    "vg_host_pipeline_create": (ctypes.c_void_p, [ctypes.c_int]),
    "vg_host_pipeline_destroy": (None, [ctypes.c_void_p]),
    "vg_host_pipeline_gemm_f16": (ctypes.c_int, [ctypes.c_void_p] * 7 + [ctypes.c_int] * 4 + [ctypes.c_void_p]),
    "vg_backend_count": (ctypes.c_int, []),
    "vg_backend_name": (ctypes.c_char_p, [ctypes.c_int]),
    "vg_backend_run": (ctypes.c_int, [ctypes.c_char_p] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3),
    "vg_engine_execute": (ctypes.c_int, [ctypes.c_int] * 4 + [ctypes.c_char_p]),
    "vg_engine_result_count": (ctypes.c_int, []),
    "vg_engine_result": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_double)]),
}
EXPORTED_SYMBOLS = tuple(_SIGS)

PLAN_FIELDS = ("cta_group", "stages", "epilogue", "pad_a", "pad_b", "k_padded", "num_m_tiles",
               "num_n_tiles", "num_kb", "group_m", "grid", "persistent", "tile_n", "version", "stream_k",
               "promote", "dyn", "promote_kb", "splits", "a_resident")
EPILOGUES = {0: "tma_f16", 1: "direct_f16", 2: "direct_f32", 3: "tma_f16_peers", 4: "staged_f16",
             5: "splitk_f16"}


class VibeGemmError(RuntimeError):
    """A C-ABI call returned a nonzero status (a cudaError_t code, or 1000 + cuBLAS status)."""

    def __init__(self, what: str, code: int):
        super().__init__(f"{what} failed with status {code}")
        self.code = code


def lib() -> ctypes.CDLL:
    """The loaded C library. Raises ImportError when it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("VIBEGEMM_B200_LIB", LIB_PATH))
        if not path.exists():
            raise ImportError(f"{path} is missing: build it with `python -m vibegemm_b200.build` "
                              "(there is no fallback implementation)")
        handle = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(code: int, what: str) -> None:
    if code != 0:
        raise VibeGemmError(what, code)


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream or None
    if isinstance(stream, int):
        return stream or None
    return stream.cuda_stream or None


def _operands(A, B, out, out_dtype):
    import torch
    if not (A.is_cuda and B.is_cuda):
        raise ValueError("A and B must be CUDA tensors (no CPU path)")
    if A.dtype != torch.float16 or B.dtype != torch.float16:
        raise TypeError("A and B must be float16")
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
        raise ValueError(f"expected A[M,K] and B[N,K], got {tuple(A.shape)} and {tuple(B.shape)}")
    if not (A.is_contiguous() and B.is_contiguous()):
        raise ValueError("A and B must be contiguous (row-major)")
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=A.device)
    elif out.shape != (M, N) or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [M, N] tensor of the output dtype")
    return int(M), int(N), int(K), out


def gemm(A, B, out=None, version: Optional[int] = None, stream=None):
    """C = A @ B.T on the B200 kernel (`version` of the ladder, default = fastest)."""
    import torch
    M, N, K, out = _operands(A, B, out, torch.float16)
    s = _stream_handle(stream)
    if version is None:
        code = lib().vg_b200_gemm_f16(A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K, s)
    else:
        code = lib().vg_b200_gemm_f16_version(version, A.data_ptr(), B.data_ptr(), out.data_ptr(),
                                              M, N, K, s)
    _check(code, "vg_b200_gemm_f16")
    return out


NOALLOC_SCRATCH_LIMIT = 2001  # VG_ERROR_NOALLOC_SCRATCH_LIMIT


def gemm_noalloc(A, B, out=None, stream=None):
    """vg_b200_gemm_f16 without any device allocation: the K-padding workspace is a fixed
    32 MiB array in the library (problems whose padded copies exceed it raise
    VibeGemmError with code NOALLOC_SCRATCH_LIMIT). Overlapping calls on one GPU race on
    that array; the caller must allocate `out` itself to avoid torch's allocator."""
    import torch
    M, N, K, out = _operands(A, B, out, torch.float16)
    code = lib().vg_b200_gemm_f16_noalloc(A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K,
                                          _stream_handle(stream))
    _check(code, "vg_b200_gemm_f16_noalloc")
    return out


def gemm_f32out(A, B, out=None, version: Optional[int] = None, stream=None):
    """Validation build: same main loop, fp32 C (no output rounding)."""
    import torch
    M, N, K, out = _operands(A, B, out, torch.float32)
    v = default_version() if version is None else version
    code = lib().vg_b200_gemm_f16_f32out(v, A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K,
                                         _stream_handle(stream))
    _check(code, "vg_b200_gemm_f16_f32out")
    return out


def cublas_gemm(A, B, out=None, stream=None):
    """The cuBLAS yardstick (cublasGemmEx, COMPUTE_32F, row-major C)."""
    import torch
    M, N, K, out = _operands(A, B, out, torch.float16)
    code = lib().vg_cublas_gemm_f16(A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K,
                                    _stream_handle(stream))
    _check(code, "vg_cublas_gemm_f16")
    return out


def cublas_gemm_f32out(A, B, out=None, stream=None):
    """cuBLAS with fp32 C (validation: its accumulation error beside gemm_f32out's)."""
    import torch
    M, N, K, out = _operands(A, B, out, torch.float32)
    code = lib().vg_cublas_gemm_f16_f32out(A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K,
                                           _stream_handle(stream))
    _check(code, "vg_cublas_gemm_f16_f32out")
    return out


def cublaslt_sweep(A, B, out=None, max_algos: int = 16, warmup: int = 3, iters: int = 10,
                   stream=None) -> list[float]:
    """Mean ms per launch of each cuBLASLt heuristic algorithm for C = A @ B.T (-1 = failed)."""
    import torch
    M, N, K, out = _operands(A, B, out, torch.float16)
    ms = (ctypes.c_float * max_algos)()
    n = ctypes.c_int(0)
    code = lib().vg_cublaslt_sweep(A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K, max_algos,
                                   warmup, iters, ms, ctypes.byref(n), _stream_handle(stream))
    _check(code, "vg_cublaslt_sweep")
    return [float(ms[i]) for i in range(n.value)]


AUTO = -1  # per-shape version choice (the default entry point's policy)


def gemm_allgather(A_local, B, c_rank_ptrs, rank: int, row0: int, stream=None,
                   c_multicast_ptr: int = 0) -> None:
    """Fused row-sharded GEMM + all-gather: writes C rows [row0, row0+M_local) into every
    rank's full C (`c_rank_ptrs[r]`, device pointers valid in this process; with
    `c_multicast_ptr` through NVLink multicast instead). Barrier across ranks before reading
    rows written by peers."""
    import torch
    if not (A_local.is_cuda and B.is_cuda) or A_local.dtype != torch.float16 or B.dtype != torch.float16:
        raise ValueError("A_local and B must be float16 CUDA tensors")
    M_local, K = A_local.shape
    N = B.shape[0]
    arr = (ctypes.c_void_p * len(c_rank_ptrs))(*c_rank_ptrs)
    code = lib().vg_b200_gemm_f16_allgather(A_local.data_ptr(), B.data_ptr(), arr,
                                            c_multicast_ptr or None, len(c_rank_ptrs), rank, row0,
                                            M_local, N, K, _stream_handle(stream))
    _check(code, "vg_b200_gemm_f16_allgather")


class HostPipeline:
    """C = A @ B.T for pinned HOST tensors, overlapping uploads, GEMMs and downloads.

    Owns the device buffers (grown on demand) and the C pipeline (three streams). Each
    call enqueues the work and makes `stream` (default: current) wait for the result;
    synchronise that stream before reading `out`. The copies run after the call returns,
    so the wrapper keeps every call's host tensors alive until an event recorded on
    `stream` after the call has completed (torch would otherwise recycle a freed pinned
    block while the library's upload still reads it).
    """

    def __init__(self, device: Optional[int] = None, chunks: int = 4):
        import torch
        self.device = torch.cuda.current_device() if device is None else device
        self.chunks = chunks
        self._h = lib().vg_host_pipeline_create(self.device)
        if not self._h:
            raise VibeGemmError("vg_host_pipeline_create", -1)
        self._bufs = {}
        self._in_flight = []  # (event, host tensors) of calls that may still be copying

    def _buf(self, name, shape):
        import torch
        t = self._bufs.get(name)
        if t is None or t.shape != shape:
            t = torch.empty(shape, dtype=torch.float16, device=f"cuda:{self.device}")
            self._bufs[name] = t
        return t

    def gemm(self, A, B, out, stream=None):
        M, K = A.shape
        N = B.shape[0]
        if A.is_cuda or B.is_cuda or out.is_cuda:
            raise ValueError("HostPipeline takes host tensors")
        if not (A.is_pinned() and B.is_pinned() and out.is_pinned()):
            raise ValueError("host tensors must be pinned (pin_memory=True)")
        dA, dB, dC = self._buf("A", (M, K)), self._buf("B", (N, K)), self._buf("C", (M, N))
        import torch
        self._in_flight = [(ev, keep) for ev, keep in self._in_flight if not ev.query()]
        code = lib().vg_host_pipeline_gemm_f16(self._h, A.data_ptr(), B.data_ptr(), out.data_ptr(),
                                               dA.data_ptr(), dB.data_ptr(), dC.data_ptr(),
                                               M, N, K, self.chunks, _stream_handle(stream))
        _check(code, "vg_host_pipeline_gemm_f16")
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream() if stream is None else stream)
        self._in_flight.append((ev, (A, B, out)))
        return out

    def close(self):
        if self._h:
            lib().vg_host_pipeline_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def versions() -> list[str]:
    L = lib()
    return [L.vg_b200_version_name(i).decode() for i in range(L.vg_b200_num_versions())]


def version_name(version: int) -> str:
    n = lib().vg_b200_version_name(version)
    if n is None:
        raise ValueError(f"no kernel version {version}")
    return n.decode()


def default_version() -> int:
    """-1: the default entry point chooses a version per shape."""
    return int(lib().vg_b200_default_version())


def is_available(device: int = 0) -> bool:
    return bool(lib().vg_b200_is_available(device))


def teardown() -> None:
    lib().vg_b200_teardown()


def device_status(reset: bool = False) -> int:
    return int(lib().vg_b200_device_status(1 if reset else 0))


def set_wait_timeout_ns(ns: int) -> None:
    lib().vg_b200_set_wait_timeout_ns(ns)


def set_raster_group(group_m: int) -> None:
    """Raster group height (M tiles) for the persistent kernels; 0 = version default."""
    _check(lib().vg_b200_set_raster_group(group_m), "vg_b200_set_raster_group")


def selftest_wait_timeout(timeout_ns: int) -> bool:
    return bool(lib().vg_b200_selftest_wait_timeout(timeout_ns))


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    r0, n = ctypes.c_longlong(), ctypes.c_longlong()
    lib().vg_shard_rows(M, world, rank, ctypes.byref(r0), ctypes.byref(n))
    return int(r0.value), int(n.value)


def raster_tile(t: int, num_m: int, num_n: int, group_m: int) -> tuple[int, int]:
    tm, tn = ctypes.c_int(), ctypes.c_int()
    lib().vg_raster_tile(t, num_m, num_n, group_m, ctypes.byref(tm), ctypes.byref(tn))
    return int(tm.value), int(tn.value)


UNIT_KINDS = {0: "full", 1: "partial", 2: "owner"}


def work_units(stream_k: int, worker: int, workers: int, num_m: int, num_n: int, group_m: int,
               num_kb: int, splits: int = 1) -> list[dict]:
    """The units a persistent worker processes (host copy of the device schedule). `stream_k`:
    0 (or False) grouped raster / split-K, 1 (or True) stream-K, 2 contiguous runs."""
    L = lib()
    n = L.vg_work_units(int(stream_k), worker, workers, num_m, num_n, group_m, num_kb, splits, None, 0)
    if n < 0:
        raise ValueError("bad schedule arguments")
    buf = (ctypes.c_int * (8 * max(n, 1)))()
    L.vg_work_units(int(stream_k), worker, workers, num_m, num_n, group_m, num_kb, splits, buf, n)
    keys = ("tile_m", "tile_n", "kb0", "kb1", "kind", "first_contrib", "last_contrib", "split")
    out = []
    for i in range(n):
        d = dict(zip(keys, buf[8 * i: 8 * i + 8]))
        d["kind"] = UNIT_KINDS[d["kind"]]
        out.append(d)
    return out


def plan(version: int, M: int, N: int, K: int, a_ptr: int = 0, b_ptr: int = 0, c_ptr: int = 0,
         f32_out: bool = False, num_sms: int = 148, allgather: bool = False) -> dict:
    """Launch plan of vg_b200_plan (mode 1 = fp32 C, 2 = fused all-gather epilogue)."""
    out = (ctypes.c_int * len(PLAN_FIELDS))()
    mode = 2 if allgather else int(bool(f32_out))
    _check(lib().vg_b200_plan(version, M, N, K, a_ptr, b_ptr, c_ptr, mode, num_sms, out),
           "vg_b200_plan")
    d = dict(zip(PLAN_FIELDS, list(out)))
    d["epilogue"] = EPILOGUES[d["epilogue"]]
    return d


def backends() -> list[str]:
    L = lib()
    return [L.vg_backend_name(i).decode() for i in range(L.vg_backend_count())]


def backend_run(name: str, A, B, C) -> None:
    """Run registered backend `name` through GemmBackend::run (legacy default stream)."""
    M, K = A.shape
    N = B.shape[0]
    _check(lib().vg_backend_run(name.encode(), A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K),
           f"backend {name!r}")


def engine_execute(M: int, N: int, K: int, inputs: str = "uniform",
                   log_path: Optional[str] = None) -> list[dict]:
    """BenchmarkEngine::execute over every registered backend; returns per-backend results."""
    L = lib()
    _check(L.vg_engine_execute(M, N, K, 1 if inputs == "normal" else 0,
                               log_path.encode() if log_path else None), "vg_engine_execute")
    res = []
    buf = ctypes.create_string_buffer(256)
    vals = (ctypes.c_double * 6)()
    for i in range(L.vg_engine_result_count()):
        _check(L.vg_engine_result(i, buf, 256, vals), "vg_engine_result")
        res.append({"name": buf.value.decode(), "avg_ms": vals[0], "tflops": vals[1],
                    "max_abs_err": vals[2], "max_rel_err": vals[3], "passed": bool(vals[4]),
                    "skipped": bool(vals[5])})
    return res
