"""ORACLE — TEST INFRASTRUCTURE ONLY.

CPU restatement of the reference (AnonymousSC2026/VibeGEMM) FP16 GEMM path, used as the
checker by ``tests/``, ``__graft_entry__.smoke()`` and as the timed CPU baseline in
``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm). The product library
never imports, links or calls anything here.

* ``liboracle.so`` (``gemm_oracle.cpp``): input generation (include/utils.cuh:59-66),
  the naive sequential-k GEMM (csrc/a100/gemm_8192x8192_v0.cuh:23-74,
  csrc/h100/gemm_8192x8192_v8.cuh:347-358) and check_error (include/utils.cuh:70-118).
* ``_ref/libvgref_host.so``: the reference's own fill_random_fp16 / check_error, compiled
  from the reference tree (host copies instead of cudaMemcpy) — pins the restatement.
* ``_ref/libvgref_gpu.so``: the reference's naive v0 kernel and its cuBLAS backend,
  compiled for sm_100a — pins the restatement on a B200 and generates golden fixtures.

Parity status: pinned — input generation and check_error against the reference's own
code (``_ref``), and the GEMM against golden outputs of the reference's v0 kernel
(``tests/golden/``).
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_HOST_PATH = HERE / "_ref" / "libvgref_host.so"
REF_GPU_PATH = HERE / "_ref" / "libvgref_gpu.so"

_lib: Optional[ctypes.CDLL] = None
_u16p = ctypes.POINTER(ctypes.c_uint16)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} missing: run `make -C oracle`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_fill_uniform_f16.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint]
        L.oracle_fill_normal_f16.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint,
                                             ctypes.c_float, ctypes.c_float]
        for name in ("oracle_gemm_f16", "oracle_gemm_f32", "oracle_gemm_f64"):
            getattr(L, name).argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_long] * 5 + [ctypes.c_int]
        L.oracle_check_error.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_float, ctypes.c_float, ctypes.c_void_p]
        L.oracle_check_error.restype = ctypes.c_int
        L.oracle_f32_to_f16_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def fill_uniform_f16(n: int, seed: int) -> np.ndarray:
    """uniform[-1,1] fp16 bit patterns (uint16), the reference's generator."""
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_fill_uniform_f16(_ptr(out), n, seed)
    return out


def fill_normal_f16(n: int, seed: int, mean: float = 0.0, std: float = 0.02) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_fill_normal_f16(_ptr(out), n, seed, mean, std)
    return out


def make_inputs(M: int, N: int, K: int, dist: str = "uniform", seed_a: int = 42,
                seed_b: int = 77) -> tuple[np.ndarray, np.ndarray]:
    """A (M×K) and B (N×K) as uint16 fp16 bit patterns, seeds 42/77 as in the engine."""
    if dist == "uniform":
        a, b = fill_uniform_f16(M * K, seed_a), fill_uniform_f16(N * K, seed_b)
    elif dist == "normal":
        a, b = fill_normal_f16(M * K, seed_a), fill_normal_f16(N * K, seed_b)
    else:
        raise ValueError(dist)
    return a.reshape(M, K), b.reshape(N, K)


def _gemm(fn: str, dtype, A: np.ndarray, B: np.ndarray, row0: int, rows: Optional[int],
          threads: int) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    M, K = A.shape
    N, K2 = B.shape
    assert K == K2
    rows = M - row0 if rows is None else rows
    C = np.empty((rows, N), dtype=dtype)
    getattr(lib(), fn)(_ptr(A), _ptr(B), _ptr(C), M, N, K, row0, rows, threads)
    return C


def gemm_f16(A, B, row0: int = 0, rows: Optional[int] = None, threads: int = 0) -> np.ndarray:
    """fp16(sequential-k fp32 FMA sum) for rows [row0, row0+rows), as uint16 bit patterns."""
    return _gemm("oracle_gemm_f16", np.uint16, A, B, row0, rows, threads)


def gemm_f32(A, B, row0: int = 0, rows: Optional[int] = None, threads: int = 0) -> np.ndarray:
    return _gemm("oracle_gemm_f32", np.float32, A, B, row0, rows, threads)


def gemm_f64(A, B, row0: int = 0, rows: Optional[int] = None, threads: int = 0) -> np.ndarray:
    return _gemm("oracle_gemm_f64", np.float64, A, B, row0, rows, threads)


def check_error(ref: np.ndarray, cmp: np.ndarray, atol: float = 1e-3, rtol: float = 1e-2):
    """The reference's check_error on fp16 bit patterns -> (passed, stats)."""
    ref = np.ascontiguousarray(ref, dtype=np.uint16).ravel()
    cmp = np.ascontiguousarray(cmp, dtype=np.uint16).ravel()
    assert ref.size == cmp.size
    st = np.zeros(5, dtype=np.float64)
    ok = lib().oracle_check_error(_ptr(ref), _ptr(cmp), ref.size, atol, rtol, _ptr(st))
    return bool(ok), {"max_abs": st[0], "max_rel": st[1], "max_abs_idx": int(st[2]),
                      "max_rel_idx": int(st[3]), "mismatches": int(st[4])}


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def acceptance(c_test: np.ndarray, c_exact: np.ndarray, K: int) -> dict:
    """BASELINE acceptance metrics of a result against an (fp64) exact product.

    abs bound 2e-2*sqrt(K/1024); rel error |c-r| / max(|r|, tau) with tau = the abs bound
    (bounded near zero), plus the reference's own unbounded form for reporting.
    """
    c = np.asarray(c_test, dtype=np.float64)
    r = np.asarray(c_exact, dtype=np.float64)
    bound = 2e-2 * np.sqrt(K / 1024.0)
    err = np.abs(c - r)
    rel = err / np.maximum(np.abs(r), bound)
    rel_ref = err / np.maximum(np.abs(r), 1e-6)
    return {"max_abs": float(err.max(initial=0.0)), "abs_bound": float(bound),
            "max_rel": float(rel.max(initial=0.0)), "max_rel_unbounded": float(rel_ref.max(initial=0.0))}


# ── the reference's own code, compiled from its sources (pinning only) ─────────────
def ref_host() -> Optional[ctypes.CDLL]:
    """Reference fill_random_fp16 / check_error on host buffers, or None if not built."""
    if not REF_HOST_PATH.exists():
        return None
    L = ctypes.CDLL(str(REF_HOST_PATH))
    L.vgref_fill_random_fp16.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint]
    L.vgref_check_error.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                    ctypes.c_float, ctypes.c_float]
    return L


def ref_gpu() -> Optional[ctypes.CDLL]:
    """Reference naive v0 kernel / cuBLAS backend / device fill on a GPU, or None."""
    if not REF_GPU_PATH.exists():
        return None
    L = ctypes.CDLL(str(REF_GPU_PATH))
    for name in ("vgref_naive_gemm", "vgref_cublas_gemm"):
        getattr(L, name).argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    L.vgref_fill_random_fp16_device.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint]
    return L
