"""vg_b200_gemm_f16_noalloc — the allocation-free entry point, through the C ABI.

It serves callers that may not allocate device memory (a host that owns the whole GPU
through its own pool, latency-critical loops, fixed memory budgets): the K-padding
workspace that vg_b200_gemm_f16 takes from the stream-ordered pool comes instead from a
fixed 32 MiB array inside the library. This file is collected last on purpose, so that a
run stopping at its first failure has already run every other test; it also passes on its
own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from conftest import to_dev, to_host

pytestmark = pytest.mark.gpu

LIMIT_CODE = 2001  # VG_ERROR_NOALLOC_SCRATCH_LIMIT


def _c_abi(vg):
    L = vg.lib()
    f = L.vg_b200_gemm_f16_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    g = L.vg_b200_gemm_f16
    g.restype = ctypes.c_int
    g.argtypes = f.argtypes
    return f, g


def _run_both(vg, orc, A_host, B_host, offset_a=0, offset_b=0):
    """Same inputs through the default entry point and the allocation-free one."""
    import torch
    f_noalloc, f_default = _c_abi(vg)
    M, K = A_host.shape
    N = B_host.shape[0]
    bufA = torch.zeros(M * K + 8, dtype=torch.float16, device="cuda")
    bufB = torch.zeros(N * K + 8, dtype=torch.float16, device="cuda")
    dA = bufA[offset_a:offset_a + M * K].view(M, K)
    dB = bufB[offset_b:offset_b + N * K].view(N, K)
    dA.copy_(to_dev(A_host))
    dB.copy_(to_dev(B_host))
    C_ref = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    C_new = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert f_default(dA.data_ptr(), dB.data_ptr(), C_ref.data_ptr(), M, N, K, s) == 0
    assert f_noalloc(dA.data_ptr(), dB.data_ptr(), C_new.data_ptr(), M, N, K, s) == 0
    torch.cuda.synchronize()
    return to_host(C_ref), to_host(C_new)


def test_noalloc_matches_default_on_two_calls_in_a_row(vg, orc):
    # Call 1: K % 8 != 0 -> both operands go through the scratch-backed pad pre-pass.
    A1, B1 = orc.make_inputs(300, 520, 4099)
    ref1, new1 = _run_both(vg, orc, A1, B1)
    ok, st = orc.check_error(ref1, new1)
    assert ok, st
    assert np.array_equal(ref1, new1)  # same kernel, same padded data
    # Call 2: different shape, misaligned A only; the scratch still holds call 1's data.
    A2, B2 = orc.make_inputs(257, 384, 96)
    ref2, new2 = _run_both(vg, orc, A2, B2, offset_a=1)
    ok, st = orc.check_error(ref2, new2)
    assert ok, st
    assert np.array_equal(ref2, new2)
    ok, st = orc.check_error(orc.gemm_f16(A2, B2), new2)  # and against the oracle
    assert ok, st
    assert vg.device_status() == 0


def test_noalloc_rejects_padded_problems_beyond_the_limit(vg):
    import torch
    f_noalloc, _ = _c_abi(vg)
    M, N, K = 4096, 4096, 8196  # padded copies: 8192 rows * 8200 * 2 B = 134 MB > 32 MiB
    A = torch.zeros(M, K, dtype=torch.float16, device="cuda")
    B = torch.zeros(N, K, dtype=torch.float16, device="cuda")
    C = torch.full((M, N), 3.0, dtype=torch.float16, device="cuda")
    rc = f_noalloc(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K,
                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == LIMIT_CODE
    assert float(C[0, 0]) == 3.0 and float(C[-1, -1]) == 3.0  # nothing was launched


def test_noalloc_needs_no_scratch_when_aligned(vg, orc):
    A, B = orc.make_inputs(1024, 2048, 512)
    ref, new = _run_both(vg, orc, A, B)
    assert np.array_equal(ref, new)


def test_noalloc_split_k_partials_live_in_the_array(vg, orc):
    """A grid too small for one wave with long K: the per-shape choice splits K (v11), whose
    fp32 partials of every split then sit in the fixed array instead of the pool before the
    reduction kernel adds them. Two calls in a row (the second finds the first one's partials
    still there) must both equal the default entry point bit for bit (same splits, same order
    of additions), and the result meets the long-K bound against the fp64 product on sampled
    rows."""
    import torch
    f_noalloc, f_default = _c_abi(vg)
    M, N, K = 256, 2048, 16384
    p = vg.plan(-1, M, N, K, 256, 256, 256)
    assert p["version"] == 11 and p["splits"] > 1 and p["pad_a"] == 0 and p["pad_b"] == 0, p
    A, B = orc.make_inputs(M, N, K)
    dA, dB = to_dev(A), to_dev(B)
    s = torch.cuda.current_stream().cuda_stream
    ref = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    assert f_default(dA.data_ptr(), dB.data_ptr(), ref.data_ptr(), M, N, K, s) == 0
    outs = []
    for _ in range(2):
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        assert f_noalloc(dA.data_ptr(), dB.data_ptr(), C.data_ptr(), M, N, K, s) == 0
        outs.append(C)
    torch.cuda.synchronize()
    for C in outs:
        assert torch.equal(C, ref)
    rows = [0, 1, 129, M - 1]
    exact = np.concatenate([orc.gemm_f64(A, B, r, 1) for r in rows])
    got = outs[1].cpu().numpy()[rows].astype(np.float64)
    bound = 2e-2 * np.sqrt(K / 1024.0)
    assert np.all(np.abs(got - exact) <= bound + 1e-2 * np.abs(exact))
    assert vg.device_status() == 0


def test_noalloc_run_time_tile_counter_lives_in_the_array(vg, orc):
    """Long K over a full wave of pair tiles: the per-shape choice is v8, whose persistent
    pairs claim tiles through a counter that every launch zeroes; here the counter sits in
    the fixed array. Two calls in a row (the second finds the first one's final count there)
    must equal the default entry point bit for bit."""
    import torch
    f_noalloc, f_default = _c_abi(vg)
    M, N, K = 2560, 4096, 16384
    p = vg.plan(-1, M, N, K, 256, 256, 256)
    assert p["version"] == 8 and p["dyn"] == 1 and p["promote_kb"] < p["num_kb"], p
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda").uniform_(-1, 1, generator=g)
    dB = torch.empty((N, K), dtype=torch.float16, device="cuda").uniform_(-1, 1, generator=g)
    s = torch.cuda.current_stream().cuda_stream
    ref = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    assert f_default(dA.data_ptr(), dB.data_ptr(), ref.data_ptr(), M, N, K, s) == 0
    for _ in range(2):
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        assert f_noalloc(dA.data_ptr(), dB.data_ptr(), C.data_ptr(), M, N, K, s) == 0
        torch.cuda.synchronize()
        assert torch.equal(C, ref)
    assert vg.device_status() == 0
