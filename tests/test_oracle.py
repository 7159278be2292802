"""The oracle (CPU restatement) pinned against the reference's own code and fixtures."""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_fill_matches_reference_golden(orc):
    g = np.load(GOLDEN / "golden_fill.npz")
    for key in g.files:
        if key.startswith("seed_"):
            seed = int(key.split("_")[1])
            assert np.array_equal(orc.fill_uniform_f16(g[key].size, seed), g[key]), key


def test_fill_matches_reference_live(orc):
    R = orc.ref_host()
    if R is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for seed in (42, 77, 99):
        n = 50_000
        ref = np.empty(n, np.uint16)
        assert R.vgref_fill_random_fp16(ref.ctypes.data, n, seed) == 0
        assert np.array_equal(orc.fill_uniform_f16(n, seed), ref)


def test_fill_range_and_determinism(orc):
    a = orc.fill_uniform_f16(100_000, 42).view(np.float16).astype(np.float32)
    assert a.min() >= -1.0 and a.max() <= 1.0
    assert abs(a.mean()) < 0.01
    b = orc.fill_normal_f16(100_000, 42).view(np.float16).astype(np.float32)
    assert abs(b.std() - 0.02) < 0.001 and abs(b.mean()) < 0.001
    assert np.array_equal(orc.fill_normal_f16(1000, 7), orc.fill_normal_f16(1000, 7))


def test_f32_to_f16_round_to_nearest_even(orc):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(200_000) * 10.0 ** rng.integers(-9, 6, 200_000)).astype(np.float32)
    edge = np.array([65504, 65519.99, 65520, 65536, 1e9, 5.96e-8, 2.98e-8, 2.99e-8, 6.1e-5,
                     -0.0, 0.0, np.inf, -np.inf, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11], np.float32)
    x = np.concatenate([x, edge, -edge])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(orc.f32_to_f16(x), want)


def test_check_error_matches_reference_golden(orc):
    g = np.load(GOLDEN / "golden_fill.npz")
    ok, st = orc.check_error(g["check_ref"], g["check_cmp"])
    assert ok == bool(g["check_passed"])
    assert st["max_abs"] == pytest.approx(float(g["check_max_abs"]), rel=1e-6)
    assert st["max_rel"] == pytest.approx(float(g["check_max_rel"]), rel=1e-6)


def _seq_fma_row(A, B, m, n):
    """Pure-Python sequential fused multiply-add (fp16 products are exact in fp64)."""
    a = A[m].view(np.float16).astype(np.float64)
    b = B[n].view(np.float16).astype(np.float64)
    acc = np.float32(0.0)
    for k in range(a.size):
        acc = np.float32(float(acc) + a[k] * b[k])
    return acc


def test_gemm_is_sequential_fma(orc):
    A, B = orc.make_inputs(40, 24, 97)
    C = orc.gemm_f32(A, B)
    for m, n in [(0, 0), (39, 23), (17, 5), (3, 20)]:
        assert C[m, n] == _seq_fma_row(A, B, m, n)


def test_gemm_f64_matches_numpy(orc):
    A, B = orc.make_inputs(65, 130, 77, dist="normal")
    exact = A.view(np.float16).astype(np.float64) @ B.view(np.float16).astype(np.float64).T
    assert np.allclose(orc.gemm_f64(A, B), exact, rtol=0, atol=1e-12)


def test_gemm_row_slices_and_threads_agree(orc):
    A, B = orc.make_inputs(37, 300, 64)
    full = orc.gemm_f16(A, B, threads=1)
    assert np.array_equal(orc.gemm_f16(A, B, threads=5), full)
    assert np.array_equal(orc.gemm_f16(A, B, row0=11, rows=9), full[11:20])


def test_gemm_known_answers(orc):
    # A = all ones, B[n, k] = k-ramp scaled: C[m, n] = sum_k B[n, k] exactly representable.
    M, N, K = 8, 16, 64
    A = np.full((M, K), np.float16(1.0)).view(np.uint16)
    Bf = (np.arange(K, dtype=np.float32)[None, :] * (np.arange(N)[:, None] + 1) / 64).astype(np.float16)
    C = orc.gemm_f16(A, Bf.view(np.uint16)).view(np.float16).astype(np.float64)
    want = Bf.astype(np.float64).sum(axis=1)
    assert np.array_equal(C, np.broadcast_to(want, (M, N)))
    # Identity B picks columns of A.
    Ai, _ = orc.make_inputs(32, 1, 32)
    I = np.eye(32, dtype=np.float16).view(np.uint16)
    assert np.array_equal(orc.gemm_f16(Ai, I), Ai)


def test_gemm_matches_reference_naive_kernel_golden(orc):
    path = GOLDEN / "golden_gemm.npz"
    if not path.exists():
        pytest.skip("golden_gemm.npz not generated yet")
    g = np.load(path)
    for (M, N, K, sa, sb) in g["shapes"]:
        A = orc.fill_uniform_f16(M * K, sa).reshape(M, K)
        B = orc.fill_uniform_f16(N * K, sb).reshape(N, K)
        key = f"{M}x{N}x{K}_s{sa}_{sb}"
        mine = orc.gemm_f16(A, B)
        assert np.array_equal(mine, g[key + "_naive"]), key            # bit-exact vs reference v0
        ok, st = orc.check_error(g[key + "_cublas"], mine)              # the reference's own arbiter
        assert ok, (key, st)


def test_acceptance_metric(orc):
    r = np.array([0.0, 1.0, -300.0])
    c = np.array([0.01, 1.001, -300.1])
    acc = orc.acceptance(c, r, K=1024)
    assert acc["abs_bound"] == pytest.approx(0.02)
    assert acc["max_abs"] == pytest.approx(0.1)
    assert acc["max_rel"] == pytest.approx(0.5)
