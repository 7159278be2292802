"""C ABI: the library loads without a GPU, exports every declared symbol, and its host
logic (planner, raster order, row sharding, registry) behaves. No compute calls."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(vg_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol(vg):
    decl = declared_symbols()
    assert len(decl) >= 20
    L = ctypes.CDLL(str(vg.LIB_PATH))
    missing = [n for n in decl if not hasattr(L, n)]
    assert not missing, missing
    assert set(decl) == set(vg.EXPORTED_SYMBOLS)


def test_versions_and_registry_order(vg):
    assert vg.versions() == ["VibeGEMM B200 v0", "VibeGEMM B200 v1", "VibeGEMM B200 v2",
                             "VibeGEMM B200 v3", "VibeGEMM B200 v4", "VibeGEMM B200 v5",
                             "VibeGEMM B200 v6", "VibeGEMM B200 v7", "VibeGEMM B200 v8",
                             "VibeGEMM B200 v9", "VibeGEMM B200 v10", "VibeGEMM B200 v11",
                             "VibeGEMM B200 v12"]
    assert vg.default_version() == -1 and vg.version_name(-1) == "VibeGEMM B200 auto"
    # cuBLAS registers at priority 0 and is the engine's reference; B200 at priority 3.
    assert vg.backends() == ["cuBLAS"] + vg.versions() + ["VibeGEMM B200 auto"]


@pytest.mark.parametrize("num_m,num_n,group", [(1, 1, 8), (32, 32, 8), (7, 13, 8), (33, 5, 4),
                                               (100, 3, 16), (5, 41, 1), (9, 9, 100)])
def test_raster_is_a_bijection(vg, num_m, num_n, group):
    seen = set()
    for t in range(num_m * num_n):
        tm, tn = vg.raster_tile(t, num_m, num_n, group)
        assert 0 <= tm < num_m and 0 <= tn < num_n
        seen.add((tm, tn))
    assert len(seen) == num_m * num_n
    assert vg.raster_tile(num_m * num_n, num_m, num_n, group) == (-1, -1)


def test_raster_groups_m_tiles(vg):
    # Consecutive tiles walk down a group of 8 M tiles before moving along N.
    order = [vg.raster_tile(t, 32, 32, 8) for t in range(16)]
    assert order[:8] == [(m, 0) for m in range(8)]
    assert order[8:16] == [(m, 1) for m in range(8)]


@pytest.mark.parametrize("M,world", [(32768, 1), (32768, 2), (32768, 8), (8191, 8), (3, 8), (0, 4)])
def test_shard_rows_partition(vg, M, world):
    covered = []
    for r in range(world):
        r0, n = vg.shard_rows(M, world, r)
        assert n >= 0
        covered.extend(range(r0, r0 + n))
    assert covered == list(range(M))


def test_plan_aligned_square(vg):
    p = vg.plan(2, 8192, 8192, 8192, 256, 256, 256)
    assert p["cta_group"] == 2 and p["epilogue"] == "tma_f16"
    assert (p["pad_a"], p["pad_b"]) == (0, 0)
    assert (p["num_m_tiles"], p["num_n_tiles"], p["num_kb"]) == (32, 32, 128)
    assert p["grid"] == 148 and p["persistent"] == 1
    p1 = vg.plan(1, 8192, 8192, 8192, 256, 256, 256)
    assert p1["cta_group"] == 1 and p1["grid"] == 148 and p1["num_m_tiles"] == 64
    p0 = vg.plan(0, 8192, 8192, 8192, 256, 256, 256)
    assert p0["persistent"] == 0 and p0["grid"] == 64 * 32 and p0["epilogue"] == "direct_f16"
    p3 = vg.plan(3, 8192, 8192, 8192, 256, 256, 256)
    assert (p3["cta_group"], p3["tile_n"], p3["stages"]) == (2, 512, 4)
    assert (p3["num_m_tiles"], p3["num_n_tiles"]) == (32, 16) and p3["grid"] == 148


@pytest.mark.parametrize("shape,want", [
    ((8192, 8192, 8192), 3), ((32768, 32768, 32768), 9),
    ((4096, 14336, 4096), 2),    # 448 256x512 tiles = 6.05 waves; 896 256x256 tiles waste less
    ((16384, 16384, 16384), 9), ((4096, 32768, 32768), 9),   # long K: chunks, sums in registers
    ((2560, 4096, 32768), 8),    # 80 256x512 tiles = 2 waves vs 160 256x256 = 3: sums in TMEM
    ((8192, 8192, 12288), 3),    # below the promotion threshold: one chain per output
    ((4096, 4096, 14336), 3),
    ((8191, 8193, 4099), 3),     # 7.4 vs 14.3 waves: estimates within 1.5 %, v3's data saving wins
    ((8192, 8192, 512), 2),      # short K: double-buffered accumulator
    ((8192, 8192, 256), 12),     # K <= 256: the same tile with A resident in shared memory
    ((1000, 3000, 2048), 5),     # fewer pair tiles than pair slots: 128x192 tiles fill one wave
    ((1000, 3000, 8192), 7),     # same tiles, long K: the fifth stage pays
    ((512, 512, 512), 5),
    ((2048, 2048, 4096), 1),     # one wave either way; at K = 4096 single CTAs beat pairs
    ((256, 2048, 32768), 11),    # 8 pair tiles, 512 k-blocks each: split-K over 74 pairs
    ((512, 8192, 32768), 8),     # 64 pair tiles on 74 pairs: v2's tile, chunked accumulation
    ((1000, 3000, 32768), 8),    # long K on an under-filled grid: chains split (v8, not v7)
    ((512, 8192, 16384), 8), ((512, 8192, 8192), 2),
    ((1000, 3000, 32), 5),
])
def test_auto_version_choice(vg, shape, want):
    assert vg.plan(-1, *shape, 256, 256, 256)["version"] == want
    assert vg.plan(want, *shape, 256, 256, 256)["version"] == want


def test_plan_tails_and_alignment(vg):
    # 8191x8193x4099: K*2 bytes not a multiple of 16 -> both operands padded to K=4104;
    # N*2 not a multiple of 16 -> direct-store epilogue.
    p = vg.plan(2, 8191, 8193, 4099, 256, 256, 256)
    assert (p["pad_a"], p["pad_b"], p["k_padded"]) == (1, 1, 4104)
    assert p["epilogue"] == "staged_f16"
    assert (p["num_m_tiles"], p["num_n_tiles"], p["num_kb"]) == (32, 33, 65)
    # 1000x3000x2048: aligned strides, partial tiles, under-filled grid.
    p = vg.plan(2, 1000, 3000, 2048, 256, 256, 256)
    assert (p["pad_a"], p["pad_b"], p["epilogue"]) == (0, 0, "tma_f16")
    assert p["grid"] == 2 * 4 * 12
    # A misaligned pointer alone pads only that operand.
    p = vg.plan(2, 512, 512, 512, 258, 256, 256)
    assert (p["pad_a"], p["pad_b"]) == (1, 0)
    # A misaligned C pointer switches to direct stores; fp32 output always direct.
    assert vg.plan(2, 512, 512, 512, 256, 256, 258)["epilogue"] == "staged_f16"
    assert vg.plan(0, 512, 512, 512, 256, 256, 258)["epilogue"] == "direct_f16"
    assert vg.plan(2, 512, 512, 512, 256, 256, 256, f32_out=True)["epilogue"] == "direct_f32"


def test_plan_of_run_time_tiles_and_chunks(vg):
    """v9: persistent 256x512 pairs claiming tiles at run time; K >= 16384 is summed in
    chunks of 64 k-blocks (K = 4096); below, one chunk. v10: the same without chunks."""
    p = vg.plan(9, 32768, 32768, 32768, 256, 256, 256)
    assert (p["dyn"], p["promote"], p["promote_kb"], p["num_kb"]) == (1, 1, 64, 512)
    assert p["grid"] == 148 and p["persistent"] == 1 and p["tile_n"] == 512
    assert vg.plan(9, 8192, 8192, 8192, 256, 256, 256)["promote_kb"] == 128  # one chunk of 128
    assert vg.plan(9, 8192, 8192, 65536, 256, 256, 256)["promote_kb"] == 64
    p10 = vg.plan(10, 32768, 32768, 32768, 256, 256, 256)  # run-time tiles, one chain
    assert (p10["dyn"], p10["promote"], p10["promote_kb"]) == (1, 0, 512)
    assert vg.plan(8, 8192, 8192, 8192, 256, 256, 256)["promote_kb"] == 64
    assert vg.plan(3, 8192, 8192, 8192, 256, 256, 256)["dyn"] == 0
    # v8 (the long-K choice on smaller grids) claims tiles at run time too; the fused
    # all-gather's choice for a long-K shard promotes as well
    p8 = vg.plan(8, 32768, 32768, 32768, 256, 256, 256)
    assert (p8["dyn"], p8["promote"], p8["promote_kb"], p8["tile_n"]) == (1, 1, 64, 256)
    p = vg.plan(-1, 4096, 32768, 32768, 256, 256, 256, allgather=True)
    assert p["version"] == 9 and p["epilogue"] == "tma_f16_peers"
    assert vg.plan(-1, 512, 8192, 32768, 256, 256, 256, allgather=True)["version"] == 8
    # at K <= 256 the fused all-gather keeps v2 (the default entry point takes v12)
    assert vg.plan(-1, 8192, 8192, 256, 256, 256, 256, allgather=True)["version"] == 2
    assert vg.plan(-1, 8192, 8192, 256, 256, 256, 256)["version"] == 12


def test_plan_of_a_resident(vg):
    """v12: with K <= 256 (4 k-blocks) A stays in shared memory over each pair's contiguous
    run of tiles (6 B stages); above that it is v2's plan."""
    p = vg.plan(12, 8192, 8192, 256, 256, 256, 256)
    assert (p["a_resident"], p["stages"], p["tile_n"], p["cta_group"], p["grid"]) == (1, 6, 256, 2, 148)
    assert p["persistent"] == 1 and p["dyn"] == 0 and p["stream_k"] == 0
    assert vg.plan(12, 512, 512, 264, 256, 256, 256)["a_resident"] == 0  # 5 k-blocks
    assert vg.plan(12, 8192, 8192, 512, 256, 256, 256)["a_resident"] == 0
    full = vg.plan(12, 8192, 8192, 8192, 256, 256, 256)
    assert (full["a_resident"], full["stages"]) == (0, 6)
    for v in range(12):
        assert vg.plan(v, 8192, 8192, 512, 256, 256, 256)["a_resident"] == 0


def test_contiguous_runs_share_row_blocks(vg):
    """The A-resident schedule: worker w takes tiles [w*T/P, (w+1)*T/P) row-major, so a
    worker changes A row-block at most ceil(run / num_n) + 1 times."""
    num_m, num_n, workers = 32, 32, 74
    seen = []
    for w in range(workers):
        units = vg.work_units(2, w, workers, num_m, num_n, 8, 8)
        lin = [u["tile_m"] * num_n + u["tile_n"] for u in units]
        assert lin == list(range(1024 * w // workers, 1024 * (w + 1) // workers))
        rows = {u["tile_m"] for u in units}
        assert len(rows) <= 2
        seen += lin
    assert sorted(seen) == list(range(num_m * num_n))


def test_plan_of_split_k(vg):
    """v11: K splits that give every pair slot a unit, >= 8 k-blocks each, and chains of at
    most 64 k-blocks from K = 16384 on; one split (plain v2) when the grid is already full."""
    p = vg.plan(11, 256, 2048, 32768, 256, 256, 256)
    assert p["splits"] == 9 and p["epilogue"] == "splitk_f16" and p["grid"] == 2 * 72
    assert vg.plan(11, 256, 2048, 32768, 256, 256, 256, f32_out=True)["epilogue"] == "direct_f32"
    assert vg.plan(11, 256, 2048, 1024, 256, 256, 256)["splits"] == 2   # 16 k-blocks: 2 x 8
    full = vg.plan(11, 8192, 8192, 8192, 256, 256, 256)
    assert full["splits"] == 1 and full["epilogue"] == "tma_f16"
    assert vg.plan(11, 8192, 8192, 32768, 256, 256, 256)["splits"] == 8  # chains <= 4096
    with pytest.raises(vg.VibeGemmError):   # no fused all-gather form
        vg.plan(11, 256, 2048, 32768, 256, 256, 256, allgather=True)


def test_plan_rejects_bad_input(vg):
    with pytest.raises(vg.VibeGemmError):
        vg.plan(len(vg.versions()), 16, 16, 16)
    with pytest.raises(vg.VibeGemmError):
        vg.plan(0, -1, 16, 16)


def test_gemm_rejects_cpu_tensors(vg):
    import torch
    a = torch.zeros(4, 8, dtype=torch.float16)
    with pytest.raises(ValueError):
        vg.gemm(a, a)


def test_allgather_plan_never_uses_stream_k(vg):
    """The fused all-gather epilogue has no stream-K or split-K form: its per-shape choice
    skips them (a 501-row shard of 1001×1024×4099 would otherwise split K) and an explicit
    v4 is refused."""
    assert vg.plan(-1, 501, 1024, 4099, 256, 256, 256)["version"] == 11
    p = vg.plan(-1, 501, 1024, 4099, 256, 256, 256, allgather=True)
    assert p["version"] != 4 and p["stream_k"] == 0 and p["epilogue"] == "tma_f16_peers"
    with pytest.raises(vg.VibeGemmError):
        vg.plan(4, 501, 1024, 4099, 256, 256, 256, allgather=True)
    import ctypes
    out = (ctypes.c_int * 20)()
    assert vg.lib().vg_b200_plan(-1, 512, 1024, 4096, 256, 256, 256, 3, 148, out) != 0  # no mode 3


def test_entry_points_fail_loudly_without_a_gpu(vg):
    """With no usable GPU every entry point returns a CUDA error code; nothing falls back to
    a CPU path. (Skipped where a GPU is visible: the pointers here are not device memory.)"""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    L = vg.lib()
    assert L.vg_b200_gemm_f16(16, 16, 16, 8, 8, 8, None) != 0
    assert L.vg_b200_gemm_f16_version(2, 16, 16, 16, 8, 8, 8, None) != 0
    assert L.vg_b200_gemm_f16_noalloc(16, 16, 16, 8, 8, 8, None) != 0
    assert L.vg_b200_is_available(0) == 0
    with pytest.raises(vg.VibeGemmError):
        vg._check(L.vg_b200_gemm_f16(16, 16, 16, 8, 8, 8, None), "vg_b200_gemm_f16")
