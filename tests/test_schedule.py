"""The persistent workers' schedules (host copy of the device code), checked without a GPU:
every (tile, k-block) iteration is processed exactly once, and stream-K's split tiles have
exactly one owner whose contributors are precisely the workers that wrote its partials."""
import collections

import pytest


@pytest.mark.parametrize("num_m,num_n,kb,workers", [(32, 32, 128, 74), (7, 13, 5, 9), (1, 1, 3, 1),
                                                    (4, 6, 32, 74), (33, 17, 65, 74)])
def test_data_parallel_covers_every_tile_once(vg, num_m, num_n, kb, workers):
    seen = collections.Counter()
    for w in range(workers):
        for u in vg.work_units(False, w, workers, num_m, num_n, 8, kb):
            assert (u["kb0"], u["kb1"], u["kind"]) == (0, kb, "full")
            seen[(u["tile_m"], u["tile_n"])] += 1
    assert len(seen) == num_m * num_n and set(seen.values()) == {1}


@pytest.mark.parametrize("num_m,num_n,kb,workers", [
    (4, 12, 32, 74),    # 1000x3000x2048 on 74 pairs: 1536 iterations, 20.8 per worker
    (2, 2, 8, 8),       # tiles split across two workers
    (1, 3, 40, 74),     # 120 iterations: workers smaller than a tile, tiles over 3 workers
    (3, 5, 7, 4),
    (16, 8, 224, 74),   # 4096x4096x14336 tiles
    (5, 1, 1, 5),       # one k-block per tile: no splits
])
def test_stream_k_partition_and_owners(vg, num_m, num_n, kb, workers):
    iters = collections.Counter()
    owners = {}
    partial_writer = collections.defaultdict(list)
    for w in range(workers):
        units = vg.work_units(True, w, workers, num_m, num_n, 8, kb)
        for j, u in enumerate(units):
            tile = (u["tile_m"], u["tile_n"])
            for k in range(u["kb0"], u["kb1"]):
                iters[(tile, k)] += 1
            if u["kind"] == "partial":
                assert j == 0, "a partial can only be a worker's first unit"
                partial_writer[tile].append(w)
            elif u["kind"] == "owner":
                assert j == len(units) - 1, "an owner can only be a worker's last unit"
                assert u["kb0"] == 0 and u["kb1"] < kb
                assert tile not in owners
                owners[tile] = (w, u["first_contrib"], u["last_contrib"])
            else:
                assert (u["kb0"], u["kb1"]) == (0, kb)
    # every iteration exactly once
    assert len(iters) == num_m * num_n * kb and set(iters.values()) == {1}
    # split tiles: one owner; contributors = exactly the partial writers, all later workers
    assert set(owners) == set(partial_writer)
    for tile, (w, first, last) in owners.items():
        assert sorted(partial_writer[tile]) == list(range(first, last + 1))
        assert first == w + 1


def test_stream_k_plan(vg):
    p = vg.plan(4, 1000, 3000, 2048, 256, 256, 256)
    assert p["stream_k"] == 1 and p["grid"] == 148  # 74 pairs, 1536 iterations
    assert vg.plan(4, 256, 256, 64, 256, 256, 256)["grid"] == 2  # 1 tile x 1 k-block: one worker
    # the per-shape choice never uses stream-K
    for shape in [(1000, 3000, 2048), (512, 512, 512), (8192, 8192, 8192), (2048, 2048, 8192)]:
        assert vg.plan(-1, *shape, 256, 256, 256)["stream_k"] == 0


@pytest.mark.parametrize("shape", [(512, 512, 512), (8192, 8192, 8192), (8191, 8193, 4099), (256, 2048, 1024),
                                   (1000, 3000, 2048), (4096, 14336, 4096), (4096, 4096, 14336),
                                   (8192, 8192, 512), (32768, 32768, 32768), (4096, 32768, 32768),
                                   (256, 2048, 32768), (1000, 3000, 8192), (8192, 8192, 256),
                                   (1000, 3000, 200)])
@pytest.mark.parametrize("version", [-1, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12])
def test_launch_plans_cover_every_iteration_once(vg, shape, version):
    """For the plan the launcher builds (grid, raster group, stream-K or not), the workers'
    units cover every (tile, k-block) iteration of the problem exactly once."""
    M, N, K = shape
    p = vg.plan(version, M, N, K, 256, 256, 256)
    num_m, num_n, kb = p["num_m_tiles"], p["num_n_tiles"], p["num_kb"]
    if not p["persistent"]:
        assert p["grid"] == num_m * num_n * p["cta_group"]  # one CTA (pair) per tile
        return
    if p["dyn"]:
        # Run-time claims: pair w starts with tile w (every pair has one: the grid is at most
        # the tile count), later claims are workers + counter value, so the tiles claimed
        # before the counter passes the end are each claimed once.
        workers = p["grid"] // p["cta_group"]
        total = num_m * num_n
        assert 1 <= workers <= total
        claimed = list(range(workers)) + [workers + c for c in range(total - workers)]
        assert sorted(claimed) == list(range(total))
        # the chunks of a tile cover its k-blocks
        chunks = -(-kb // p["promote_kb"])
        assert (chunks - 1) * p["promote_kb"] < kb <= chunks * p["promote_kb"]
        return
    workers = p["grid"] // p["cta_group"]
    covered = collections.Counter()
    for w in range(workers):
        mode = 2 if p["a_resident"] else int(p["stream_k"])
        for u in vg.work_units(mode, w, workers, num_m, num_n, p["group_m"], kb, p["splits"]):
            covered[(u["tile_m"], u["tile_n"])] += u["kb1"] - u["kb0"]
    assert len(covered) == num_m * num_n and set(covered.values()) == {kb}
