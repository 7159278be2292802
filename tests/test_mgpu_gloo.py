"""Host logic of the multi-GPU row-block path, run as world-size-2 gloo ranks on CPU.
The compute step is the oracle; sharding, shard sizes and the C all-gather are the
same code the GPU bench uses (vibegemm_b200.mgpu)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, q):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    import oracle
    from vibegemm_b200.mgpu import RowShardedGemm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A, B = oracle.make_inputs(M, N, K)
        sh = RowShardedGemm(M, N, K, rank, world)
        r0, rows = sh.local
        A_loc = torch.from_numpy(A[r0:r0 + rows].view(np.float16).copy())
        C_loc = torch.zeros((rows, N), dtype=torch.float16)

        def cpu_gemm(a, b, c):
            c.copy_(torch.from_numpy(oracle.gemm_f16(a.numpy().view(np.uint16), b).view(np.float16)))

        sh.run(A_loc, B, C_loc, cpu_gemm)
        full = sh.gather(C_loc)
        q.put((rank, r0, rows, full.numpy().view(np.uint16).copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [96, 95, 1])
def test_row_sharded_gemm_gloo_world2(M):
    import oracle
    from vibegemm_b200.mgpu import shard_rows
    N, K, world = 40, 24, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    out = [q.get(timeout=10) for _ in range(world)]
    A, B = oracle.make_inputs(M, N, K)
    want = oracle.gemm_f16(A, B)
    covered = 0
    for rank, r0, rows, full in out:
        assert (r0, rows) == shard_rows(M, world, rank)
        assert np.array_equal(full, want)
        covered += rows
    assert covered == M


def test_shard_rows_python_matches_c_abi(vg):
    from vibegemm_b200.mgpu import shard_rows
    for M in (0, 1, 7, 8, 8191, 32768):
        for world in (1, 2, 3, 4, 8):
            for r in range(world):
                assert shard_rows(M, world, r) == vg.shard_rows(M, world, r)


def _leaver(rank, world, port, q):
    """Rank 1 joins the group, then leaves before the all-gather of C; rank 0 must get an
    error from its collective within the process-group timeout instead of hanging."""
    import sys
    import time
    from datetime import timedelta
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    from vibegemm_b200.mgpu import RowShardedGemm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before the abrupt exit
        os._exit(0)  # leaves between steps: no collective of its own is in flight
    sh = RowShardedGemm(64, 16, 8, rank, world)
    C_loc = torch.zeros((sh.local[1], 16), dtype=torch.float16)
    t0 = time.time()
    try:
        sh.gather(C_loc)
        q.put((rank, "no error"))
    except Exception as e:  # the surviving rank learns of the failure from the collective
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_that_leaves_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = dict(q.get(timeout=10) for _ in range(2))
    assert out[1] == "left"
    assert out[0].startswith("error after"), out[0]
