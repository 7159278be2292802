"""Fused row-sharded GEMM + all-gather of C on 2 GPUs (skipped with fewer GPUs).

Each rank computes its row block of C with vg_b200_gemm_f16_allgather, whose epilogue also
writes the rows into the other rank's full C over NVLink — one store per peer, or one
NVLink-multicast (multimem) store when the node supports NVLS; after a barrier every rank's
full C must equal a single-GPU GEMM of the whole problem with the same kernel version, bit
for bit, and pass the reference's check_error against the CPU oracle.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, multicast, side_stream, q):
    import sys
    from datetime import timedelta
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    import oracle
    import vibegemm_b200 as vg
    from vibegemm_b200.mgpu import FusedAllGatherGemm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        A, B = oracle.make_inputs(M, N, K)
        fused = FusedAllGatherGemm(M, N, K, rank, world, multicast=multicast)
        r0, rows = fused.sh.local
        dA = torch.from_numpy(A[r0:r0 + rows].view(np.int16).copy()).cuda().view(torch.float16)
        dB = torch.from_numpy(B.view(np.int16).copy()).cuda().view(torch.float16)
        # Twice: repeated launches into the same buffers. On a side stream, the barrier must
        # still order every rank's kernel (it synchronises the device before the collective).
        s = torch.cuda.Stream() if side_stream else torch.cuda.current_stream()
        s.wait_stream(torch.cuda.current_stream())
        for _ in range(2):
            fused.run(dA, dB, stream=s)
        fused.barrier()
        # Reference: the whole problem on this GPU with the version the shards resolved to.
        # Every version except stream-K keeps one accumulation chain per output and agrees
        # bit for bit, but the whole problem's own per-shape choice may be stream-K.
        v = vg.plan(-1, rows, N, K, 256, 256, 256, allgather=True)["version"]
        full = vg.gemm(torch.from_numpy(A.view(np.int16).copy()).cuda().view(torch.float16), dB,
                       version=v)
        torch.cuda.synchronize()
        got = fused.C.cpu().view(torch.int16).numpy().view(np.uint16)
        if K <= 8192:
            # And against the CPU oracle (the reference's naive GEMM restated), with the
            # reference engine's check_error: an error common to both GPU launches would not
            # pass this.
            ok_oracle, st = oracle.check_error(oracle.gemm_f16(A, B), got)
        else:
            # Long K (chunked accumulation): rows of both shards against the fp64 product,
            # BASELINE tolerances (bounded relative error <= 1e-2, per-element check_error
            # form with atol 2e-2*sqrt(K/1024)).
            rows = [0, 1, M // 2 - 1, M // 2, M - 1]
            exact = np.concatenate([oracle.gemm_f64(A, B, r, 1) for r in rows])
            c = got[rows].view(np.float16).astype(np.float64)
            st = oracle.acceptance(c, exact, K=K)
            ok_oracle = st["max_rel"] <= 1e-2 and bool(
                np.all(np.abs(c - exact) <= st["abs_bound"] + 1e-2 * np.abs(exact)))
        q.put((rank, bool(torch.equal(fused.C, full)), vg.device_status(), bool(fused.c_multicast_ptr),
               bool(ok_oracle), str(st)))
        fused.barrier()
        del fused
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("side_stream", [False, True], ids=["current_stream", "side_stream"])
@pytest.mark.parametrize("multicast", [False, True], ids=["p2p", "nvls"])
@pytest.mark.parametrize("M,N,K", [(1536, 2048, 1024), (1001, 1024, 4099), (5120, 4096, 16384)])
def test_fused_gemm_allgather_two_gpus(M, N, K, multicast, side_stream):
    """(5120, 4096, 16384): each rank's 2560-row shard is a full wave of pair tiles at long K,
    so the shards run v8 (run-time tiles, chunked accumulation) with the peer epilogue."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, multicast, side_stream, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert [r[1] for r in res] == [True, True], res
    assert [r[2] for r in res] == [0, 0], res
    assert [r[4] for r in res] == [True, True], res  # each rank's full C vs the oracle
    if multicast and not res[0][3]:
        pytest.skip("no NVLink multicast on this node (per-peer path was checked)")
