"""Row-block sharding of one GEMM across the GPUs of a node (one process per GPU).

C[M,N] = A[M,K] · B[N,K]^T is split by contiguous row blocks of A (and C): rank r owns
rows [r·ceil(M/P), min(M, (r+1)·ceil(M/P))) — the same split as the C ABI's
``vg_shard_rows``. B is replicated on every rank. K is never split, so the data path
needs no reduction; the only optional collective is an all-gather of C, which is
copy-free because the row-major C shards are contiguous slices of the full C
(uneven last shards are padded to the common block height for the collective).

The compute step is a parameter (``gemm_fn``): the B200 kernel on GPUs, the CPU oracle in
the world-size-2 gloo tests of this host logic.

``FusedAllGatherGemm`` replaces GEMM-then-all-gather by one kernel per rank
(``vg_b200_gemm_f16_allgather``): its epilogue writes every finished C tile into the full C
of every rank over NVLink while the tensor cores work on the next tile. The full-size C
buffers live in symmetric memory (torch's allocator maps each rank's buffer into every
peer's address space); torch is only the allocator and the barrier here.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, rows) of rank `rank`; identical to vg_shard_rows in the C ABI."""
    if M <= 0 or world <= 0 or not 0 <= rank < world:
        return 0, 0
    per = -(-M // world)
    lo = min(M, per * rank)
    hi = min(M, lo + per)
    return lo, hi - lo


@dataclass
class RowShardedGemm:
    M: int
    N: int
    K: int
    rank: int
    world: int

    @property
    def block_rows(self) -> int:
        return -(-self.M // self.world) if self.M > 0 else 0

    @property
    def local(self) -> tuple[int, int]:
        return shard_rows(self.M, self.world, self.rank)

    def run(self, A_local, B, C_local, gemm_fn: Callable) -> None:
        """Local shard product: C_local[rows, N] = A_local[rows, K] · B^T."""
        if self.local[1] > 0:
            gemm_fn(A_local, B, C_local)

    def gather(self, C_local, group=None):
        """All-gather of the row shards into the full M×N C (returned on every rank)."""
        import torch
        import torch.distributed as dist

        rows = self.local[1]
        blk = self.block_rows
        send = C_local
        if rows != blk:  # uneven tail shard: pad to the common block height
            send = torch.zeros((blk, self.N), dtype=C_local.dtype, device=C_local.device)
            if rows:
                send[:rows].copy_(C_local[:rows])
        full = torch.empty((blk * self.world, self.N), dtype=C_local.dtype, device=C_local.device)
        dist.all_gather_into_tensor(full, send.contiguous(), group=group)
        return full[: self.M]


class FusedAllGatherGemm:
    """Row-sharded GEMM with the all-gather of C fused into the kernel's epilogue.

    Every rank holds the full C (``self.C[:M]``, padded to world × block rows so all ranks
    allocate the same size) in symmetric memory. ``run`` launches the fused kernel on the
    current stream; call ``barrier`` before reading rows written by other ranks.
    """

    def __init__(self, M: int, N: int, K: int, rank: int, world: int, group=None,
                 multicast: bool = True):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.sh = RowShardedGemm(M, N, K, rank, world)
        self.rank, self.world = rank, world
        self.group = group if group is not None else dist.group.WORLD
        blk = self.sh.block_rows
        self.C_full = symm.empty((blk * world, N), dtype=torch.float16, device=torch.cuda.current_device())
        self.handle = symm.rendezvous(self.C_full, self.group)
        base = self.handle.buffer_ptrs[rank]
        offset = self.C_full.data_ptr() - base
        self.c_rank_ptrs = [int(p) + offset for p in self.handle.buffer_ptrs]
        # NVLink multicast (NVLS) address of the same buffers, when the node supports it.
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        self.c_multicast_ptr = mc + offset if (multicast and mc) else 0

    @property
    def C(self):
        return self.C_full[: self.sh.M]

    def run(self, A_local, B, stream=None) -> None:
        import vibegemm_b200 as vg
        r0, rows = self.sh.local
        if rows > 0:
            vg.gemm_allgather(A_local, B, self.c_rank_ptrs, self.rank, r0, stream,
                              self.c_multicast_ptr)

    def barrier(self) -> None:
        """Every rank's fused kernels (on any stream) have finished, so every rank's full C
        holds all rows. This device is synchronised BEFORE the process-group barrier: a
        barrier's own collective orders only the current stream (and a gloo barrier no GPU
        work at all), so a rank whose kernel ran on another stream could otherwise pass it
        while its peer stores are still landing."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        torch.cuda.synchronize()
