"""Multi-GPU partitioning of the MXFP8 GEMM (one process per GPU).

* M-shard (primary): rank g owns rows [row0, row0 + rows) of A / SFA / C, B is
  replicated; no collective on the data path.  Row ranges are multiples of 128
  so that a shard of the tensor-core scale layout is a pointer offset.
* N-shard (column parallel): rank g owns columns [col0, col0 + cols) of B / SFB
  / C and A is replicated; the bf16 column slabs are all-gathered over NCCL
  (NVLink) into [G, M, cols] and transposed locally into [M, N].

The local compute step is injectable so that the partition / gather logic can be
exercised on CPU ranks (gloo) with a CPU stand-in; in production it is
``ops.mxfp8_gemm`` on the rank's own GPU.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def _range(total: int, world: int, rank: int, align: int) -> tuple[int, int]:
    blocks = (total + align - 1) // align
    per = (blocks + world - 1) // world
    lo = min(total, rank * per * align)
    hi = min(total, (rank + 1) * per * align)
    return lo, hi - lo


def row_range(M: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """(row0, rows) of rank's M-shard."""
    return _range(M, world, rank, align)


def col_range(N: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """(col0, cols) of rank's N-shard."""
    return _range(N, world, rank, align)


def sf_tc_row_offset(row0: int, k: int) -> int:
    """Byte offset of row `row0` (a multiple of 128) in a tensor-core-layout scale buffer."""
    assert row0 % 128 == 0
    return (row0 // 128) * ((k // 32 + 3) // 4) * 512


def m_sharded(local_gemm: Callable[[int, int], torch.Tensor], M: int, world: int, rank: int) -> torch.Tensor:
    """Run the rank's row shard: local_gemm(row0, rows) -> C rows [rows, N]."""
    row0, rows = row_range(M, world, rank)
    return local_gemm(row0, rows)


def n_sharded_allgather(local_gemm: Callable[[int, int], torch.Tensor], N: int, world: int, rank: int,
                        group=None) -> torch.Tensor:
    """Column-parallel GEMM + all-gather of the output slabs -> full C [M, N].

    Every rank takes the same collective steps; column shards must be equal-sized
    (N divisible by 128 * world) so that the slabs stack."""
    col0, cols = col_range(N, world, rank)
    assert N % (128 * world) == 0, "N-shard needs N divisible by 128 * world"
    c_local = local_gemm(col0, cols).contiguous()  # [M, cols]
    slabs = [torch.empty_like(c_local) for _ in range(world)]
    dist.all_gather(slabs, c_local, group=group)
    return torch.stack(slabs, 0).permute(1, 0, 2).reshape(c_local.shape[0], N)
