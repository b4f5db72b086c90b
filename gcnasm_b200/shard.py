"""Multi-GPU partitioning of the MXFP8 GEMM (one process per GPU).

* M-shard (primary): rank g owns rows [row0, row0 + rows) of A / SFA / C, B is
  replicated; no collective on the data path.  Row ranges are multiples of 128
  so that a shard of the tensor-core scale layout is a pointer offset.
* N-shard (column parallel): rank g owns columns [col0, col0 + cols) of B / SFB
  / C and A is replicated; the bf16 column slabs are all-gathered over NCCL
  (NVLink) into [G, M, cols], handed over as that slab layout or re-assembled
  into [M, N]; or gathered panel by panel while the GEMM computes the next panel.
* N-shard with the gather folded into the GEMM: every rank's full-width C lives
  in symmetric memory (mapped into every process); each rank's GEMM epilogue
  stores its columns straight into all ranks' C over NVLink, and a one-element
  NCCL all-reduce on the stream orders the ranks before C is read.

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
                        group=None, layout: str = "mn") -> torch.Tensor:
    """Column-parallel GEMM + all-gather of the output slabs.

    layout "mn": the full C [M, N] (the gathered slabs re-assembled, one copy);
    layout "slabs": C as gathered, [world, M, N / world] -- slab g holds columns
    [g * N / world, (g + 1) * N / world) -- written by the collective in place,
    with no assembly copy.  Every rank takes the same collective steps; column
    shards must be equal-sized (N divisible by 128 * world)."""
    col0, cols = col_range(N, world, rank)
    assert N % (128 * world) == 0, "N-shard needs N divisible by 128 * world"
    assert layout in ("mn", "slabs")
    c_local = local_gemm(col0, cols).contiguous()  # [M, cols]
    M = c_local.shape[0]
    out = torch.empty((world, M, cols), dtype=c_local.dtype, device=c_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, c_local, group=group)  # straight into the slabs
    else:  # backends without the flat form (gloo, the CPU tests): one slab view per rank
        dist.all_gather(list(out.unbind(0)), c_local, group=group)
    if layout == "slabs":
        return out
    return out.permute(1, 0, 2).reshape(M, N)


def n_sharded_allgather_panels(local_gemm_rows: Callable[[int, int], torch.Tensor], M: int, N: int, world: int,
                               rank: int, panels: int = 4, group=None) -> torch.Tensor:
    """Column-parallel GEMM whose output all-gather overlaps the GEMM itself.

    The rank's GEMM runs in `panels` row panels (local_gemm_rows(row0, rows) ->
    this rank's columns of C rows [row0, row0 + rows), [rows, N / world]); each
    panel's all-gather is started asynchronously as soon as the panel is computed
    and runs on the collective's own stream while the next panel's GEMM runs.
    Returns C in the slab layout [world, M, N / world] (see n_sharded_allgather),
    complete once the call returns (the current stream waits for every gather)."""
    col0, cols = col_range(N, world, rank)
    assert N % (128 * world) == 0, "N-shard needs N divisible by 128 * world"
    out = None
    works = []
    rows_per = -(-M // panels)
    rows_per = -(-rows_per // 128) * 128  # panels start on 128-row tile (and scale-atom) boundaries
    for row0 in range(0, M, rows_per):
        rows = min(rows_per, M - row0)
        c_p = local_gemm_rows(row0, rows).contiguous()
        if out is None:
            out = torch.empty((world, M, cols), dtype=c_p.dtype, device=c_p.device)
        # slab g's rows [row0, row0 + rows) are contiguous, so every rank's piece lands in place
        works.append(dist.all_gather([out[g, row0:row0 + rows] for g in range(world)], c_p, group=group,
                                     async_op=True))
    for w in works:
        w.wait()
    return out


def peer_output(M: int, N: int, dtype: torch.dtype, group=None) -> tuple[torch.Tensor, list[int]]:
    """This rank's full-width [M, N] C in torch symmetric memory and the base
    address of every rank's C as mapped into this process (rank order)."""
    from torch.distributed import _symmetric_memory as symm_mem

    g = group if group is not None else dist.group.WORLD
    c = symm_mem.empty((M, N), dtype=dtype, device=torch.device("cuda", torch.cuda.current_device()))
    handle = symm_mem.rendezvous(c, g)
    return c, [int(x) for x in handle.buffer_ptrs]


def n_sharded_peer_out(qa: torch.Tensor, sfa: torch.Tensor, qb_local: torch.Tensor, sfb_local: torch.Tensor,
                       c_full: torch.Tensor, peer_ptrs: list[int], N: int, world: int, rank: int,
                       barrier: torch.Tensor, group=None) -> torch.Tensor:
    """Column-parallel MXFP8 GEMM with the all-gather folded into its epilogue:
    this rank's columns go straight into every rank's c_full; `barrier` (one
    float32 element on this GPU) carries the all-reduce that orders the ranks
    before any of them reads c_full.  Returns c_full, complete on every rank."""
    from . import ops

    col0, cols = col_range(N, world, rank)
    assert qb_local.shape[0] == cols and len(peer_ptrs) == world
    ops.mxfp8_gemm_peer_out(qa, qb_local, sfa, sfb_local, c_full, peer_ptrs, rank, col0)
    dist.all_reduce(barrier, group=group)
    return c_full


def a2a_window(M: int, N: int, world: int, dtype: torch.dtype, group=None) -> tuple[torch.Tensor, list[int]]:
    """This rank's all-to-all receive window [world * M, N / world] (rows grouped by
    source rank) in torch symmetric memory, and every rank's window as mapped into
    this process (rank order)."""
    return peer_output(world * M, N // world, dtype, group)


def gemm_a2a(qa: torch.Tensor, sfa: torch.Tensor, qb: torch.Tensor, sfb: torch.Tensor, window: torch.Tensor,
             peer_ptrs: list[int], rank: int, barrier: torch.Tensor, group=None) -> torch.Tensor:
    """MXFP8 GEMM whose output is all-to-all'd in its epilogue (the opus_gemm_dist
    GEMM -> A2A step): this rank computes C for its own M rows and all N columns and
    column shard q lands in rank q's window rows [rank * M, (rank + 1) * M).  The
    all-reduce of `barrier` orders the ranks before any reads its window.  Returns
    this rank's window: [world * M, N / world], block s from source rank s."""
    from . import ops

    ops.mxfp8_gemm_a2a_out(qa, qb, sfa, sfb, window, peer_ptrs, rank)
    dist.all_reduce(barrier, group=group)
    return window
