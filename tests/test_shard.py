"""Multi-GPU partitioning logic on CPU ranks (gloo, world size 2): the M-shard row
ranges and the N-shard all-gathers (assembled [M, N], slab layout, and panel by
panel) reassemble the full product.  The local GEMM
is the oracle here (a CPU stand-in injected by the test); on GPUs it is the
library's kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gcnasm_b200 import shard


def test_ranges_partition():
    for total in (1, 127, 128, 8192, 65536, 28672):
        for world in (1, 2, 4, 8):
            got = [shard.row_range(total, world, r) for r in range(world)]
            pos = 0
            for lo, n in got:
                assert n >= 0
                if n:
                    assert lo == pos and lo % 128 == 0
                pos += n
            assert pos == total
    assert shard.sf_tc_row_offset(256, 8192) == 2 * 64 * 512


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, N, K, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from oracle import oracle as O

    qa, sa = O.quant_mx(O.normal_rows(1234, 0, M, K))
    qb, sb = O.quant_mx(O.normal_rows(5678, 0, N, K))

    def local_rows(row0, rows):  # M-shard: this rank's rows, B replicated
        return torch.from_numpy(O.gemm_mx(qa[row0:row0 + rows], qb, sa[row0:row0 + rows], sb, rows, N, K))

    def local_cols(col0, cols):  # N-shard: this rank's columns, A replicated
        return torch.from_numpy(O.gemm_mx(qa, qb[col0:col0 + cols], sa, sb[col0:col0 + cols], M, cols, K))

    def local_rows_cols(row0, rows):  # N-shard by row panels: this rank's columns of rows [row0, row0 + rows)
        col0, cols = shard.col_range(N, world, rank)
        return torch.from_numpy(O.gemm_mx(qa[row0:row0 + rows], qb[col0:col0 + cols], sa[row0:row0 + rows],
                                          sb[col0:col0 + cols], rows, cols, K))

    part = shard.m_sharded(local_rows, M, world, rank)
    gathered = shard.n_sharded_allgather(local_cols, N, world, rank)
    slabs = shard.n_sharded_allgather(local_cols, N, world, rank, layout="slabs")
    panels = shard.n_sharded_allgather_panels(local_rows_cols, M, N, world, rank, panels=3)
    np.save(os.path.join(out_dir, f"m{rank}.npy"), part.numpy())
    np.save(os.path.join(out_dir, f"n{rank}.npy"), gathered.numpy())
    np.save(os.path.join(out_dir, f"s{rank}.npy"), slabs.numpy())
    np.save(os.path.join(out_dir, f"p{rank}.npy"), panels.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_m_and_n_shard_gloo_world2(tmp_path, oracle):
    M, N, K, world = 300, 512, 128, 2
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    qa, sa = oracle.quant_mx(oracle.normal_rows(1234, 0, M, K))
    qb, sb = oracle.quant_mx(oracle.normal_rows(5678, 0, N, K))
    full = oracle.gemm_mx(qa, qb, sa, sb, M, N, K)
    m_parts = np.concatenate([np.load(tmp_path / f"m{r}.npy") for r in range(world)], 0)
    assert np.array_equal(m_parts, full)
    cols = N // world
    slab_ref = np.stack([full[:, g * cols:(g + 1) * cols] for g in range(world)])
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"n{r}.npy"), full)
        assert np.array_equal(np.load(tmp_path / f"s{r}.npy"), slab_ref)
        assert np.array_equal(np.load(tmp_path / f"p{r}.npy"), slab_ref)
