"""Column-parallel MXFP8 GEMM over two GPUs with the output all-gather folded into
the GEMM epilogue (b2g_gemm_mxfp8_peer_out: every rank's columns are stored
straight into every rank's full-width C in symmetric memory), and the NCCL
all-gather form, against the single-GPU GEMM of the full problem on the same
seeded inputs.  Each element is accumulated the same way in all three, so the
results must be bit-identical.  Then the GEMM -> all-to-all epilogue
(b2g_gemm_mxfp8_a2a_out) against each source rank's single-GPU GEMM.  Needs two GPUs (skipped otherwise); the ranks are
child processes with a short process-group timeout.
"""
import os
import socket

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int) -> None:
    import datetime
    import sys

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from gcnasm_b200 import ops, shard

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        for (M, N, K, dtype) in ((512, 1024, 1024, torch.bfloat16), (300, 512, 768, torch.float32)):
            g = torch.Generator(device=dev)
            qa, sfa = ops.quant_mxfp8(torch.randn(M, K, device=dev, generator=g.manual_seed(11)), "tc")
            qb, sfb = ops.quant_mxfp8(torch.randn(N, K, device=dev, generator=g.manual_seed(12)), "tc")
            ref = ops.mxfp8_gemm(qa, qb, sfa, sfb, out_dtype=dtype)
            col0, cols = shard.col_range(N, world, rank)
            qb_l = qb[col0:col0 + cols]
            sfb_l = sfb[shard.sf_tc_row_offset(col0, K):shard.sf_tc_row_offset(col0 + cols, K)]
            # fused: epilogue stores into every rank's C
            c_full, ptrs = shard.peer_output(M, N, dtype)
            c_full.fill_(float("nan"))
            dist.barrier()
            barrier = torch.zeros(1, device=dev)
            for _ in range(2):  # twice in a row: the same bits
                out = shard.n_sharded_peer_out(qa, sfa, qb_l, sfb_l, c_full, ptrs, N, world, rank, barrier)
                torch.cuda.synchronize()
                assert torch.equal(out, ref), (M, N, K, dtype, rank)
            # NCCL all-gather of the slabs
            def local(c0, nc):
                return ops.mxfp8_gemm(qa, qb_l, sfa, sfb_l, out_dtype=dtype)
            gathered = shard.n_sharded_allgather(local, N, world, rank)
            torch.cuda.synchronize()
            assert torch.equal(gathered, ref), (M, N, K, dtype, rank, "allgather")
            # slab layout [world, M, N / world], and gathered panel by panel under the GEMM
            slabs = shard.n_sharded_allgather(local, N, world, rank, layout="slabs")
            slab_ref = torch.stack([ref[:, g * cols:(g + 1) * cols] for g in range(world)])
            torch.cuda.synchronize()
            assert torch.equal(slabs, slab_ref), (M, N, K, dtype, rank, "slabs")
            if M % 128 == 0:
                def local_rows(r0, nr):
                    return ops.mxfp8_gemm(qa[r0:r0 + nr], qb_l,
                                          sfa[shard.sf_tc_row_offset(r0, K):shard.sf_tc_row_offset(r0 + nr, K)],
                                          sfb_l, out_dtype=dtype)
                panels = shard.n_sharded_allgather_panels(local_rows, M, N, world, rank, panels=3)
                torch.cuda.synchronize()
                assert torch.equal(panels, slab_ref), (M, N, K, dtype, rank, "panels")
            assert ops.device_status() == 0
            dist.barrier()
            del c_full
        # GEMM -> all-to-all (b2g_gemm_mxfp8_a2a_out): rank s computes C_s for its own
        # M rows and all N columns; rank r's window gets column shard r of every C_s
        M, N, K = 256, 1024, 512
        dtype = torch.bfloat16
        cols = N // world
        win, wptrs = shard.a2a_window(M, N, world, dtype)
        win.fill_(float("nan"))
        dist.barrier()
        g = torch.Generator(device=dev)
        qb, sfb = ops.quant_mxfp8(torch.randn(N, K, device=dev, generator=g.manual_seed(22)), "tc")
        refs, mine = [], None
        for src in range(world):
            qa_s, sfa_s = ops.quant_mxfp8(torch.randn(M, K, device=dev, generator=g.manual_seed(30 + src)), "tc")
            refs.append(ops.mxfp8_gemm(qa_s, qb, sfa_s, sfb, out_dtype=dtype))
            if src == rank:
                mine = (qa_s, sfa_s)
        barrier = torch.zeros(1, device=dev)
        out = shard.gemm_a2a(mine[0], mine[1], qb, sfb, win, wptrs, rank, barrier)
        torch.cuda.synchronize()
        for src in range(world):
            assert torch.equal(out[src * M:(src + 1) * M], refs[src][:, rank * cols:(rank + 1) * cols]), (src, rank)
        assert ops.device_status() == 0
        dist.barrier()
        del win
    finally:
        dist.destroy_process_group()


def test_column_parallel_peer_out_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from gcnasm_b200 import build
    build.build()
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)
