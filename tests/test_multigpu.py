"""Column-parallel MXFP8 GEMM over two GPUs with the output all-gather folded into
the GEMM epilogue (b2g_gemm_mxfp8_peer_out: every rank's columns are stored
straight into every rank's full-width C in symmetric memory), and the NCCL
all-gather form, against the single-GPU GEMM of the full problem on the same
seeded inputs.  Each element is accumulated the same way in all three, so the
results must be bit-identical.  Needs two GPUs (skipped otherwise); the ranks are
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
            assert ops.device_status() == 0
            dist.barrier()
            del c_full
    finally:
        dist.destroy_process_group()


def test_column_parallel_peer_out_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from gcnasm_b200 import build
    build.build()
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)
