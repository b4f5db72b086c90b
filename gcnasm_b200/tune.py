"""Benchmark / tuning harness for the sm_100a FP8 GEMMs (one GPU).

The reference's host drivers time each kernel with 200 warm-up + 100 timed
launches and report TFLOP/s (opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_host.cc:92-126);
block_scale_1x128x1 adds BENCH_WARMUP / BENCH_ITERS / BENCH_ROUNDS and reports the
best / median / worst round (block_scale_1x128x1_gemm/..._host.cc:103-154); f4gemm
takes -m -n -k --splitk --bpreshuffle --iters (asm_f4gemm/main.cpp:32-109).  This
harness keeps those flags and environment knobs, adds the mode (mx | mx4 | blk | plain),
and with --sweep times every manifest tile x split candidate and writes a CSV
tuning table (tile choice per shape).

    python -m gcnasm_b200.tune --mode mx -m 8192 -n 8192 -k 8192
    python -m gcnasm_b200.tune --mode mx -m 16 -n 28672 -k 4096 --out f32 --sweep --csv table.csv
"""
from __future__ import annotations

import argparse
import csv
import os
import statistics
import sys

import torch

from . import capi, ops


def operands(mode, M, N, K, dev, group_n=128, bpre=False):
    g = torch.Generator(device=dev)
    if mode == "mx4":
        # the f4gemm data recipe (asm_f4gemm/f4gemm_ref.hpp:150-177): uniform E2M1 nibbles,
        # UE8M0 exponents 124..130
        qa = torch.randint(0, 256, (M, K // 2), dtype=torch.uint8, device=dev, generator=g.manual_seed(1234))
        qb = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g.manual_seed(5678))
        sa = torch.randint(124, 131, (M, K // 32), dtype=torch.uint8, device=dev, generator=g.manual_seed(11))
        sb = torch.randint(124, 131, (N, K // 32), dtype=torch.uint8, device=dev, generator=g.manual_seed(12))
        if bpre:
            qb = ops.shuffle_weight_16x16(qb)
        return qa, qb, ops.sf_rowmajor_to_tc(sa, K), ops.sf_rowmajor_to_tc(sb, K)
    x = torch.randn(M, K, device=dev, generator=g.manual_seed(1234))
    w = torch.randn(N, K, device=dev, generator=g.manual_seed(5678))
    if mode == "mx":
        qa, sfa = ops.quant_mxfp8(x, "tc")
        qb, sfb = ops.quant_mxfp8(w, "tc")
        if bpre:
            qb = ops.shuffle_weight_16x16(qb)
        return qa, qb, sfa, sfb
    if mode == "blk":
        qa, sfa = ops.quant_1x128(x)
        qb, sfb = ops.quant_128x128(w) if group_n == 128 else ops.quant_1x128(w)
        return qa, qb, sfa, sfb
    qa, _ = ops.quant_1x128(x)
    qb, _ = ops.quant_1x128(w)
    if bpre:
        qb = ops.shuffle_weight_16x16(qb)
    return qa, qb, None, None


def make_call(mode, ab, out, log2, group_n=128, bpre=False):
    qa, qb, sfa, sfb = ab
    if mode == "mx":
        return lambda: ops.mxfp8_gemm(qa, qb, sfa, sfb, out=out, log2_k_split=log2, b_preshuffled=bpre)
    if mode == "mx4":
        return lambda: ops.mxfp4_gemm(qa, qb, sfa, sfb, out=out, log2_k_split=log2, b_preshuffled=bpre)
    if mode == "blk":
        return lambda: ops.gemm_a8w8_blockscale(qa, qb, sfa, sfb, group_n=group_n, out=out, log2_k_split=log2)
    return lambda: ops.gemm_a8w8(qa, qb, out=out, log2_k_split=log2, b_preshuffled=bpre)


class Clocks:
    """Median SM clock (MHz) and power (W) of GPU 0 while the timed rounds run (NVML)."""

    def __init__(self):
        self.samples = []
        self._stop = None

    def __enter__(self):
        import threading
        import time
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        except Exception:
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                         nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
                except Exception:
                    pass
                time.sleep(0.002)

        self._thr = threading.Thread(target=loop, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *a):
        if self._stop:
            self._stop.set()
            self._thr.join(timeout=5)

    def summary(self):
        if not self.samples:
            return "clocks n/a"
        sm = statistics.median(c for c, _ in self.samples)
        pw = statistics.median(w for _, w in self.samples)
        return f"sm {sm:.0f} MHz  {pw:.0f} W"


def time_rounds(fn, warmup, iters, rounds, flush_bytes=0, graph=False):
    """Best / median / worst per-call milliseconds over `rounds` rounds of `iters` calls.

    graph=True captures the `iters` calls in one CUDA graph and times its
    replay: device time per call without the host's per-call cost (a GEMM of a
    few microseconds is otherwise bounded by the Python + ctypes call)."""
    buf = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda") if flush_bytes else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    run = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
    res = []
    for _ in range(rounds):
        if buf is not None:
            buf.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        if run is not None:
            run()
        else:
            for _ in range(iters):
                fn()
        b.record()
        torch.cuda.synchronize()
        res.append(a.elapsed_time(b) / iters)
    res.sort()
    return res[0], res[len(res) // 2], res[-1]


def algorithmic_bytes(mode, M, N, K, out_bytes, group_n=128):
    if mode == "mx":
        return M * K + N * K + (M + N) * (K // 32) + out_bytes * M * N
    if mode == "mx4":
        return (M * K + N * K) // 2 + (M + N) * (K // 32) + out_bytes * M * N
    if mode == "blk":
        sfb = (N // 128) * (K // 128) if group_n == 128 else N * (K // 128)
        return M * K + N * K + 4 * M * (K // 128) + 4 * sfb + out_bytes * M * N
    return M * K + N * K + out_bytes * M * N


def main(argv=None):
    env = os.environ
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--mode", choices=["mx", "mx4", "blk", "plain"], default="mx")
    ap.add_argument("-m", type=int, default=8192)
    ap.add_argument("-n", type=int, default=8192)
    ap.add_argument("-k", type=int, default=8192)
    ap.add_argument("--group-n", type=int, default=128)
    ap.add_argument("--out", choices=["bf16", "f32"], default="bf16")
    ap.add_argument("--splitk", type=int, default=0, help="log2 of the K split (-1: heuristic)")
    ap.add_argument("--bpreshuffle", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=int(env.get("BENCH_WARMUP", 20)))
    ap.add_argument("--iters", type=int, default=int(env.get("BENCH_ITERS", 20)))
    ap.add_argument("--rounds", type=int, default=int(env.get("BENCH_ROUNDS", 5)))
    ap.add_argument("--flush-l2", action="store_true", help="write 256 MiB before each round")
    ap.add_argument("--graph", action="store_true", help="replay the timed calls from a CUDA graph")
    ap.add_argument("--sweep", action="store_true", help="time split candidates 0..4 and report the best")
    ap.add_argument("--csv", default="", help="append sweep results to this CSV")
    a = ap.parse_args(argv)

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    M, N, K = a.m, a.n, a.k
    od = torch.bfloat16 if a.out == "bf16" else torch.float32
    ab = operands(a.mode, M, N, K, dev, a.group_n, bool(a.bpreshuffle))
    out = torch.empty((M, N), dtype=od, device=dev)
    flops = 2.0 * M * N * K
    nbytes = algorithmic_bytes(a.mode, M, N, K, out.element_size(), a.group_n)
    splits = list(range(0, 5)) if a.sweep else [a.splitk]
    rows = []
    for l2 in splits:
        fn = make_call(a.mode, ab, out, l2, a.group_n, bool(a.bpreshuffle))
        try:
            with Clocks() as clk:
                best, med, worst = time_rounds(fn, a.warmup, a.iters, a.rounds, 256 << 20 if a.flush_l2 else 0,
                                               a.graph)
        except capi.B2GError as e:
            print(f"split {l2}: {e}")
            continue
        tf = lambda t: flops / (t * 1e-3) / 1e12  # noqa: E731
        gb = lambda t: nbytes / (t * 1e-3) / 1e9  # noqa: E731
        print(f"[{a.mode} M={M} N={N} K={K} out={a.out} log2_split={l2} bpre={a.bpreshuffle}{' graph' if a.graph else ''}] "
              f"best={best * 1e3:.2f} us  median={med * 1e3:.2f} us  worst={worst * 1e3:.2f} us  "
              f"{tf(best):.1f} TFLOP/s  {gb(best):.1f} GB/s  [{clk.summary()}]")
        rows.append([a.mode, M, N, K, a.out, a.bpreshuffle, l2, f"{best * 1e3:.3f}", f"{tf(best):.2f}",
                     f"{gb(best):.1f}"])
    if a.sweep and rows:
        best = min(rows, key=lambda r: float(r[7]))
        print(f"best split: log2={best[6]} ({best[7]} us)")
    if a.csv and rows:
        new = not os.path.exists(a.csv)
        with open(a.csv, "a", newline="") as f:
            w = csv.writer(f)
            if new:
                w.writerow(["mode", "M", "N", "K", "out", "bpreshuffle", "log2_split", "us", "tflops", "gbs"])
            w.writerows(rows)
    st = ops.device_status()
    if st:
        print(f"device status {st}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
