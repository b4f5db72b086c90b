"""Host-side mirror of the reference's f4gemm launch helpers, for MXFP8.

Same names, argument meaning and error behaviour as asm_f4gemm/f4gemm.hpp and
asm_f4gemm/f4gemm_ref.hpp (the manifest loader, the tile heuristic, the grid /
split-K rule, the kernarg filler, the padded buffer geometry), so a host driver
written against the reference reads the same here.  The kernels behind it are
this library's sm_100a ones (``capi.b2g_gemm_mxfp8_f4gemm``), and the manifest
is the library's own tile table (``manifest/b2g_mxfp8_sm100a.csv``) instead of
aiter's code-object list.
"""
from __future__ import annotations

import csv
import ctypes as C
import os
from dataclasses import dataclass, field

from . import capi

MANIFEST = os.path.join(os.path.dirname(os.path.abspath(__file__)), "manifest", "b2g_mxfp8_sm100a.csv")


class F4gemmError(RuntimeError):
    """Raised where the reference host code prints a message and exits."""


@dataclass
class Config:  # asm_f4gemm/f4gemm.hpp:120-128
    tile_M: int = 0
    tile_N: int = 0
    splitK: int = 0
    bpreshuffle: int = 0
    knl_name: str = ""
    co_name: str = ""


def load_configs(csv_path: str = MANIFEST) -> list[Config]:
    """asm_f4gemm/f4gemm.hpp:141-200: columns taken from the header row; rows with
    a different field count or without names are skipped."""
    if not os.path.exists(csv_path):
        raise F4gemmError(f"[f4gemm] cannot open manifest {csv_path}")
    with open(csv_path, newline="") as f:
        lines = f.read().splitlines()
    if not lines:
        raise F4gemmError(f"[f4gemm] empty manifest {csv_path}")
    cols = [c.strip() for c in lines[0].split(",")]
    out = []
    for line in lines[1:]:
        if not line.strip():
            continue
        vals = [v.strip() for v in line.split(",")]
        if len(vals) != len(cols):
            continue
        c = Config()
        for k, v in zip(cols, vals):
            if k == "tile_M":
                c.tile_M = int(v)
            elif k == "tile_N":
                c.tile_N = int(v)
            elif k == "splitK":
                c.splitK = int(v)
            elif k == "bpreshuffle":
                c.bpreshuffle = int(v)
            elif k == "knl_name":
                c.knl_name = v
            elif k == "co_name":
                c.co_name = v
        if c.knl_name and c.co_name:
            out.append(c)
    return out


def select_kernel(M: int, N: int, K: int, num_cu: int, log2_k_split: int, bpreshuffle: int,
                  cfgs: list[Config]) -> tuple[int, int]:
    """asm_f4gemm/f4gemm.hpp:210-267 -> (index or -1, log2 split)."""
    empty_cu, rnd, effi = num_cu, 0xFFFFFFFF, 1.0
    split_en = 1 if log2_k_split > 0 else 0
    bpre_en = 0 if bpreshuffle == 0 else 1
    sel, sel_split = -1, 1
    for i, cfg in enumerate(cfgs):
        if cfg.bpreshuffle != bpre_en or cfg.splitK < split_en:
            continue
        if cfg.tile_M == 128 and cfg.tile_N == 512 and N % cfg.tile_N != 0:
            continue
        if log2_k_split >= 0 and cfg.splitK:
            splits = [1 << log2_k_split]
        elif cfg.splitK:
            splits = [2, 4, 8, 16]
        else:
            splits = [1]
        for sk in splits:
            tg = ((M + cfg.tile_M - 1) // cfg.tile_M) * ((N + cfg.tile_N - 1) // cfg.tile_N) * sk
            lr = (tg + num_cu - 1) // num_cu
            le = float(C.c_float(cfg.tile_M * cfg.tile_N / (cfg.tile_M + cfg.tile_N)).value)
            earlier, same = lr < rnd, lr == rnd
            more_busy = empty_cu > (lr * num_cu - tg)
            better = le > effi
            if earlier or (same and (more_busy or better)):
                rnd, empty_cu, effi, sel, sel_split = lr, lr * num_cu - tg, le, i, sk
    return sel, sel_split.bit_length() - 1


@dataclass
class LaunchDesc:  # asm_f4gemm/f4gemm.hpp:322-327
    gdx: int = 0
    gdy: int = 0
    gdz: int = 1
    log2_k_split: int = 0
    zero_out: bool = False


def make_launch(cfg: Config, M: int, N: int, K: int, log2_k_split: int) -> LaunchDesc:
    """asm_f4gemm/f4gemm.hpp:329-349 (raises where the reference exits)."""
    d = LaunchDesc()
    if cfg.splitK == 1:
        d.log2_k_split = log2_k_split
        k_num = 1 << d.log2_k_split
        if K % k_num != 0:
            raise F4gemmError(f"[f4gemm] K({K}) % (1 << log2_k_split)({k_num}) != 0")
        d.zero_out = k_num > 1
        k_per_tg = K // k_num
        k_per_tg = ((k_per_tg + 255) // 256) * 256
        d.gdz = (K + k_per_tg - 1) // k_per_tg
    d.gdx = (N + cfg.tile_N - 1) // cfg.tile_N
    d.gdy = (M + cfg.tile_M - 1) // cfg.tile_M
    return d


def fill_args(d_D, d_C, d_A, d_B, d_ScaleA, d_ScaleB, M, N, K, stride_D0, stride_ScaleA0, stride_ScaleB0,
              alpha, beta, log2_k_split) -> capi.F4gemmKernelArgs:
    """asm_f4gemm/f4gemm.hpp:355-392.  For MXFP8 an element is a byte, so the
    A/B strides in elements (K) are byte strides."""
    a = capi.F4gemmKernelArgs()
    C.memset(C.byref(a), 0, C.sizeof(a))
    a.ptr_D, a.ptr_C, a.ptr_A, a.ptr_B = d_D, d_C, d_A, d_B
    a.alpha, a.beta = alpha, beta
    a.stride_C0 = stride_D0  # the kernels read stride_C0 for D as well
    a.stride_D0 = stride_D0
    a.stride_A0 = K
    a.stride_B0 = K
    a.M, a.N, a.K = M, N, K
    a.ptr_ScaleA, a.ptr_ScaleB = d_ScaleA, d_ScaleB
    a.stride_ScaleA0 = stride_ScaleA0
    a.stride_ScaleB0 = stride_ScaleB0
    a.log2_k_split = log2_k_split
    return a


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def round_up(a: int, b: int) -> int:
    return cdiv(a, b) * b


@dataclass
class Shape:
    """Padded buffer geometry, asm_f4gemm/f4gemm_ref.hpp:61-73, with one byte per
    E4M3 element (the reference's Kp = K/2 packs two e2m1 values per byte)."""
    M: int
    N: int
    K: int
    elem_bits: int = field(default=8)

    def Kp(self) -> int:
        return self.K * self.elem_bits // 8

    def Ks(self) -> int:
        return self.K // 32

    def scale_cols(self) -> int:
        return round_up(self.Ks(), 8)

    def a_rows_pad(self) -> int:
        return round_up(self.M, 256)

    def b_rows_pad(self) -> int:
        return round_up(self.N, 256)

    def scale_a_rows(self) -> int:
        return round_up(self.M, 256)

    def scale_b_rows(self) -> int:
        return round_up(self.N, 256)

    def d_rows_pad(self) -> int:
        return round_up(self.M, 32)


def launch(args: capi.F4gemmKernelArgs, bpreshuffle: int, out_dtype: int = capi.OUT_BF16, stream: int = 0,
           fp4: bool = False) -> None:
    """Kernel::launch (asm_f4gemm/f4gemm.hpp:297-309) on this library's kernels: MXFP8
    operands, or with fp4=True the reference's own MXFP4 (packed E2M1) operands."""
    fn = "b2g_gemm_mxfp4_f4gemm" if fp4 else "b2g_gemm_mxfp8_f4gemm"
    capi.check(getattr(capi.lib(), fn)(C.byref(args), int(bpreshuffle), int(out_dtype), C.c_void_p(stream)), fn)
