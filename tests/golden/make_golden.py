"""Generate tests/golden/f4gemm_ref_golden.npz from the reference's own code.

The reference's asm_f4gemm host files (f4gemm_ref.hpp, f4gemm.hpp) are compiled
from the reference tree into oracle/_ref/libf4gemm_ref.so (oracle/Makefile,
REF=<reference root>).  This script calls that library -- the real reference
implementation, not a restatement -- and stores its outputs as small fixtures,
so the tests can pin the oracle and the product's host logic on machines where
the reference tree is absent.

    make -C oracle REF=<reference root> && python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "f4gemm_ref_golden.npz")

# A manifest shaped like aiter's f4gemm list (tiles, splitK capability, B
# preshuffle) to exercise every branch of select_kernel, plus the library's own.
SYNTH_MANIFEST = np.array([
    # tile_M, tile_N, splitK, bpreshuffle
    [256, 256, 1, 1], [128, 512, 1, 1], [96, 640, 1, 1], [128, 256, 1, 1], [64, 256, 0, 1],
    [32, 128, 1, 1], [256, 128, 1, 1], [160, 384, 0, 1], [256, 256, 0, 0],
], dtype=np.int32)
LIB_MANIFEST = np.array([[128, 256, 1, 0], [128, 128, 1, 0], [128, 256, 1, 1], [128, 128, 1, 1],
                        [256, 256, 1, 0], [256, 256, 1, 1]], dtype=np.int32)

# asm_f4gemm/run_tests.sh:363-367 heuristic shapes, the split-K sweep shape and
# the benchmark configs' shapes
SHAPES = np.array([
    [128, 1024, 1024], [256, 2048, 2048], [300, 2048, 1024], [1, 4096, 2048], [17, 512, 256],
    [512, 1024, 2048], [2048, 8192, 1024], [4096, 4096, 512], [256, 1024, 4096], [8192, 8192, 8192],
    [512, 512, 512], [1, 28672, 4096], [16, 28672, 4096], [64, 28672, 4096], [16, 4096, 14336],
    [128, 7168, 2048], [16384, 7168, 18432], [65536, 28672, 8192],
], dtype=np.int32)


def det_bytes(n: int, salt: int) -> np.ndarray:
    i = np.arange(n, dtype=np.uint64)
    return ((i * np.uint64(2654435761) + np.uint64(salt)) >> np.uint64(7)).astype(np.uint8)


def main() -> None:
    R = O.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libf4gemm_ref.so missing: make -C oracle REF=<reference root>")
    g: dict[str, np.ndarray] = {}

    g["e8m0"] = np.array([R.ref_e8m0_to_f32(i) for i in range(256)], dtype=np.float32)

    N, Kp = 48, 128
    src = det_bytes(N * Kp, 11)
    dst = np.empty_like(src)
    R.ref_shuffle_weight_16x16(src, dst, N, Kp)
    g["sw_src"], g["sw_dst"], g["sw_shape"] = src, dst, np.array([N, Kp], np.int32)

    rows, cols, sm, sn = 40, 12, 256, 16
    s = det_bytes(rows * cols, 5)
    d = np.empty(sm * sn, np.uint8)
    R.ref_shuffle_scale(s, rows, cols, sm, sn, d)
    g["ss_src"], g["ss_dst"], g["ss_shape"] = s, d, np.array([rows, cols, sm, sn], np.int32)

    shp = []
    for M, Nn, K in SHAPES:
        o = np.empty(7, np.int32)
        R.ref_shape(int(M), int(Nn), int(K), o)
        shp.append(o)
    g["shape_out"] = np.array(shp)

    opers = {}
    for name, rows_, K, seed in (("a", 8, 64, 1234), ("b", 4, 64, 5678)):
        packed = np.empty(rows_ * K // 2, np.uint8)
        scales = np.empty(rows_ * K // 32, np.uint8)
        deq = np.empty(rows_ * K, np.float32)
        R.ref_make_operand(rows_, K, seed, packed, scales, deq)
        g[f"op_{name}_packed"], g[f"op_{name}_scales"], g[f"op_{name}_dequant"] = packed, scales, deq
        opers[name] = deq
    D = np.empty(8 * 4, np.float32)
    R.ref_reference_gemm(opers["a"], opers["b"], 8, 4, 64, 1.0, D)
    g["ref_gemm_D"] = D

    for mname, man in (("synth", SYNTH_MANIFEST), ("lib", LIB_MANIFEST)):
        rows_out = []
        for M, Nn, K in SHAPES:
            for num_cu in (148, 256):
                for l2 in (-1, 0, 1, 2, 4):
                    for bps in (0, 1):
                        idx, lo = C.c_int(), C.c_int()
                        R.ref_select_kernel(int(M), int(Nn), int(K), num_cu, l2, bps, len(man),
                                            np.ascontiguousarray(man[:, 0]), np.ascontiguousarray(man[:, 1]),
                                            np.ascontiguousarray(man[:, 2]), np.ascontiguousarray(man[:, 3]),
                                            C.byref(idx), C.byref(lo))
                        rows_out.append([M, Nn, K, num_cu, l2, bps, idx.value, lo.value])
        g[f"select_{mname}"] = np.array(rows_out, np.int32)
    g["manifest_synth"], g["manifest_lib"] = SYNTH_MANIFEST, LIB_MANIFEST

    ml = []
    for tm, tn, sk in ((256, 256, 1), (128, 512, 1), (64, 256, 0), (96, 640, 1)):
        for M, Nn, K in SHAPES:
            for l2 in (0, 1, 2, 3, 4, 7):
                o = np.zeros(5, np.int32)
                rc = R.ref_make_launch(tm, tn, sk, int(M), int(Nn), int(K), l2, o)
                ml.append([tm, tn, sk, M, Nn, K, l2, rc, *o])
    g["make_launch"] = np.array(ml, np.int32)

    buf = np.zeros(R.ref_kernel_args_size(), np.uint8)
    R.ref_fill_args(buf, C.c_void_p(0x1000), C.c_void_p(0x2000), C.c_void_p(0x3000), C.c_void_p(0x4000),
                    C.c_void_p(0x5000), C.c_void_p(0x6000), 300, 2048, 1024, 2048, 32, 32, 1.5, 0.0, 2)
    g["fill_args"] = buf

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
