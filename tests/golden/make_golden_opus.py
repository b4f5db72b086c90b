"""Generate tests/golden/opus_gemm_ref_golden.npz from the reference's own opus
CPU GEMMs.

``oracle/extract_gemm_ref.py`` cuts the unchanged ``gemm_ref`` functions out of
the reference's host sources and ``oracle/Makefile`` compiles them into
``oracle/_ref/libopus_ref.so``.  This script runs that library -- the reference's
own loops, not a restatement -- on seeded operands (``oracle.opus_case``) and
stores inputs and outputs as small fixtures, so that the oracle's restatements
stay pinned where the reference tree is absent.

    make -C oracle REF=<reference root> && python tests/golden/make_golden_opus.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "opus_gemm_ref_golden.npz")

# (loop, recipe, M, N, K, seed): the four loops, each on the reference hosts' own
# data recipe; the block-scale loops also on N(0,1) data quantised as the
# benchmarks do and on every finite E4M3 byte with wide-range scales
CASES = [
    ("blockscale", "uniform", 16, 256, 256, 11),
    ("blockscale", "normal", 16, 256, 256, 12),
    ("blockscale", "bytes", 8, 256, 256, 13),
    ("blockscale_1x128x1", "uniform", 16, 256, 256, 21),
    ("blockscale_1x128x1", "normal", 16, 256, 256, 22),
    ("blockscale_1x128x1", "bytes", 8, 128, 256, 23),
    ("fp8_gemm", "uniform", 16, 64, 256, 31),
    ("fp8_gemm", "bytes", 8, 64, 256, 32),
    ("flatmm", "uniform", 16, 64, 256, 41),
    ("flatmm", "bytes", 8, 64, 256, 42),
]


def main() -> None:
    if O.opus_ref_lib() is None:
        raise SystemExit("oracle/_ref/libopus_ref.so missing: make -C oracle REF=<reference root>")
    g: dict[str, np.ndarray] = {"cases": np.array([f"{c[0]}|{c[1]}|{c[2]}|{c[3]}|{c[4]}|{c[5]}" for c in CASES])}
    for i, (loop, recipe, M, N, K, seed) in enumerate(CASES):
        case = O.opus_case(loop, recipe, M, N, K, seed)
        for key in ("a", "b", "sfa", "sfb"):
            if key in case:
                g[f"{i}_{key}"] = case[key]
        g[f"{i}_c"] = O.run_opus_case(case, "reference")
    g["e4m3"] = np.array([O.opus_ref_lib().ref_opus_e4m3_to_f32(v) for v in range(256)], np.float32)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
