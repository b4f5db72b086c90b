"""Host-side logic on CPU: the C ABI loads and exports every declared symbol,
its argument blocks match the reference's byte layouts, the tile heuristic /
launch rule / manifest reproduce the reference's own code (golden fixtures made
from oracle/_ref), and invalid calls return status codes without a GPU."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

from gcnasm_b200 import capi, f4gemm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b2g", "gemm.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(b2g_\w+)\s*\(", txt, re.M)))


def test_library_exports_every_declared_symbol():
    L = capi.lib()
    decl = declared_symbols()
    assert len(decl) >= 20
    assert set(decl) == set(capi.EXPORTS)
    for s in decl:
        assert hasattr(L, s), s
    assert L.b2g_version() >= 100


def test_kernel_args_bytes_match_reference(golden):
    a = f4gemm.fill_args(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000, 300, 2048, 1024, 2048, 32, 32, 1.5, 0.0, 2)
    mine = np.frombuffer(bytes(a), np.uint8)
    assert C.sizeof(a) == 0x174 == golden["fill_args"].size
    assert np.array_equal(mine, golden["fill_args"])


def _reference_root():
    from oracle import oracle as O
    return O.reference_root()


@pytest.mark.skipif(not (_reference_root() and os.path.isdir(os.path.join(_reference_root(), "opus_gemm"))),
                    reason="reference tree not present")
def test_c_header_layouts_match_reference_headers():
    ref = _reference_root()
    src = r'''
#include <cstddef>
#include <cstdio>
#define __host__
#define __device__
namespace refbs {
#include "opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_common.h"
}
namespace ref1x128 {
#include "opus_gemm/block_scale_1x128x1_gemm/gemm_a8w8_1x128x1_blockscale_common.h"
}
#include "b2g/gemm.h"
#define CHK(A, B, F) if (offsetof(A, F) != offsetof(B, F)) { printf("%s\n", #F); return 1; }
#define ALL(A, B) CHK(A,B,ptr_a) CHK(A,B,ptr_b) CHK(A,B,ptr_c) CHK(A,B,m) CHK(A,B,n) CHK(A,B,k) CHK(A,B,batch) \
  CHK(A,B,stride_a) CHK(A,B,stride_b) CHK(A,B,stride_c) CHK(A,B,stride_a_batch) CHK(A,B,stride_b_batch) \
  CHK(A,B,stride_c_batch) CHK(A,B,ptr_sfa) CHK(A,B,ptr_sfb) CHK(A,B,stride_sfa) CHK(A,B,stride_sfb) \
  CHK(A,B,stride_sfa_batch) CHK(A,B,stride_sfb_batch)
int main() {
  ALL(refbs::opus_gemm_kargs, ::opus_gemm_kargs)
  ALL(ref1x128::opus_gemm_kargs, ::opus_gemm_kargs)
  if (sizeof(refbs::opus_gemm_kargs) != sizeof(::opus_gemm_kargs)) return 2;
  if (sizeof(b2g_f4gemm_kargs) != 0x174) return 3;
  if (offsetof(b2g_f4gemm_kargs, stride_C0) != 0x80 || offsetof(b2g_f4gemm_kargs, M) != 0xe0 ||
      offsetof(b2g_f4gemm_kargs, ptr_ScaleA) != 0x110 || offsetof(b2g_f4gemm_kargs, log2_k_split) != 0x170) return 4;
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "t.cpp")
        open(p, "w").write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["g++", "-std=c++17", "-I", ref, "-I", os.path.join(ROOT, "include"), p, "-o", exe],
                       check=True)
        assert subprocess.run([exe]).returncode == 0


def test_select_kernel_mirror_matches_reference(golden):
    for mname in ("synth", "lib"):
        man = golden[f"manifest_{mname}"]
        cfgs = [f4gemm.Config(int(r[0]), int(r[1]), int(r[2]), int(r[3]), f"k{i}", f"k{i}.co")
                for i, r in enumerate(man)]
        for M, N, K, cu, l2, bps, idx, lo in golden[f"select_{mname}"]:
            got = f4gemm.select_kernel(int(M), int(N), int(K), int(cu), int(l2), int(bps), cfgs)
            assert got == (idx, lo), (mname, M, N, K, cu, l2, bps)


def test_b2g_select_matches_reference_on_library_manifest(golden):
    L = capi.lib()
    man = golden["manifest_lib"]
    assert L.b2g_manifest_size() == len(man)
    for i, r in enumerate(man):
        tm, tn, sk, bp = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        assert L.b2g_manifest_entry(i, C.byref(tm), C.byref(tn), C.byref(sk), C.byref(bp), None) == 0
        assert (tm.value, tn.value, sk.value, bp.value) == tuple(int(v) for v in r)
    for M, N, K, cu, l2, bps, idx, lo in golden["select_lib"]:
        i, tm, tn, l = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        rc = L.b2g_select(int(M), int(N), int(K), int(cu), int(l2), int(bps), C.byref(i), C.byref(tm),
                          C.byref(tn), C.byref(l))
        assert (rc == 0) == (idx >= 0)
        if idx >= 0:
            assert (i.value, l.value) == (idx, lo)


def test_manifest_csv_matches_library_table():
    cfgs = f4gemm.load_configs()
    L = capi.lib()
    assert len(cfgs) == L.b2g_manifest_size()
    for i, c in enumerate(cfgs):
        tm, tn, sk, bp, nm = C.c_int(), C.c_int(), C.c_int(), C.c_int(), C.c_char_p()
        L.b2g_manifest_entry(i, C.byref(tm), C.byref(tn), C.byref(sk), C.byref(bp), C.byref(nm))
        assert (c.tile_M, c.tile_N, c.splitK, c.bpreshuffle, c.knl_name) == (
            tm.value, tn.value, sk.value, bp.value, nm.value.decode())


def test_load_configs_matches_reference_parser(oracle):
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    cap = 64
    arr = [np.zeros(cap, np.int32) for _ in range(4)]
    n = R.ref_load_configs(f4gemm.MANIFEST.encode(), cap, *arr)
    cfgs = f4gemm.load_configs()
    assert n == len(cfgs)
    for i, c in enumerate(cfgs):
        assert (c.tile_M, c.tile_N, c.splitK, c.bpreshuffle) == tuple(int(a[i]) for a in arr)


def test_make_launch_mirror_matches_reference(golden):
    for tm, tn, sk, M, N, K, l2, rc, gdx, gdy, gdz, lo, zo in golden["make_launch"]:
        cfg = f4gemm.Config(int(tm), int(tn), int(sk))
        if rc:
            with pytest.raises(f4gemm.F4gemmError):
                f4gemm.make_launch(cfg, int(M), int(N), int(K), int(l2))
            continue
        d = f4gemm.make_launch(cfg, int(M), int(N), int(K), int(l2))
        assert (d.gdx, d.gdy, d.gdz, d.log2_k_split, int(d.zero_out)) == (gdx, gdy, gdz, lo, zo)


def test_shape_mirror_matches_reference(golden):
    from tests.golden.make_golden import SHAPES
    for (M, N, K), out in zip(SHAPES, golden["shape_out"]):
        s = f4gemm.Shape(int(M), int(N), int(K), elem_bits=4)  # the reference's packed e2m1
        assert [s.Kp(), s.Ks(), s.scale_cols(), s.a_rows_pad(), s.b_rows_pad(), s.scale_a_rows(),
                s.d_rows_pad()] == list(out)
    assert f4gemm.Shape(16, 4096, 8192).Kp() == 8192  # one byte per E4M3 element


def test_invalid_arguments_return_status_without_gpu():
    L = capi.lib()
    # null kargs
    assert L.b2g_gemm_a8w8_blockscale(None, 128, 0, 0, None) == capi.B2G_ERR_INVALID_ARG
    assert L.b2g_gemm_mxfp8_f4gemm(None, 1, 0, None) == capi.B2G_ERR_INVALID_ARG
    # bad out dtype / group_n / K / N / alignment (fake, never dereferenced pointers)
    k = capi.OpusGemmKargs()
    k.ptr_a, k.ptr_b, k.ptr_c, k.ptr_sfa, k.ptr_sfb = 0x10000, 0x20000, 0x30000, 0x40000, 0x50000
    k.m, k.n, k.k, k.batch = 256, 512, 256, 1
    k.stride_a, k.stride_b, k.stride_c, k.stride_sfa, k.stride_sfb = 256, 256, 512, 256, 2
    assert L.b2g_gemm_a8w8_blockscale(C.byref(k), 128, 7, 0, None) == capi.B2G_ERR_INVALID_ARG
    assert L.b2g_gemm_a8w8_blockscale(C.byref(k), 64, 1, 0, None) == capi.B2G_ERR_INVALID_ARG
    k.k = 200
    assert L.b2g_gemm_a8w8_blockscale(C.byref(k), 128, 1, 0, None) == capi.B2G_ERR_UNSUPPORTED
    k.k, k.n = 256, 500
    assert L.b2g_gemm_a8w8_blockscale(C.byref(k), 128, 1, 0, None) == capi.B2G_ERR_UNSUPPORTED
    k.n, k.ptr_a = 512, 0x10008
    assert L.b2g_gemm_a8w8_blockscale(C.byref(k), 128, 1, 0, None) == capi.B2G_ERR_ALIGNMENT
    k.ptr_a, k.m = 0x10000, 0
    assert L.b2g_gemm_a8w8_blockscale(C.byref(k), 128, 1, 0, None) == capi.B2G_ERR_INVALID_ARG
    a = f4gemm.fill_args(0x1000, 0x2008, 0x3000, 0x4000, 0x5000, 0x6000, 16, 4096, 4096, 4096, 128, 128, 1.0, 0.5, 0)
    assert L.b2g_gemm_mxfp8_f4gemm(C.byref(a), 1, 0, None) == capi.B2G_ERR_ALIGNMENT  # beta * C, C misaligned
    a = f4gemm.fill_args(0x1000, 0, 0x3000, 0x4000, 0x5000, 0x6000, 16, 4096, 4016, 4096, 128, 128, 1.0, 0.0, 0)
    assert L.b2g_gemm_mxfp8_f4gemm(C.byref(a), 1, 0, None) == capi.B2G_ERR_UNSUPPORTED  # K % 32
    assert L.b2g_shuffle_weight_16x16(None, None, 16, 32, None) == capi.B2G_ERR_INVALID_ARG
    assert L.b2g_set_wait_timeout_ms(0) == capi.B2G_ERR_INVALID_ARG
    assert capi.status_string(capi.B2G_ERR_DEVICE_TIMEOUT) == "device wait timed out"
    assert b"K" in L.b2g_last_error() or len(L.b2g_last_error()) > 0


def test_peer_out_validation_without_gpu():
    """b2g_gemm_mxfp8_peer_out refuses bad peer lists, offsets and pitches before any
    device work (fake, never dereferenced pointers)."""
    L = capi.lib()
    args = capi.Mxfp8Args(0x10000, 0x20000, 0x30000, 0x40000, 0, 512, 1024, 1024, 1024, 1024, 0, 1.0, 0,
                          capi.OUT_BF16, 0)
    ptrs = (C.c_void_p * 2)(0x100000, 0x200000)
    assert L.b2g_gemm_mxfp8_peer_out(None, ptrs, 2, 0, 2048, 0, None) == capi.B2G_ERR_INVALID_ARG
    assert L.b2g_gemm_mxfp8_peer_out(C.byref(args), ptrs, 0, 0, 2048, 0, None) == capi.B2G_ERR_INVALID_ARG
    assert L.b2g_gemm_mxfp8_peer_out(C.byref(args), ptrs, 9, 0, 2048, 0, None) == capi.B2G_ERR_INVALID_ARG
    assert L.b2g_gemm_mxfp8_peer_out(C.byref(args), ptrs, 2, 2, 2048, 0, None) == capi.B2G_ERR_INVALID_ARG
    # columns [1536, 2560) do not fit 2048-column buffers
    assert L.b2g_gemm_mxfp8_peer_out(C.byref(args), ptrs, 2, 1, 2048, 1536, None) == capi.B2G_ERR_INVALID_ARG
    # bf16 column offset of 4 elements = 8 bytes
    assert L.b2g_gemm_mxfp8_peer_out(C.byref(args), ptrs, 2, 1, 2048, 4, None) == capi.B2G_ERR_ALIGNMENT
    bad = (C.c_void_p * 2)(0x100000, 0x200008)
    assert L.b2g_gemm_mxfp8_peer_out(C.byref(args), bad, 2, 1, 2048, 1024, None) == capi.B2G_ERR_ALIGNMENT
    assert b"peer" in L.b2g_last_error()


def test_mxfp4_validation_without_gpu():
    """MXFP4 entries refuse K off the 256-element granule (the reference's f4gemm
    contract, asm_f4gemm/main.cpp:141-150) and odd element strides before any
    device work (fake, never dereferenced pointers)."""
    from gcnasm_b200 import f4gemm
    L = capi.lib()
    args = capi.Mxfp8Args(0x10000, 0x20000, 0x30000, 0x40000, 0x50000, 256, 1024, 1152, 1152, 1152, 1024, 1.0, 0,
                          capi.OUT_BF16, 0)
    assert L.b2g_gemm_mxfp4(C.byref(args), None) == capi.B2G_ERR_UNSUPPORTED  # K = 1152: not a multiple of 256
    args = capi.Mxfp8Args(0x10000, 0x20000, 0x30000, 0x40000, 0x50000, 256, 1024, 1024, 1025, 1024, 1024, 1.0, 0,
                          capi.OUT_BF16, 0)
    assert L.b2g_gemm_mxfp4(C.byref(args), None) == capi.B2G_ERR_ALIGNMENT  # odd element stride
    a = f4gemm.fill_args(0x50000, None, 0x10000, 0x20000, 0x30000, 0x40000, 256, 1024, 1056, 1024, 40, 40,
                         1.0, 0.0, 0)
    assert L.b2g_gemm_mxfp4_f4gemm(C.byref(a), 1, capi.OUT_BF16, None) == capi.B2G_ERR_UNSUPPORTED
    assert b"256" in L.b2g_last_error()


def test_epilogue_validation_without_gpu():
    """b2g_gemm_mxfp8_ex refuses misaligned C / bias before any device work."""
    L = capi.lib()
    args = capi.Mxfp8Args(0x10000, 0x20000, 0x30000, 0x40000, 0x50000, 256, 1024, 1024, 1024, 1024, 1024, 1.0, 0,
                          capi.OUT_BF16, 0)
    epi = capi.Epilogue(0x60008, 1024, 1.0, None)  # C base not 16-byte aligned
    assert L.b2g_gemm_mxfp8_ex(C.byref(args), C.byref(epi), None) == capi.B2G_ERR_ALIGNMENT
    epi = capi.Epilogue(0x60000, 1020, 1.0, None)  # ldc < N
    assert L.b2g_gemm_mxfp8_ex(C.byref(args), C.byref(epi), None) == capi.B2G_ERR_ALIGNMENT
    epi = capi.Epilogue(None, 0, 0.0, 0x70004)  # bias base not 16-byte aligned
    assert L.b2g_gemm_mxfp8_ex(C.byref(args), C.byref(epi), None) == capi.B2G_ERR_ALIGNMENT
    assert b"bias" in L.b2g_last_error()


def test_a2a_out_validation_without_gpu():
    """b2g_gemm_mxfp8_a2a_out refuses uneven or too narrow column shards and bad peer
    lists before any device work (fake, never dereferenced pointers)."""
    L = capi.lib()
    args = capi.Mxfp8Args(0x10000, 0x20000, 0x30000, 0x40000, 0, 512, 1024, 1024, 1024, 1024, 0, 1.0, 0,
                          capi.OUT_BF16, 0)
    ptrs = (C.c_void_p * 3)(0x100000, 0x200000, 0x300000)
    assert L.b2g_gemm_mxfp8_a2a_out(C.byref(args), ptrs, 3, 0, None) == capi.B2G_ERR_INVALID_ARG  # 1024 % 3
    args.n = 288
    assert L.b2g_gemm_mxfp8_a2a_out(C.byref(args), ptrs, 3, 0, None) == capi.B2G_ERR_UNSUPPORTED  # 96 % 64
    args.n = 1152
    assert L.b2g_gemm_mxfp8_a2a_out(C.byref(args), ptrs, 3, 3, None) == capi.B2G_ERR_INVALID_ARG  # self
    bad = (C.c_void_p * 3)(0x100000, 0x200008, 0x300000)
    assert L.b2g_gemm_mxfp8_a2a_out(C.byref(args), bad, 3, 0, None) == capi.B2G_ERR_ALIGNMENT


def test_sf_tc_bytes():
    L = capi.lib()
    assert L.b2g_sf_tc_bytes(8192, 8192) == 64 * 64 * 512
    assert L.b2g_sf_tc_bytes(1, 32) == 512
    assert L.b2g_sf_tc_bytes(129, 160) == 2 * 2 * 512
