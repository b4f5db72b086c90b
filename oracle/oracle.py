"""numpy/ctypes front end of the CPU checkers.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by ``__graft_entry__.smoke()`` and
by the CPU-baseline leg of ``bench.py`` -- and only there, as the checker.  The
product package ``gcnasm_b200`` never imports this module.

Two shared objects sit behind it:

* ``oracle/_build/liboracle.so`` -- the C restatement (``b2g_oracle.c``) of the
  reference's CPU GEMMs, formats, quantisers and layout shuffles;
* ``oracle/_ref/libf4gemm_ref.so`` -- the reference's own ``asm_f4gemm`` host
  code compiled from its sources (present only where the reference tree was
  available at build time; see ``oracle/Makefile``);
* ``oracle/_ref/libopus_ref.so`` -- the reference's own opus CPU ``gemm_ref``
  loops, cut unchanged out of its host sources (``oracle/extract_gemm_ref.py``)
  and compiled with an E4M3 stand-in for ``__hip_fp8_e4m3`` (same condition).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None
_OPUS = None

u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def reference_root() -> str | None:
    """The reference project tree, where this machine has it: $B2G_REFERENCE_ROOT,
    else a directory named ``reference`` beside this repository's root; None when
    neither exists (the checkers then use the prebuilt oracle/_ref libraries and the
    committed golden fixtures)."""
    cand = os.environ.get("B2G_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(cand) else None


def build(reference_root: str | None = None) -> None:
    """Compile the oracle (and, when the reference tree exists, oracle/_ref)."""
    cmd = ["make", "-s", "-C", HERE]
    if reference_root:
        cmd.append(f"REF={reference_root}")
    subprocess.run(cmd, check=True)


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        i64 = C.c_int64
        L.orc_e4m3_to_f32.argtypes = [C.c_uint8]; L.orc_e4m3_to_f32.restype = C.c_float
        L.orc_f32_to_e4m3.argtypes = [C.c_float]; L.orc_f32_to_e4m3.restype = C.c_uint8
        L.orc_e8m0_to_f32.argtypes = [C.c_uint8]; L.orc_e8m0_to_f32.restype = C.c_float
        L.orc_f32_to_bf16.argtypes = [C.c_float]; L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_mx_scale_byte.argtypes = [C.c_float]; L.orc_mx_scale_byte.restype = C.c_uint8
        L.orc_mt19937_64.argtypes = [C.c_uint64, u64p, C.c_size_t]
        L.orc_normal_rows.argtypes = [C.c_uint64, i64, i64, i64, f32p]
        L.orc_quant_mx.argtypes = [f32p, i64, i64, u8p, u8p]
        L.orc_quant_1x128.argtypes = [f32p, i64, i64, u8p, f32p]
        L.orc_quant_128x128.argtypes = [f32p, i64, i64, u8p, f32p]
        ci = C.c_int
        L.orc_gemm_blockscale.argtypes = [u8p, u8p, f32p, f32p, f32p] + [ci] * 11
        L.orc_gemm_blockscale_1x128x1.argtypes = [u8p, u8p, f32p, f32p, f32p] + [ci] * 11
        L.orc_gemm_blockscale_f64.argtypes = [u8p, u8p, f32p, f32p, f64p] + [ci] * 12
        L.orc_gemm_a8w8.argtypes = [u8p, u8p, f32p] + [ci] * 6
        L.orc_gemm_a8w8_kn.argtypes = [u8p, u8p, f32p] + [ci] * 6
        L.orc_gemm_mx.argtypes = [u8p, u8p, u8p, u8p] + [ci] * 7 + [C.c_float, ci, f32p, ci]
        L.orc_gemm_mxfp4.argtypes = [u8p, u8p, u8p, u8p] + [ci] * 7 + [C.c_float, ci, f32p, ci]
        L.orc_e2m1_to_f32.argtypes = [C.c_uint8]; L.orc_e2m1_to_f32.restype = C.c_float
        L.orc_f32_to_e2m1.argtypes = [C.c_float]; L.orc_f32_to_e2m1.restype = C.c_uint8
        L.orc_mxfp4_scale_byte.argtypes = [C.c_float]; L.orc_mxfp4_scale_byte.restype = C.c_uint8
        L.orc_quant_mxfp4.argtypes = [f32p, i64, i64, u8p, u8p]
        L.orc_shuffle_weight_16x16.argtypes = [u8p, u8p, ci, ci]
        L.orc_shuffle_scale.argtypes = [u8p, ci, ci, ci, ci, u8p]
        L.orc_flatmm_shuffle_b.argtypes = [u8p, u8p, ci, ci]
        L.orc_sf_to_tc_layout.argtypes = [u8p, ci, ci, u8p]
        L.orc_max_threads.restype = ci
        _LIB = L
    return _LIB


def ref_lib() -> C.CDLL | None:
    """The reference's own f4gemm host code (None when oracle/_ref was not built)."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libf4gemm_ref.so")
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        ci = C.c_int
        R.ref_e8m0_to_f32.argtypes = [C.c_uint8]; R.ref_e8m0_to_f32.restype = C.c_float
        R.ref_shuffle_weight_16x16.argtypes = [u8p, u8p, ci, ci]
        R.ref_shuffle_scale.argtypes = [u8p, ci, ci, ci, ci, u8p]
        R.ref_shape.argtypes = [ci, ci, ci, i32p]
        R.ref_make_operand.argtypes = [ci, ci, C.c_uint32, u8p, u8p, f32p]
        R.ref_reference_gemm.argtypes = [f32p, f32p, ci, ci, ci, C.c_float, f32p]
        R.ref_select_kernel.argtypes = [ci] * 7 + [i32p] * 4 + [C.POINTER(ci), C.POINTER(ci)]
        R.ref_make_launch.argtypes = [ci] * 7 + [i32p]; R.ref_make_launch.restype = ci
        R.ref_kernel_args_size.restype = ci
        R.ref_fill_args.argtypes = [u8p] + [C.c_void_p] * 6 + [ci] * 6 + [C.c_float, C.c_float, ci]
        R.ref_load_configs.argtypes = [C.c_char_p, ci, i32p, i32p, i32p, i32p]; R.ref_load_configs.restype = ci
        _REF = R
    return _REF


def opus_ref_lib() -> C.CDLL | None:
    """The reference's own opus gemm_ref loops (None when oracle/_ref was not built)."""
    global _OPUS
    if _OPUS is None:
        path = os.path.join(HERE, "_ref", "libopus_ref.so")
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        ci = C.c_int
        R.ref_opus_blockscale.argtypes = [u8p, u8p, f32p, f32p, f32p] + [ci] * 11
        R.ref_opus_blockscale_1x128x1.argtypes = [u8p, u8p, f32p, f32p, f32p] + [ci] * 11
        R.ref_opus_fp8_gemm.argtypes = [u8p, u8p, f32p] + [ci] * 6
        R.ref_opus_flatmm.argtypes = [u8p, u8p, f32p] + [ci] * 6
        R.ref_opus_e4m3_to_f32.argtypes = [C.c_uint8]; R.ref_opus_e4m3_to_f32.restype = C.c_float
        _OPUS = R
    return _OPUS


# --------------------------------------------------------------------------- formats
def e4m3_table() -> np.ndarray:
    L = lib()
    return np.array([L.orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)


_E4M3 = None


def e4m3_decode(q: np.ndarray) -> np.ndarray:
    global _E4M3
    if _E4M3 is None:
        _E4M3 = e4m3_table()
    return _E4M3[q]


def e8m0_decode(e: np.ndarray) -> np.ndarray:
    e = np.asarray(e, dtype=np.uint32)
    bits = np.where(e == 0, 0x00400000, np.where(e == 0xFF, 0x7F800001, e << 23)).astype(np.uint32)
    return bits.view(np.float32)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.array([L.orc_f32_to_bf16(float(v)) for v in flat], dtype=np.uint16).reshape(np.shape(x))


# --------------------------------------------------------------------------- data
def normal_rows(seed: int, row0: int, nrows: int, cols: int) -> np.ndarray:
    out = np.empty((nrows, cols), dtype=np.float32)
    lib().orc_normal_rows(seed, row0, nrows, cols, out)
    return out


def quant_mx(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    q = np.empty((rows, K), dtype=np.uint8)
    sf = np.empty((rows, (K + 31) // 32), dtype=np.uint8)
    lib().orc_quant_mx(x, rows, K, q, sf)
    return q, sf


def quant_1x128(x: np.ndarray):
    """-> q [rows, K] E4M3, sf [K/128, rows] fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    q = np.empty((rows, K), dtype=np.uint8)
    sf = np.empty((K // 128, rows), dtype=np.float32)
    lib().orc_quant_1x128(x, rows, K, q, sf)
    return q, sf


def quant_128x128(x: np.ndarray):
    """-> q [N, K] E4M3, sf [N/128, K/128] fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    N, K = x.shape
    q = np.empty((N, K), dtype=np.uint8)
    sf = np.empty((N // 128, K // 128), dtype=np.float32)
    lib().orc_quant_128x128(x, N, K, q, sf)
    return q, sf


# --------------------------------------------------------------------------- GEMMs
def gemm_blockscale(a, b, sfa, sfb, m, n, k, stride_sfa, stride_sfb, group_n, sfb_kmajor):
    """Reference gemm_ref of block_scale_gemm (sfb_kmajor=0) or 1x128x1 (=1); fp32 C."""
    c = np.empty((m, n), dtype=np.float32)
    fn = lib().orc_gemm_blockscale_1x128x1 if sfb_kmajor else lib().orc_gemm_blockscale
    fn(np.ascontiguousarray(a), np.ascontiguousarray(b), np.ascontiguousarray(sfa, dtype=np.float32),
       np.ascontiguousarray(sfb, dtype=np.float32), c, m, n, k, k, k, n, stride_sfa, stride_sfb, 1, group_n, 128)
    return c


def gemm_blockscale_f64(a, b, sfa, sfb, m, n, k, stride_sfa, stride_sfb, group_n, sfb_kmajor):
    c = np.empty((m, n), dtype=np.float64)
    lib().orc_gemm_blockscale_f64(np.ascontiguousarray(a), np.ascontiguousarray(b),
                                  np.ascontiguousarray(sfa, dtype=np.float32),
                                  np.ascontiguousarray(sfb, dtype=np.float32), c, m, n, k, k, k, n,
                                  stride_sfa, stride_sfb, 1, group_n, 128, int(sfb_kmajor))
    return c


def gemm_a8w8(a, b, m, n, k):
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_gemm_a8w8(np.ascontiguousarray(a), np.ascontiguousarray(b), c, m, n, k, k, k, n)
    return c


def gemm_a8w8_kn(a, b_kn, m, n, k):
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_gemm_a8w8_kn(np.ascontiguousarray(a), np.ascontiguousarray(b_kn), c, m, n, k, k, n, n)
    return c


def gemm_mx(a, b, sfa, sfb, m, n, k, alpha=1.0, acc_f64=True):
    d = np.empty((m, n), dtype=np.float32)
    lib().orc_gemm_mx(np.ascontiguousarray(a), np.ascontiguousarray(b), np.ascontiguousarray(sfa),
                      np.ascontiguousarray(sfb), m, n, k, a.shape[1], b.shape[1], sfa.shape[1], sfb.shape[1],
                      float(alpha), int(acc_f64), d, n)
    return d


def gemm_mxfp4(a, b, sfa, sfb, m, n, k, alpha=1.0, acc_f64=True):
    """MXFP4 reference GEMM (asm_f4gemm/f4gemm_ref.hpp:181-222) on packed e2m1
    operands [rows][K/2 bytes] with UE8M0 scales [rows][>= K/32]."""
    d = np.empty((m, n), dtype=np.float32)
    lib().orc_gemm_mxfp4(np.ascontiguousarray(a), np.ascontiguousarray(b), np.ascontiguousarray(sfa),
                         np.ascontiguousarray(sfb), m, n, k, a.shape[1], b.shape[1], sfa.shape[1], sfb.shape[1],
                         float(alpha), int(acc_f64), d, n)
    return d


E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
                dtype=np.float32)


def quant_mxfp4(x: np.ndarray):
    """fp32 [rows, K] -> (packed e2m1 [rows, K/2], UE8M0 scales [rows, K/32]); the MX
    scale rule with e2m1's max 6, round to nearest even onto the e2m1 grid."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    q = np.empty((rows, K // 2), dtype=np.uint8)
    sf = np.empty((rows, K // 32), dtype=np.uint8)
    lib().orc_quant_mxfp4(x, rows, K, q, sf)
    return q, sf


def e2m1_decode(packed: np.ndarray) -> np.ndarray:
    """Packed e2m1 bytes [rows][K/2] -> fp32 [rows][K], element 2i from the low nibble."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.float32)
    out[..., 0::2] = E2M1[p & 15]
    out[..., 1::2] = E2M1[p >> 4]
    return out


def fp4_operand(rows: int, K: int, seed: int):
    """Random MXFP4 operand with the reference's data recipe (make_operand,
    f4gemm_ref.hpp:150-177): uniform nibbles 0..15 and UE8M0 exponents 124..130
    (2^-3 .. 2^3); numpy's generator stands in for std::mt19937.  Returns
    (packed [rows][K/2] uint8, scales [rows][K/32] uint8)."""
    rs = np.random.RandomState(seed)
    packed = rs.randint(0, 256, size=(rows, K // 2)).astype(np.uint8)
    scales = rs.randint(124, 131, size=(rows, K // 32)).astype(np.uint8)
    return packed, scales


def encode_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> OCP E4M3 bytes, round to nearest even, saturating (the reference
    hosts' static_cast<host_fp8_t>(float))."""
    L = lib()
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.array([L.orc_f32_to_e4m3(float(v)) for v in flat], dtype=np.uint8).reshape(np.shape(x))


def opus_case(loop: str, recipe: str, M: int, N: int, K: int, seed: int) -> dict:
    """Seeded operands for one of the reference's opus gemm_ref loops.

    loop: "blockscale" (GROUP_N=128, SFB [N/128, K/128]), "blockscale_1x128x1"
    (GROUP_N=1, SFB [K/128, N]), "fp8_gemm" (no scales, B [N, K]) or "flatmm"
    (no scales, B [K, N]).  recipe:
      "uniform" -- the reference hosts' own data: A = E4M3(U[0,1)), B = E4M3(U[-.5,.5)),
                   fp32 scales U[.8,1.2) (block_scale_gemm/..._host.cc:206-209,
                   fp8_gemm/gemm_a8w8_8wave.cc:698-699); numpy's seeded generator
                   stands in for their unseeded std::mt19937;
      "normal"  -- N(0,1) rows quantised with the 1x128 / 128x128 (or per-column)
                   amax/448 recipe the benchmarks use (block-scale loops only);
      "bytes"   -- every finite E4M3 byte (0x00-0x7E with either sign: subnormals,
                   the largest value 448, negative zero) and scales over [2^-8, 2^8).
    Returns the operands and the loop's integer arguments."""
    rs = np.random.RandomState(seed)
    G = K // 128
    scaled = loop.startswith("blockscale")
    gn = 1 if loop == "blockscale_1x128x1" else 128
    b_rows, b_cols = (K, N) if loop == "flatmm" else (N, K)
    out = {"loop": loop, "M": M, "N": N, "K": K, "group_n": gn}
    if recipe == "uniform":
        a = encode_e4m3(rs.uniform(0.0, 1.0, (M, K)).astype(np.float32))
        b = encode_e4m3(rs.uniform(-0.5, 0.5, (b_rows, b_cols)).astype(np.float32))
        sfa = rs.uniform(0.8, 1.2, (G, M)).astype(np.float32)
        sfb = rs.uniform(0.8, 1.2, (N // 128, G) if gn == 128 else (G, N)).astype(np.float32)
    elif recipe == "normal":
        if not scaled:
            raise ValueError("the normal recipe is for the block-scale loops")
        a, sfa = quant_1x128(normal_rows(seed, 0, M, K))
        w = normal_rows(seed + 1, 0, N, K)
        if gn == 128:
            b, sfb = quant_128x128(w)
        else:  # per-column weight scales: a 1x128 quantiser over B's rows, [K/128, N]
            b, sfb = quant_1x128(w)
    elif recipe == "bytes":
        mag = rs.randint(0, 0x7F, (M, K)).astype(np.uint8)
        a = mag | (rs.randint(0, 2, (M, K)) * 0x80).astype(np.uint8)
        mag = rs.randint(0, 0x7F, (b_rows, b_cols)).astype(np.uint8)
        b = mag | (rs.randint(0, 2, (b_rows, b_cols)) * 0x80).astype(np.uint8)
        sfa = np.exp2(rs.uniform(-8, 8, (G, M))).astype(np.float32)
        sfb = np.exp2(rs.uniform(-8, 8, (N // 128, G) if gn == 128 else (G, N))).astype(np.float32)
    else:
        raise ValueError(recipe)
    out["a"], out["b"] = np.ascontiguousarray(a), np.ascontiguousarray(b)
    if scaled:
        out["sfa"], out["sfb"] = np.ascontiguousarray(sfa), np.ascontiguousarray(sfb)
        out["stride_sfa"] = M
        out["stride_sfb"] = G if gn == 128 else N
    return out


def run_opus_case(case: dict, which: str = "oracle") -> np.ndarray:
    """Run the oracle's restated loop (which="oracle") or the reference's own
    compiled gemm_ref (which="reference") on an opus_case; fp32 C [M, N]."""
    M, N, K, loop = case["M"], case["N"], case["K"], case["loop"]
    c = np.empty((M, N), dtype=np.float32)
    if which == "oracle":
        L = lib()
        fns = {"blockscale": L.orc_gemm_blockscale, "blockscale_1x128x1": L.orc_gemm_blockscale_1x128x1,
               "fp8_gemm": L.orc_gemm_a8w8, "flatmm": L.orc_gemm_a8w8_kn}
    else:
        R = opus_ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref/libopus_ref.so is not built")
        fns = {"blockscale": R.ref_opus_blockscale, "blockscale_1x128x1": R.ref_opus_blockscale_1x128x1,
               "fp8_gemm": R.ref_opus_fp8_gemm, "flatmm": R.ref_opus_flatmm}
    fn = fns[loop]
    if loop.startswith("blockscale"):
        fn(case["a"], case["b"], case["sfa"], case["sfb"], c, M, N, K, K, K, N, case["stride_sfa"],
           case["stride_sfb"], 1, case["group_n"], 128)
    elif loop == "fp8_gemm":
        fn(case["a"], case["b"], c, M, N, K, K, K, N)
    else:
        fn(case["a"], case["b"], c, M, N, K, K, N, N)
    return c


# --------------------------------------------------------------------------- layouts
def shuffle_weight_16x16(src: np.ndarray, N: int, Kp: int) -> np.ndarray:
    dst = np.empty(N * Kp, dtype=np.uint8)
    lib().orc_shuffle_weight_16x16(np.ascontiguousarray(src, dtype=np.uint8).ravel(), dst, N, Kp)
    return dst


def shuffle_scale(src: np.ndarray, rows: int, cols: int, sm: int, sn: int) -> np.ndarray:
    dst = np.empty(sm * sn, dtype=np.uint8)
    lib().orc_shuffle_scale(np.ascontiguousarray(src, dtype=np.uint8).ravel(), rows, cols, sm, sn, dst)
    return dst


def flatmm_shuffle_b(b_kn: np.ndarray, N: int, K: int) -> np.ndarray:
    out = np.empty(N * K, dtype=np.uint8)
    lib().orc_flatmm_shuffle_b(np.ascontiguousarray(b_kn, dtype=np.uint8).ravel(), out, N, K)
    return out


def sf_to_tc_layout(sf: np.ndarray) -> np.ndarray:
    rows, cols = sf.shape
    out = np.empty(((rows + 127) // 128) * ((cols + 3) // 4) * 512, dtype=np.uint8)
    lib().orc_sf_to_tc_layout(np.ascontiguousarray(sf, dtype=np.uint8), rows, cols, out)
    return out


def round_up(a: int, b: int) -> int:
    return (a + b - 1) // b * b


def max_threads() -> int:
    return lib().orc_max_threads()


# --------------------------------------------------------------------------- tolerances
def check_bf16(got_f32: np.ndarray, ref: np.ndarray) -> float:
    """Acceptance for bf16 C: max|err| <= 2^-7 * max_n |ref[m, n]| per row.
    Returns the worst ratio err / bound (pass when <= 1)."""
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(np.asarray(got_f32, dtype=np.float64) - ref)
    bound = np.maximum(np.abs(ref).max(axis=1, keepdims=True), 1e-30) * 2.0 ** -7
    return float((err / bound).max()) if err.size else 0.0


def check_f32(got: np.ndarray, ref: np.ndarray) -> float:
    """Acceptance for fp32 C: |err| / max(|ref|, 2^-7 * rowmax) <= 1e-3.
    Returns the worst relative error."""
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(np.asarray(got, dtype=np.float64) - ref)
    floor = np.maximum(np.abs(ref).max(axis=1, keepdims=True), 1e-30) * 2.0 ** -7
    den = np.maximum(np.abs(ref), floor)
    return float((err / den).max()) if err.size else 0.0
