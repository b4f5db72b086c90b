"""ctypes binding of the C ABI in ``include/b2g/gemm.h`` (``_lib/libb2g.so``).

The structures mirror the reference's host argument blocks byte for byte:

* :class:`OpusGemmKargs` -- ``opus_gemm_kargs``
  (opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_common.h:4-25);
* :class:`OpusGemmKargsA8W8` -- the fp8_gemm prefix (opus_gemm/fp8_gemm/gemm_a8w8_8wave.cc:99-113);
* :class:`F4gemmKernelArgs` -- the packed 0x174-byte f4gemm kernarg block
  (asm_f4gemm/f4gemm.hpp:64-115).

There is no fallback: if the shared object is missing the import of any entry
point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libb2g.so")

B2G_OK = 0
B2G_ERR_INVALID_ARG = 1
B2G_ERR_UNSUPPORTED = 2
B2G_ERR_ALIGNMENT = 3
B2G_ERR_CUDA = 4
B2G_ERR_DEVICE_TIMEOUT = 5
B2G_ERR_NO_DEVICE = 6
B2G_ERR_WORKSPACE = 7
OUT_BF16 = 0
OUT_F32 = 1

# every symbol include/b2g/gemm.h declares
EXPORTS = [
    "b2g_gemm_a8w8_blockscale", "b2g_gemm_a8w8", "b2g_gemm_a8w8_preshuffled", "b2g_gemm_mxfp8_f4gemm",
    "b2g_gemm_mxfp4_f4gemm", "b2g_gemm_mxfp8", "b2g_gemm_mxfp4", "b2g_gemm_mxfp8_ex", "b2g_gemm_mxfp4_ex", "b2g_gemm_mxfp8_peer_out", "b2g_gemm_mxfp8_a2a_out", "b2g_set_static_weights", "b2g_gemm_mxfp8_noalloc", "b2g_select", "b2g_manifest_size", "b2g_manifest_entry", "b2g_sf_tc_bytes",
    "b2g_sf_rowmajor_to_tc", "b2g_sf_f4gemm_to_tc", "b2g_shuffle_scale", "b2g_shuffle_weight_16x16",
    "b2g_unshuffle_weight_16x16", "b2g_quant_mxfp8", "b2g_quant_mxfp8_ex", "b2g_quant_mxfp4",
    "b2g_quant_1x128", "b2g_quant_1x128_ex", "b2g_quant_128x128",
    "b2g_device_status", "b2g_set_wait_timeout_ms", "b2g_debug_force_stall", "b2g_status_string",
    "b2g_last_error", "b2g_version",
]


class B2GError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = ""
        try:
            msg = lib().b2g_last_error().decode(errors="replace")
        except Exception:  # pragma: no cover
            pass
        super().__init__(f"{where}: status {status} ({status_string(status)}) {msg}")


class OpusGemmKargs(C.Structure):
    _fields_ = [
        ("ptr_a", C.c_void_p), ("ptr_b", C.c_void_p), ("ptr_c", C.c_void_p),
        ("m", C.c_int), ("n", C.c_int), ("k", C.c_int), ("batch", C.c_int),
        ("stride_a", C.c_int), ("stride_b", C.c_int), ("stride_c", C.c_int),
        ("stride_a_batch", C.c_int), ("stride_b_batch", C.c_int), ("stride_c_batch", C.c_int),
        ("ptr_sfa", C.c_void_p), ("ptr_sfb", C.c_void_p),
        ("stride_sfa", C.c_int), ("stride_sfb", C.c_int),
        ("stride_sfa_batch", C.c_int), ("stride_sfb_batch", C.c_int),
    ]


class OpusGemmKargsA8W8(C.Structure):
    _fields_ = OpusGemmKargs._fields_[:13]


def _slot(name, ctype, pad_words):
    return [(name, ctype), (f"_pad_{name}", C.c_uint * pad_words)]


class F4gemmKernelArgs(C.Structure):
    _pack_ = 1
    _fields_ = (
        _slot("ptr_D", C.c_void_p, 2) + _slot("ptr_C", C.c_void_p, 2) + _slot("ptr_A", C.c_void_p, 2)
        + _slot("ptr_B", C.c_void_p, 2) + _slot("alpha", C.c_float, 3) + _slot("beta", C.c_float, 3)
        + _slot("stride_D0", C.c_uint, 3) + _slot("stride_D1", C.c_uint, 3) + _slot("stride_C0", C.c_uint, 3)
        + _slot("stride_C1", C.c_uint, 3) + _slot("stride_A0", C.c_uint, 3) + _slot("stride_A1", C.c_uint, 3)
        + _slot("stride_B0", C.c_uint, 3) + _slot("stride_B1", C.c_uint, 3) + _slot("M", C.c_uint, 3)
        + _slot("N", C.c_uint, 3) + _slot("K", C.c_uint, 3) + _slot("ptr_ScaleA", C.c_void_p, 2)
        + _slot("ptr_ScaleB", C.c_void_p, 2) + _slot("stride_ScaleA0", C.c_uint, 3)
        + _slot("stride_ScaleA1", C.c_uint, 3) + _slot("stride_ScaleB0", C.c_uint, 3)
        + _slot("stride_ScaleB1", C.c_uint, 3) + [("log2_k_split", C.c_int)]
    )


assert C.sizeof(F4gemmKernelArgs) == 0x174


class Mxfp8Args(C.Structure):
    _fields_ = [
        ("a", C.c_void_p), ("b", C.c_void_p), ("sfa", C.c_void_p), ("sfb", C.c_void_p), ("d", C.c_void_p),
        ("m", C.c_int), ("n", C.c_int), ("k", C.c_int),
        ("lda", C.c_longlong), ("ldb", C.c_longlong), ("ldd", C.c_longlong),
        ("alpha", C.c_float), ("b_preshuffled", C.c_int), ("out_dtype", C.c_int), ("log2_k_split", C.c_int),
    ]


class Epilogue(C.Structure):
    """b2g_epilogue: D = alpha * A . B^T + beta * C + bias[n] (C, bias in D's type)."""
    _fields_ = [("c", C.c_void_p), ("ldc", C.c_longlong), ("beta", C.c_float), ("bias", C.c_void_p)]


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"gcnasm_b200: CUDA library {LIB_PATH} is not built; run "
                               "`python -m gcnasm_b200.build` (there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        vp, ci, ll = C.c_void_p, C.c_int, C.c_longlong
        L.b2g_gemm_a8w8_blockscale.argtypes = [C.POINTER(OpusGemmKargs), ci, ci, ci, vp]
        L.b2g_gemm_a8w8.argtypes = [C.POINTER(OpusGemmKargsA8W8), C.c_float, ci, ci, vp]
        L.b2g_gemm_a8w8_preshuffled.argtypes = [C.POINTER(OpusGemmKargsA8W8), C.c_float, ci, ci, vp]
        L.b2g_gemm_mxfp8_f4gemm.argtypes = [C.POINTER(F4gemmKernelArgs), ci, ci, vp]
        L.b2g_gemm_mxfp8.argtypes = [C.POINTER(Mxfp8Args), vp]
        L.b2g_gemm_mxfp4.argtypes = [C.POINTER(Mxfp8Args), vp]
        L.b2g_gemm_mxfp8_ex.argtypes = [C.POINTER(Mxfp8Args), C.POINTER(Epilogue), vp]
        L.b2g_gemm_mxfp4_ex.argtypes = [C.POINTER(Mxfp8Args), C.POINTER(Epilogue), vp]
        L.b2g_gemm_mxfp4_f4gemm.argtypes = [C.POINTER(F4gemmKernelArgs), ci, ci, vp]
        L.b2g_gemm_mxfp8_noalloc.argtypes = [C.POINTER(Mxfp8Args), vp]
        L.b2g_set_static_weights.argtypes = [ci]
        L.b2g_gemm_mxfp8_peer_out.argtypes = [C.POINTER(Mxfp8Args), C.POINTER(vp), ci, ci, ll, ll, vp]
        L.b2g_gemm_mxfp8_a2a_out.argtypes = [C.POINTER(Mxfp8Args), C.POINTER(vp), ci, ci, vp]
        pi = C.POINTER(ci)
        L.b2g_select.argtypes = [ci, ci, ci, ci, ci, ci, pi, pi, pi, pi]
        L.b2g_manifest_entry.argtypes = [ci, pi, pi, pi, pi, C.POINTER(C.c_char_p)]
        L.b2g_sf_tc_bytes.argtypes = [ci, ci]
        L.b2g_sf_tc_bytes.restype = ll
        L.b2g_sf_rowmajor_to_tc.argtypes = [vp, ci, ci, ll, vp, vp]
        L.b2g_sf_f4gemm_to_tc.argtypes = [vp, ci, ci, ci, vp, vp]
        L.b2g_shuffle_scale.argtypes = [vp, ci, ci, ci, ci, vp, vp]
        L.b2g_shuffle_weight_16x16.argtypes = [vp, vp, ci, ci, vp]
        L.b2g_unshuffle_weight_16x16.argtypes = [vp, vp, ci, ci, vp]
        L.b2g_quant_mxfp8.argtypes = [vp, ci, ci, ll, vp, ll, vp, vp, vp]
        L.b2g_quant_1x128.argtypes = [vp, ci, ci, vp, vp, vp]
        L.b2g_quant_mxfp8_ex.argtypes = [vp, ci, ci, ci, ll, vp, ll, vp, vp, vp]
        L.b2g_quant_mxfp4.argtypes = [vp, ci, ci, ci, ll, vp, ll, vp, vp, vp]
        L.b2g_quant_1x128_ex.argtypes = [vp, ci, ci, ci, vp, vp, vp]
        L.b2g_quant_128x128.argtypes = [vp, ci, ci, vp, vp, vp]
        L.b2g_device_status.argtypes = [pi, ci]
        L.b2g_set_wait_timeout_ms.argtypes = [ci]
        L.b2g_debug_force_stall.argtypes = [ci]
        L.b2g_status_string.argtypes = [ci]
        L.b2g_status_string.restype = C.c_char_p
        L.b2g_last_error.restype = C.c_char_p
        _LIB = L
    return _LIB


def status_string(s: int) -> str:
    return lib().b2g_status_string(s).decode()


def check(status: int, where: str) -> None:
    if status != B2G_OK:
        raise B2GError(status, where)
