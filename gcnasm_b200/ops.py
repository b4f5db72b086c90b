"""torch-tensor front end over the C ABI.

PyTorch supplies device memory and streams here; every computation runs in
``libb2g.so``.  Tensors holding E4M3 / UE8M0 bytes are ``torch.uint8`` so that
no torch fp8 semantics are involved.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import capi


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> C.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _out_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return capi.OUT_BF16
    if dtype == torch.float32:
        return capi.OUT_F32
    raise ValueError(f"unsupported output dtype {dtype}")


def sf_tc_bytes(rows: int, k: int) -> int:
    return int(capi.lib().b2g_sf_tc_bytes(rows, k))


def _x_code(x: torch.Tensor) -> int:
    if x.dtype == torch.float32:
        return capi.OUT_F32
    if x.dtype == torch.bfloat16:
        return capi.OUT_BF16
    raise ValueError(f"quantiser input must be fp32 or bf16, not {x.dtype}")


def quant_mxfp8(x: torch.Tensor, sf_layout: str = "tc", stream=None):
    """fp32 or bf16 [rows, K] -> (q uint8 [rows, K] E4M3, scales uint8) with scales in
    the tensor-core atom layout ("tc", flat) or row-major [rows, K/32] ("rowmajor")."""
    assert x.is_cuda and x.dim() == 2
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.uint8, device=x.device)
    sf_tc = torch.empty(sf_tc_bytes(rows, k), dtype=torch.uint8, device=x.device) if sf_layout == "tc" else None
    sf_rm = torch.empty((rows, k // 32), dtype=torch.uint8, device=x.device) if sf_layout == "rowmajor" else None
    capi.check(capi.lib().b2g_quant_mxfp8_ex(x.data_ptr(), _x_code(x), rows, k, x.stride(0), q.data_ptr(),
                                             q.stride(0), _ptr(sf_tc), _ptr(sf_rm), _stream(stream)),
               "b2g_quant_mxfp8_ex")
    return q, (sf_tc if sf_layout == "tc" else sf_rm)


def quant_mxfp4(x: torch.Tensor, sf_layout: str = "tc", stream=None):
    """fp32 or bf16 [rows, K] -> (packed E2M1 uint8 [rows, K/2], scales uint8) with
    scales as in quant_mxfp8 (b2g_quant_mxfp4: s = 2^ceil(log2(amax/6)) per 1x32)."""
    assert x.is_cuda and x.dim() == 2
    rows, k = x.shape
    q = torch.empty((rows, k // 2), dtype=torch.uint8, device=x.device)
    sf_tc = torch.empty(sf_tc_bytes(rows, k), dtype=torch.uint8, device=x.device) if sf_layout == "tc" else None
    sf_rm = torch.empty((rows, k // 32), dtype=torch.uint8, device=x.device) if sf_layout == "rowmajor" else None
    capi.check(capi.lib().b2g_quant_mxfp4(x.data_ptr(), _x_code(x), rows, k, x.stride(0), q.data_ptr(),
                                          q.stride(0), _ptr(sf_tc), _ptr(sf_rm), _stream(stream)),
               "b2g_quant_mxfp4")
    return q, (sf_tc if sf_layout == "tc" else sf_rm)


def quant_1x128(x: torch.Tensor, stream=None):
    """fp32 or bf16 [rows, K] -> (E4M3 q, fp32 scales [K/128, rows], amax/448 per 1x128)."""
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.uint8, device=x.device)
    sf = torch.empty((k // 128, rows), dtype=torch.float32, device=x.device)
    capi.check(capi.lib().b2g_quant_1x128_ex(x.data_ptr(), _x_code(x), rows, k, q.data_ptr(), sf.data_ptr(),
                                             _stream(stream)), "b2g_quant_1x128_ex")
    return q, sf


def quant_128x128(x: torch.Tensor, stream=None):
    n, k = x.shape
    q = torch.empty((n, k), dtype=torch.uint8, device=x.device)
    sf = torch.empty((n // 128, k // 128), dtype=torch.float32, device=x.device)
    capi.check(capi.lib().b2g_quant_128x128(x.data_ptr(), n, k, q.data_ptr(), sf.data_ptr(), _stream(stream)),
               "b2g_quant_128x128")
    return q, sf


def sf_rowmajor_to_tc(sf: torch.Tensor, k: int, stream=None) -> torch.Tensor:
    rows, cols = sf.shape
    out = torch.empty(sf_tc_bytes(rows, k), dtype=torch.uint8, device=sf.device)
    capi.check(capi.lib().b2g_sf_rowmajor_to_tc(sf.data_ptr(), rows, cols, sf.stride(0), out.data_ptr(),
                                                _stream(stream)), "b2g_sf_rowmajor_to_tc")
    return out


def sf_f4gemm_to_tc(sf_shuffled: torch.Tensor, rows: int, k: int, sn: int, stream=None) -> torch.Tensor:
    out = torch.empty(sf_tc_bytes(rows, k), dtype=torch.uint8, device=sf_shuffled.device)
    capi.check(capi.lib().b2g_sf_f4gemm_to_tc(sf_shuffled.data_ptr(), rows, k // 32, sn, out.data_ptr(),
                                              _stream(stream)), "b2g_sf_f4gemm_to_tc")
    return out


def shuffle_scale(sf: torch.Tensor, sm: int, sn: int, stream=None) -> torch.Tensor:
    rows, cols = sf.shape
    out = torch.empty(sm * sn, dtype=torch.uint8, device=sf.device)
    capi.check(capi.lib().b2g_shuffle_scale(sf.data_ptr(), rows, cols, sm, sn, out.data_ptr(), _stream(stream)),
               "b2g_shuffle_scale")
    return out


def shuffle_weight_16x16(w: torch.Tensor, stream=None) -> torch.Tensor:
    n, kp = w.shape
    out = torch.empty_like(w)
    capi.check(capi.lib().b2g_shuffle_weight_16x16(w.data_ptr(), out.data_ptr(), n, kp, _stream(stream)),
               "b2g_shuffle_weight_16x16")
    return out


def unshuffle_weight_16x16(w: torch.Tensor, stream=None) -> torch.Tensor:
    n, kp = w.shape
    out = torch.empty_like(w)
    capi.check(capi.lib().b2g_unshuffle_weight_16x16(w.data_ptr(), out.data_ptr(), n, kp, _stream(stream)),
               "b2g_unshuffle_weight_16x16")
    return out


def mxfp8_gemm(a: torch.Tensor, b: torch.Tensor, sfa_tc: torch.Tensor, sfb_tc: torch.Tensor,
               out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0,
               b_preshuffled: bool = False, log2_k_split: int = 0, stream=None, c: torch.Tensor | None = None,
               beta: float = 0.0, bias: torch.Tensor | None = None) -> torch.Tensor:
    """D[M, N] = alpha * A[M, K] . B[N, K]^T (+ beta * c + bias[n]), MXFP8 operands with
    tensor-core-layout scales."""
    m, k = a.shape
    n = b.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    args = capi.Mxfp8Args(a.data_ptr(), b.data_ptr(), sfa_tc.data_ptr(), sfb_tc.data_ptr(), out.data_ptr(),
                          m, n, k, a.stride(0), k if b_preshuffled else b.stride(0), out.stride(0), alpha,
                          int(b_preshuffled), _out_code(out.dtype), log2_k_split)
    epi = _epilogue(c, beta, bias, out)
    if epi is None:
        capi.check(capi.lib().b2g_gemm_mxfp8(C.byref(args), _stream(stream)), "b2g_gemm_mxfp8")
    else:
        capi.check(capi.lib().b2g_gemm_mxfp8_ex(C.byref(args), C.byref(epi), _stream(stream)), "b2g_gemm_mxfp8_ex")
    return out


def _epilogue(c, beta, bias, out):
    """b2g_epilogue for D = alpha * A . B^T + beta * c + bias[n], or None without terms.
    c and bias must have the output's dtype (c [M, >= N] rows, bias [N])."""
    if c is None and bias is None:
        return None
    for t, name in ((c, "c"), (bias, "bias")):
        if t is not None and t.dtype != out.dtype:
            raise ValueError(f"{name} must have the output dtype {out.dtype}")
    return capi.Epilogue(c.data_ptr() if c is not None else None, c.stride(0) if c is not None else 0,
                         float(beta), bias.data_ptr() if bias is not None else None)


def mxfp4_gemm(a: torch.Tensor, b: torch.Tensor, sfa_tc: torch.Tensor, sfb_tc: torch.Tensor,
               out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0,
               b_preshuffled: bool = False, log2_k_split: int = 0, stream=None, c: torch.Tensor | None = None,
               beta: float = 0.0, bias: torch.Tensor | None = None) -> torch.Tensor:
    """D[M, N] = alpha * A . B^T with MXFP4 operands (b2g_gemm_mxfp4): a [M, K/2] and
    b [N, K/2] uint8 of packed E2M1 (element 2i in the low nibble), scales in the
    tensor-core atom layout for K elements."""
    m, kh = a.shape
    n = b.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    args = capi.Mxfp8Args(a.data_ptr(), b.data_ptr(), sfa_tc.data_ptr(), sfb_tc.data_ptr(), out.data_ptr(),
                          m, n, 2 * kh, 2 * a.stride(0), 2 * kh if b_preshuffled else 2 * b.stride(0),
                          out.stride(0), alpha, int(b_preshuffled), _out_code(out.dtype), log2_k_split)
    epi = _epilogue(c, beta, bias, out)
    if epi is None:
        capi.check(capi.lib().b2g_gemm_mxfp4(C.byref(args), _stream(stream)), "b2g_gemm_mxfp4")
    else:
        capi.check(capi.lib().b2g_gemm_mxfp4_ex(C.byref(args), C.byref(epi), _stream(stream)), "b2g_gemm_mxfp4_ex")
    return out


def set_static_weights(on: bool) -> None:
    """b2g_set_static_weights: let decode GEMMs (M <= 128) read B and its scales
    before the preceding kernel on the stream completes (weights no kernel writes)."""
    capi.check(capi.lib().b2g_set_static_weights(int(bool(on))), "b2g_set_static_weights")


def mxfp8_gemm_peer_out(a: torch.Tensor, b: torch.Tensor, sfa_tc: torch.Tensor, sfb_tc: torch.Tensor,
                        c_full: torch.Tensor, peer_ptrs, self_index: int, col_offset: int, alpha: float = 1.0,
                        b_preshuffled: bool = False, stream=None) -> None:
    """This GPU's columns [col_offset, col_offset + N) of C = alpha * A . B^T (B: [N, K],
    this GPU's column slab) stored straight into every GPU's full-width C
    (b2g_gemm_mxfp8_peer_out).  c_full is this GPU's [M, ldd] buffer (bf16 or fp32);
    peer_ptrs[i] the base address of GPU i's buffer as mapped in this process."""
    m, k = a.shape
    n = b.shape[0]
    args = capi.Mxfp8Args(a.data_ptr(), b.data_ptr(), sfa_tc.data_ptr(), sfb_tc.data_ptr(), 0,
                          m, n, k, a.stride(0), k if b_preshuffled else b.stride(0), 0, alpha,
                          int(b_preshuffled), _out_code(c_full.dtype), 0)
    ptrs = (C.c_void_p * len(peer_ptrs))(*[C.c_void_p(int(x)) for x in peer_ptrs])
    capi.check(capi.lib().b2g_gemm_mxfp8_peer_out(C.byref(args), ptrs, len(peer_ptrs), self_index,
                                                  c_full.stride(0), col_offset, _stream(stream)),
               "b2g_gemm_mxfp8_peer_out")


def mxfp8_gemm_a2a_out(a: torch.Tensor, b: torch.Tensor, sfa_tc: torch.Tensor, sfb_tc: torch.Tensor,
                       window: torch.Tensor, peer_ptrs, self_index: int, alpha: float = 1.0,
                       b_preshuffled: bool = False, stream=None) -> None:
    """C = alpha * A . B^T for this GPU's M rows and all N columns, column shard q stored
    into peer q's window rows [self_index * M, (self_index + 1) * M) (b2g_gemm_mxfp8_a2a_out).
    window is this GPU's [n_peers * M, N / n_peers] buffer (its dtype is the output type);
    peer_ptrs[i] the base address of GPU i's window as mapped in this process."""
    m, k = a.shape
    n = b.shape[0]
    args = capi.Mxfp8Args(a.data_ptr(), b.data_ptr(), sfa_tc.data_ptr(), sfb_tc.data_ptr(), 0,
                          m, n, k, a.stride(0), k if b_preshuffled else b.stride(0), 0, alpha,
                          int(b_preshuffled), _out_code(window.dtype), 0)
    ptrs = (C.c_void_p * len(peer_ptrs))(*[C.c_void_p(int(x)) for x in peer_ptrs])
    capi.check(capi.lib().b2g_gemm_mxfp8_a2a_out(C.byref(args), ptrs, len(peer_ptrs), self_index, _stream(stream)),
               "b2g_gemm_mxfp8_a2a_out")


def opus_kargs(a, b, c, sfa=None, sfb=None, stride_sfa=0, stride_sfb=0, batch=1,
               stride_sfa_batch=0, stride_sfb_batch=0) -> capi.OpusGemmKargs:
    """Fill opus_gemm_kargs the way the reference hosts do
    (opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_host.cc:228-247)."""
    k = capi.OpusGemmKargs()
    m, kk = a.shape[-2], a.shape[-1]
    n = b.shape[-2]
    k.ptr_a, k.ptr_b, k.ptr_c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    k.m, k.n, k.k, k.batch = m, n, kk, batch
    k.stride_a, k.stride_b, k.stride_c = a.stride(-2), b.stride(-2), c.stride(-2)
    k.stride_a_batch = a.stride(0) if a.dim() == 3 else m * kk
    k.stride_b_batch = b.stride(0) if b.dim() == 3 else n * kk
    k.stride_c_batch = c.stride(0) if c.dim() == 3 else m * n
    k.ptr_sfa = _ptr(sfa) or 0
    k.ptr_sfb = _ptr(sfb) or 0
    k.stride_sfa, k.stride_sfb = stride_sfa, stride_sfb
    k.stride_sfa_batch, k.stride_sfb_batch = stride_sfa_batch, stride_sfb_batch
    return k


def gemm_a8w8_blockscale(a, b, sfa, sfb, group_n: int = 128, out_dtype=torch.float32, log2_k_split: int = 0,
                         out=None, stream=None) -> torch.Tensor:
    """opus block_scale_gemm (group_n=128: SFB [N/128, K/128]) or
    block_scale_1x128x1_gemm (group_n=1: SFB [K/128, N]); SFA [K/128, M]."""
    m, kk = a.shape
    n = b.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    stride_sfb = (kk // 128) if group_n == 128 else sfb.stride(0)
    ka = opus_kargs(a, b, out, sfa, sfb, stride_sfa=sfa.stride(0), stride_sfb=stride_sfb)
    capi.check(capi.lib().b2g_gemm_a8w8_blockscale(C.byref(ka), group_n, _out_code(out.dtype), log2_k_split,
                                                   _stream(stream)), "b2g_gemm_a8w8_blockscale")
    return out


def gemm_a8w8(a, b, alpha: float = 1.0, out_dtype=torch.float32, log2_k_split: int = 0, b_preshuffled=False,
              out=None, stream=None) -> torch.Tensor:
    m, kk = a.shape[-2], a.shape[-1]
    n = b.shape[-2] if not b_preshuffled else b.numel() // kk
    batch = a.shape[0] if a.dim() == 3 else 1
    if out is None:
        out = torch.empty((batch, m, n) if a.dim() == 3 else (m, n), dtype=out_dtype, device=a.device)
    full = opus_kargs(a, b if not b_preshuffled else b.view(-1, n, kk), out, batch=batch)
    ka = capi.OpusGemmKargsA8W8()
    C.memmove(C.byref(ka), C.byref(full), C.sizeof(ka))
    fn = capi.lib().b2g_gemm_a8w8_preshuffled if b_preshuffled else capi.lib().b2g_gemm_a8w8
    capi.check(fn(C.byref(ka), alpha, _out_code(out.dtype), log2_k_split, _stream(stream)), "b2g_gemm_a8w8")
    return out


def device_status(clear: bool = True) -> int:
    st = C.c_int(0)
    capi.lib().b2g_device_status(C.byref(st), int(clear))
    return st.value
