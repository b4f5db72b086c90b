"""b2g_gemm_mxfp8_noalloc: the MXFP8 GEMM for callers that cannot allocate device
memory (a host whose device memory all belongs to its own pool allocator).  Its
split-K partials live in the library's fixed file-scope scratch array instead of
a cudaMalloc'd workspace.

Called through the C ABI twice in a row, with different inputs, and each result
compared with the allocating entry point b2g_gemm_mxfp8 on the same inputs,
within the bf16 tolerance the parity tests use (max|err| <= 2^-7 * row max).
Self-contained so it passes alone in a fresh process as well as after the rest
of the suite (this file is collected last on purpose).
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _bf16_ratio(got: torch.Tensor, ref: torch.Tensor) -> float:
    g = got.double().cpu().numpy()
    r = ref.double().cpu().numpy()
    bound = np.maximum(np.abs(r).max(axis=1, keepdims=True), 1e-30) * 2.0 ** -7
    return float((np.abs(g - r) / bound).max())


def _operands(seed, M, N, K, dev):
    from gcnasm_b200 import ops

    x = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(seed))
    w = torch.randn(N, K, device=dev, generator=torch.Generator(device=dev).manual_seed(seed + 1000))
    qa, sfa = ops.quant_mxfp8(x, "tc")
    qb, sfb = ops.quant_mxfp8(w, "tc")
    return qa, sfa, qb, sfb


def test_noalloc_matches_allocating_entry_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gcnasm_b200 import build, capi, ops

    build.build()
    L = capi.lib()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    M, N, K, log2 = 64, 1024, 4096, 2  # 4-way split-K, bf16 out: partials in the fixed scratch
    for seed in (101, 202):
        qa, sfa, qb, sfb = _operands(seed, M, N, K, dev)
        ref = ops.mxfp8_gemm(qa, qb, sfa, sfb, out_dtype=torch.bfloat16, log2_k_split=log2)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        args = capi.Mxfp8Args(qa.data_ptr(), qb.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr(),
                              M, N, K, K, K, N, 1.0, 0, capi.OUT_BF16, log2)
        rc = L.b2g_gemm_mxfp8_noalloc(C.byref(args), C.c_void_p(stream.cuda_stream))
        assert rc == capi.B2G_OK, L.b2g_last_error()
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        assert _bf16_ratio(out, ref) <= 1.0

    # a split whose partials exceed the fixed scratch is refused before any work
    big = capi.Mxfp8Args(qa.data_ptr(), qb.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), out.data_ptr(),
                         8192, 8192, 8192, 8192, 8192, 8192, 1.0, 0, capi.OUT_BF16, 3)
    assert L.b2g_gemm_mxfp8_noalloc(C.byref(big), C.c_void_p(stream.cuda_stream)) == capi.B2G_ERR_WORKSPACE
    assert b"scratch" in L.b2g_last_error()
