"""b2g_gemm_mxfp8_noalloc: the MXFP8 GEMM for callers that cannot allocate device
memory -- a serving engine or framework that reserves the GPU's memory for its own
pool at start-up, where a library cudaMalloc either fails or takes memory the pool
cannot see.  Its scratch (the decode kernel's piece slots for M <= 128, split-K
partials for larger M) lives in the library's fixed file-scope device array.

Each case calls it through the C ABI twice in a row with different inputs (the
second call finds the first call's leftovers in the shared array) and checks each
result against the CPU oracle (f64-accumulate MX GEMM over the dequantised
operands) within the parity tests' tolerances -- bf16: max|err| <= 2^-7 * row max;
fp32: |err| / max(|ref|, 2^-7 * row max) <= 1e-3 -- and against the allocating
entry point b2g_gemm_mxfp8 on the same inputs.

Collected last on purpose (file name), and self-contained: it passes alone in a
fresh process as well as after the rest of the suite.
"""
import ctypes as C

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

BF16_TOL = 1.0
F32_TOL = 1e-3

# (M, N, K, log2_k_split, out): which part of the fixed array each case uses
CASES = [
    (64, 1024, 4096, 0, "bf16"),    # decode kernel (M <= 128): piece slots of its split tiles
    (128, 1024, 4096, 0, "f32"),    # decode kernel at MP = 128: the largest slot set
    (256, 1024, 2048, 2, "bf16"),   # 4-way split-K, bf16 out: fp32 partials, then the reduce
]


def _env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gcnasm_b200 import build, capi

    build.build()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    return capi, capi.lib(), dev


def _operands(O, seed, M, N, K):
    qa, sa = O.quant_mx(O.normal_rows(seed, 0, M, K))
    qb, sb = O.quant_mx(O.normal_rows(seed + 1000, 0, N, K))
    return qa, sa, qb, sb


def _check(O, got, ref, out):
    g = got.float().cpu().numpy()
    if out == "bf16":
        r = O.check_bf16(g, ref)
        assert r <= BF16_TOL, f"bf16 error ratio {r}"
    else:
        r = O.check_f32(g, ref)
        assert r <= F32_TOL, f"fp32 relative error {r}"


@pytest.mark.parametrize("M,N,K,log2,out", CASES)
def test_noalloc_matches_oracle_and_allocating_entry_two_calls(oracle, M, N, K, log2, out):
    capi, L, dev = _env()
    from gcnasm_b200 import ops

    O = oracle
    stream = torch.cuda.current_stream()
    tdt = torch.bfloat16 if out == "bf16" else torch.float32
    code = capi.OUT_BF16 if out == "bf16" else capi.OUT_F32
    for seed in (101, 202):
        qa, sa, qb, sb = _operands(O, seed, M, N, K)
        ref = O.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
        ta, tb = torch.from_numpy(qa).to(dev), torch.from_numpy(qb).to(dev)
        tsa = torch.from_numpy(O.sf_to_tc_layout(sa)).to(dev)
        tsb = torch.from_numpy(O.sf_to_tc_layout(sb)).to(dev)
        d = torch.full((M, N), float("nan"), dtype=tdt, device=dev)
        args = capi.Mxfp8Args(ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(), tsb.data_ptr(), d.data_ptr(),
                              M, N, K, K, K, N, 1.0, 0, code, log2)
        rc = L.b2g_gemm_mxfp8_noalloc(C.byref(args), C.c_void_p(stream.cuda_stream))
        assert rc == capi.B2G_OK, L.b2g_last_error()
        torch.cuda.synchronize()
        assert not torch.isnan(d.float()).any()
        _check(O, d, ref, out)
        alloc = ops.mxfp8_gemm(ta, tb, tsa, tsb, out_dtype=tdt, log2_k_split=log2)
        torch.cuda.synchronize()
        _check(O, alloc, ref, out)
        # both entry points run the same kernels in the same order: identical bits
        assert torch.equal(d, alloc)
    st = C.c_int(-1)
    assert L.b2g_device_status(C.byref(st), 0) == capi.B2G_OK and st.value == 0


def test_noalloc_refusal_and_timeout_visibility(oracle):
    """Scratch needs beyond the array are refused before any device work; a bounded
    wait that runs out inside a no-alloc call shows in b2g_device_status, which clears
    it, after which the next no-alloc call is correct again."""
    capi, L, dev = _env()
    O = oracle
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    M, N, K = 128, 256, 256  # the shape the allocating path's stall test uses (decode kernel)
    qa, sa, qb, sb = _operands(O, 7, M, N, K)
    ta, tb = torch.from_numpy(qa).to(dev), torch.from_numpy(qb).to(dev)
    tsa = torch.from_numpy(O.sf_to_tc_layout(sa)).to(dev)
    tsb = torch.from_numpy(O.sf_to_tc_layout(sb)).to(dev)
    d = torch.empty((M, N), dtype=torch.float32, device=dev)

    # 8-way split of an 8192^3 bf16 GEMM: 2 GiB of partials.  Only the host checks
    # run (the pointers are never dereferenced).
    big = capi.Mxfp8Args(ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(), tsb.data_ptr(), d.data_ptr(),
                         8192, 8192, 8192, 8192, 8192, 8192, 1.0, 0, capi.OUT_BF16, 3)
    assert L.b2g_gemm_mxfp8_noalloc(C.byref(big), stream) == capi.B2G_ERR_WORKSPACE
    assert b"fixed scratch array" in L.b2g_last_error()

    args = capi.Mxfp8Args(ta.data_ptr(), tb.data_ptr(), tsa.data_ptr(), tsb.data_ptr(), d.data_ptr(),
                          M, N, K, K, K, N, 1.0, 0, capi.OUT_F32, 0)
    st = C.c_int(0)
    assert L.b2g_device_status(C.byref(st), 1) == capi.B2G_OK
    L.b2g_set_wait_timeout_ms(200)
    L.b2g_debug_force_stall(1)
    try:
        assert L.b2g_gemm_mxfp8_noalloc(C.byref(args), stream) == capi.B2G_OK
        rc = L.b2g_device_status(C.byref(st), 1)
        assert rc == capi.B2G_ERR_DEVICE_TIMEOUT and st.value != 0, (rc, st.value)
    finally:
        L.b2g_debug_force_stall(0)
        L.b2g_set_wait_timeout_ms(4000)
    assert L.b2g_device_status(C.byref(st), 0) == capi.B2G_OK and st.value == 0
    assert L.b2g_gemm_mxfp8_noalloc(C.byref(args), stream) == capi.B2G_OK
    torch.cuda.synchronize()
    _check(O, d, O.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True), "f32")
    assert L.b2g_device_status(C.byref(st), 0) == capi.B2G_OK and st.value == 0
