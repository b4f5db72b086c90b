"""GPU parity: every kernel path through the C ABI against the CPU oracle on the
same seeded inputs.

Tolerances (the acceptance bounds of this library, written here as asserted):
  * bf16 C:  max |err| <= 2^-7 * max_n |ref[m, n]|     per row   (check_bf16 <= 1)
  * fp32 C:  |err| / max(|ref|, 2^-7 * rowmax) <= 1e-3            (check_f32 <= 1e-3)
  * quantisers, layout shuffles: bit-exact.
The reference for MX is the oracle's f64-accumulate GEMM over dequantised
operands (asm_f4gemm/f4gemm_ref.hpp:181-222); for the opus paths it is the f64
form of gemm_ref (opus_gemm/*/..._host.cc gemm_ref).
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

BF16_TOL = 1.0
F32_TOL = 1e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gcnasm_b200 import build
    build.build()
    return torch.device("cuda:0")


def T(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def mx_operands(oracle, M, N, K, seed_a=1234, seed_b=5678):
    x = oracle.normal_rows(seed_a, 0, M, K)
    w = oracle.normal_rows(seed_b, 0, N, K)
    qa, sa = oracle.quant_mx(x)
    qb, sb = oracle.quant_mx(w)
    return qa, sa, qb, sb


def check_out(out, ref, out_dtype):
    got = out.float().cpu().numpy()
    if out_dtype == torch.bfloat16:
        r = check_bf16(got, ref)
        assert r <= BF16_TOL, f"bf16 error ratio {r}"
    else:
        r = check_f32(got, ref)
        assert r <= F32_TOL, f"fp32 relative error {r}"
    return r


def check_bf16(got, ref):
    from oracle import oracle as O
    return O.check_bf16(got, ref)


def check_f32(got, ref):
    from oracle import oracle as O
    return O.check_f32(got, ref)


# ------------------------------------------------------------------ quantisers / layouts (bit-exact)
@pytest.mark.parametrize("M,K", [(300, 512), (1, 32), (129, 4096)])
def test_quant_mx_bitexact(dev, oracle, M, K):
    from gcnasm_b200 import ops
    x = oracle.normal_rows(1234, 0, M, K) * 3.0
    x[0, :32] = 0.0  # all-zero block -> scale byte 1
    q_ref, sf_ref = oracle.quant_mx(x)
    q, sf_tc = ops.quant_mxfp8(T(x, dev), "tc")
    q2, sf_rm = ops.quant_mxfp8(T(x, dev), "rowmajor")
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(q2.cpu().numpy(), q_ref)
    assert np.array_equal(sf_rm.cpu().numpy(), sf_ref)
    assert np.array_equal(sf_tc.cpu().numpy(), oracle.sf_to_tc_layout(sf_ref))


@pytest.mark.parametrize("M,K", [(300, 512), (129, 4096)])
def test_quant_bf16_input_bitexact(dev, oracle, M, K):
    """bf16 activations into the MXFP8 and 1x128 quantisers: bit-identical to the fp32
    quantiser on the (exactly) widened values."""
    from gcnasm_b200 import ops
    xb = torch.from_numpy(oracle.normal_rows(77, 0, M, K) * 5.0).to(torch.bfloat16)
    xf = xb.float().numpy()
    q_ref, sf_ref = oracle.quant_mx(xf)
    q, sf = ops.quant_mxfp8(xb.to(dev), "rowmajor")
    q1_ref, s1_ref = oracle.quant_1x128(xf)
    q1, s1 = ops.quant_1x128(xb.to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(sf.cpu().numpy(), sf_ref)
    assert np.array_equal(q1.cpu().numpy(), q1_ref) and np.array_equal(s1.cpu().numpy(), s1_ref)


@pytest.mark.parametrize("M,K,dtype", [(300, 512, "f32"), (1, 32, "f32"), (129, 4096, "bf16"), (64, 256, "bf16")])
def test_quant_mxfp4_bitexact(dev, oracle, M, K, dtype):
    """b2g_quant_mxfp4 (packed e2m1 + UE8M0 1x32) against the oracle's restatement:
    packed bytes, row-major scales and the tensor-core scale layout bit-exact; includes
    an all-zero block, exact e2m1 ties and values past the saturation point."""
    from gcnasm_b200 import ops
    x = oracle.normal_rows(4321, 0, M, K) * 3.0
    x[0, :32] = 0.0
    if K >= 64:
        x[0, 32:40] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0], np.float32)  # ties, scale 2^0
        x[0, 40:64] = 0.0
    t = torch.from_numpy(x)
    if dtype == "bf16":
        t = t.to(torch.bfloat16)
    q_ref, sf_ref = oracle.quant_mxfp4(t.float().numpy())
    q, sf_tc = ops.quant_mxfp4(t.to(dev), "tc")
    q2, sf_rm = ops.quant_mxfp4(t.to(dev), "rowmajor")
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(q2.cpu().numpy(), q_ref)
    assert np.array_equal(sf_rm.cpu().numpy(), sf_ref)
    assert np.array_equal(sf_tc.cpu().numpy(), oracle.sf_to_tc_layout(sf_ref))


def test_quant_mxfp4_then_gemm(dev, oracle):
    """bf16 activations and weights quantised on the device to MXFP4, then the MXFP4
    GEMM: the result is the oracle GEMM of the oracle-quantised operands."""
    from gcnasm_b200 import ops
    M, N, K = 256, 512, 1024
    xb = torch.from_numpy(oracle.normal_rows(5, 0, M, K)).to(torch.bfloat16)
    wb = torch.from_numpy(oracle.normal_rows(6, 0, N, K)).to(torch.bfloat16)
    pa, sa = oracle.quant_mxfp4(xb.float().numpy())
    pb, sb = oracle.quant_mxfp4(wb.float().numpy())
    ref = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    qa, sfa = ops.quant_mxfp4(xb.to(dev))
    qb, sfb = ops.quant_mxfp4(wb.to(dev))
    out = ops.mxfp4_gemm(qa, qb, sfa, sfb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    check_out(out, ref, torch.float32)


def test_quant_1x128_and_128x128_bitexact(dev, oracle):
    from gcnasm_b200 import ops
    x = oracle.normal_rows(7, 0, 256, 512)
    q_ref, s_ref = oracle.quant_1x128(x)
    q, s = ops.quant_1x128(T(x, dev))
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)
    q_ref, s_ref = oracle.quant_128x128(x)
    q, s = ops.quant_128x128(T(x, dev))
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)


def test_layout_kernels_bitexact(dev, oracle):
    from gcnasm_b200 import ops
    rs = np.random.RandomState(5)
    N, Kp = 96, 512
    w = rs.randint(0, 256, (N, Kp)).astype(np.uint8)
    ws = ops.shuffle_weight_16x16(T(w, dev))
    assert np.array_equal(ws.cpu().numpy().ravel(), oracle.shuffle_weight_16x16(w, N, Kp))
    assert np.array_equal(ops.unshuffle_weight_16x16(ws).cpu().numpy(), w)
    for rows, cols in ((300, 32), (17, 8), (256, 448)):
        sm, sn = oracle.round_up(rows, 256), oracle.round_up(cols, 8)
        sf = rs.randint(1, 255, (rows, cols)).astype(np.uint8)
        sh = ops.shuffle_scale(T(sf, dev), sm, sn)
        assert np.array_equal(sh.cpu().numpy(), oracle.shuffle_scale(sf, rows, cols, sm, sn))
        tc = ops.sf_f4gemm_to_tc(sh, rows, cols * 32, sn)
        assert np.array_equal(tc.cpu().numpy(), oracle.sf_to_tc_layout(sf))
        tc2 = ops.sf_rowmajor_to_tc(T(sf, dev), cols * 32)
        assert np.array_equal(tc2.cpu().numpy(), oracle.sf_to_tc_layout(sf))


# ------------------------------------------------------------------ MXFP8 native entry
MX_SHAPES = [(128, 256, 128), (512, 512, 512), (300, 512, 1024), (1, 256, 256), (17, 512, 256),
             (100, 272, 160), (256, 1024, 2048)]


@pytest.mark.parametrize("M,N,K", MX_SHAPES)
@pytest.mark.parametrize("out_dtype", ["bf16", "f32"])
def test_mxfp8_native(dev, oracle, M, N, K, out_dtype):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    out = ops.mxfp8_gemm(T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev),
                         T(oracle.sf_to_tc_layout(sb), dev), out_dtype=od)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, od)


@pytest.mark.parametrize("M,N,K", [(256, 512, 512), (33, 1024, 1024)])
def test_mxfp8_native_preshuffled_b(dev, oracle, M, N, K):
    from gcnasm_b200 import ops
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    b_sh = T(oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K), dev)
    for bn_pre in (True,):
        out = ops.mxfp8_gemm(T(qa, dev), b_sh, T(oracle.sf_to_tc_layout(sa), dev),
                             T(oracle.sf_to_tc_layout(sb), dev), out_dtype=torch.float32, b_preshuffled=bn_pre)
        torch.cuda.synchronize()
        check_out(out, ref, torch.float32)


@pytest.mark.parametrize("log2", [1, 2, 3])
@pytest.mark.parametrize("out_dtype", ["bf16", "f32"])
def test_mxfp8_splitk(dev, oracle, log2, out_dtype):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    M, N, K = 64, 1024, 4096
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    out = ops.mxfp8_gemm(T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev),
                         T(oracle.sf_to_tc_layout(sb), dev), out_dtype=od, log2_k_split=log2)
    torch.cuda.synchronize()
    check_out(out, ref, od)


# ------------------------------------------------------------------ f4gemm ABI (reference-facing)
F4_SHAPES = [(128, 1024, 1024), (300, 2048, 1024), (1, 4096, 2048), (17, 512, 256), (512, 1024, 2048)]


@pytest.mark.parametrize("M,N,K", F4_SHAPES)
@pytest.mark.parametrize("bpre", [1, 0])
def test_f4gemm_abi(dev, oracle, M, N, K, bpre):
    """asm_f4gemm/run_tests.sh heuristic shapes through the reference's kernarg block."""
    from gcnasm_b200 import f4gemm
    sh = f4gemm.Shape(M, N, K)
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    hA = np.zeros((sh.a_rows_pad(), K), np.uint8); hA[:M] = qa
    hB = np.zeros((sh.b_rows_pad(), K), np.uint8)
    hB[:N] = oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K) if bpre else qb
    hSA = oracle.shuffle_scale(sa, M, sh.Ks(), sh.scale_a_rows(), sh.scale_cols())
    hSB = oracle.shuffle_scale(sb, N, sh.Ks(), sh.scale_b_rows(), sh.scale_cols())
    dA, dB, dSA, dSB = T(hA, dev), T(hB, dev), T(hSA, dev), T(hSB, dev)
    dD = torch.zeros((sh.d_rows_pad(), N), dtype=torch.bfloat16, device=dev)
    args = f4gemm.fill_args(dD.data_ptr(), None, dA.data_ptr(), dB.data_ptr(), dSA.data_ptr(), dSB.data_ptr(),
                            M, N, K, N, sh.scale_cols(), sh.scale_cols(), 1.0, 0.0, 0)
    f4gemm.launch(args, bpre)
    torch.cuda.synchronize()
    check_out(dD[:M], ref, torch.bfloat16)


@pytest.mark.parametrize("split", [1, 2, 3, 4])
def test_f4gemm_abi_splitk(dev, oracle, split):
    """asm_f4gemm/run_tests.sh split-K sweep shape (M=256 N=1024 K=4096), log2 split 1..4."""
    from gcnasm_b200 import f4gemm
    M, N, K = 256, 1024, 4096
    sh = f4gemm.Shape(M, N, K)
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    dA = T(qa, dev)
    dB = T(oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K), dev)
    dSA = T(oracle.shuffle_scale(sa, M, sh.Ks(), sh.scale_a_rows(), sh.scale_cols()), dev)
    dSB = T(oracle.shuffle_scale(sb, N, sh.Ks(), sh.scale_b_rows(), sh.scale_cols()), dev)
    dD = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)  # no zeroing needed
    args = f4gemm.fill_args(dD.data_ptr(), None, dA.data_ptr(), dB.data_ptr(), dSA.data_ptr(), dSB.data_ptr(),
                            M, N, K, N, sh.scale_cols(), sh.scale_cols(), 1.0, 0.0, split)
    f4gemm.launch(args, 1)
    torch.cuda.synchronize()
    check_out(dD, ref, torch.bfloat16)


@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("split", [0, 2])
@pytest.mark.parametrize("in_place", [False, True])
def test_f4gemm_abi_beta(dev, oracle, out, split, in_place):
    """D = alpha * A . B^T + beta * C through the f4gemm kernarg block
    (f4gemm_ref.hpp:179-210: v = alpha * acc in fp32, then v += beta * C), C separate
    from D or D itself; the reference formula is evaluated on the oracle's GEMM."""
    from gcnasm_b200 import capi, f4gemm
    M, N, K = 200, 512, 1024  # M not a multiple of the tile
    od = torch.bfloat16 if out == "bf16" else torch.float32
    sh = f4gemm.Shape(M, N, K)
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    alpha, beta = 0.75, -1.25
    acc = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    c_in = torch.from_numpy(oracle.normal_rows(99, 0, M, N)).to(od)
    c_f = c_in.float().numpy().astype(np.float64)
    ref = (np.float32(alpha) * acc.astype(np.float32)).astype(np.float64) + np.float64(np.float32(beta)) * c_f
    dA = T(qa, dev)
    dB = T(oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K), dev)
    dSA = T(oracle.shuffle_scale(sa, M, sh.Ks(), sh.scale_a_rows(), sh.scale_cols()), dev)
    dSB = T(oracle.shuffle_scale(sb, N, sh.Ks(), sh.scale_b_rows(), sh.scale_cols()), dev)
    dC = c_in.to(dev)
    dD = dC if in_place else torch.full((M, N), float("nan"), dtype=od, device=dev)
    args = f4gemm.fill_args(dD.data_ptr(), dC.data_ptr(), dA.data_ptr(), dB.data_ptr(), dSA.data_ptr(),
                            dSB.data_ptr(), M, N, K, N, sh.scale_cols(), sh.scale_cols(), alpha, beta, split)
    f4gemm.launch(args, 1, capi.OUT_F32 if out == "f32" else capi.OUT_BF16)
    torch.cuda.synchronize()
    check_out(dD, ref, od)


# ------------------------------------------------------------------ opus block-scale paths
@pytest.mark.parametrize("group_n", [128, 1])
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (300, 512, 1024), (128, 1024, 2048)])
@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
def test_blockscale(dev, oracle, group_n, M, N, K, out_dtype):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    x = oracle.normal_rows(1234, 0, M, K)
    w = oracle.normal_rows(5678, 0, N, K)
    qa, sfa = oracle.quant_1x128(x)
    if group_n == 128:
        qb, sfb = oracle.quant_128x128(w)
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    else:
        qb, sfb_rows = oracle.quant_1x128(w)  # [K/128, N]
        sfb = sfb_rows
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, N, 1, 1)
    out = ops.gemm_a8w8_blockscale(T(qa, dev), T(qb, dev), T(sfa, dev), T(sfb, dev), group_n=group_n, out_dtype=od)
    torch.cuda.synchronize()
    check_out(out, ref, od)


def test_blockscale_reference_data_recipe(dev, oracle):
    """The reference host's own input recipe (gemm_a8w8_blockscale_host.cc:207-210:
    A in U[0,1), B in U[-0.5,0.5), scales in U[0.8,1.2)) with its 1e-3 absolute
    criterion (valid_vector, :46-63) on fp32 C -- seeded here."""
    from gcnasm_b200 import ops
    rs = np.random.RandomState(2024)
    M, N, K = 256, 512, 256
    a = np.array([oracle.lib().orc_f32_to_e4m3(float(v)) for v in rs.uniform(0, 1, M * K)], np.uint8).reshape(M, K)
    b = np.array([oracle.lib().orc_f32_to_e4m3(float(v)) for v in rs.uniform(-.5, .5, N * K)], np.uint8).reshape(N, K)
    sfa = rs.uniform(0.8, 1.2, (K // 128, M)).astype(np.float32)
    sfb = rs.uniform(0.8, 1.2, (N // 128, K // 128)).astype(np.float32)
    ref = oracle.gemm_blockscale(a, b, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    out = ops.gemm_a8w8_blockscale(T(a, dev), T(b, dev), T(sfa, dev), T(sfb, dev), group_n=128,
                                   out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert float(np.abs(out.cpu().numpy() - ref).max()) <= 1e-3 * max(1.0, float(np.abs(ref).max()) / 64)


@pytest.mark.parametrize("log2", [1, 2])
def test_blockscale_splitk(dev, oracle, log2):
    from gcnasm_b200 import ops
    M, N, K = 128, 512, 2048
    x = oracle.normal_rows(11, 0, M, K)
    w = oracle.normal_rows(12, 0, N, K)
    qa, sfa = oracle.quant_1x128(x)
    qb, sfb = oracle.quant_128x128(w)
    ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    for od in (torch.float32, torch.bfloat16):
        out = ops.gemm_a8w8_blockscale(T(qa, dev), T(qb, dev), T(sfa, dev), T(sfb, dev), group_n=128, out_dtype=od,
                                       log2_k_split=log2)
        torch.cuda.synchronize()
        check_out(out, ref, od)


# Shapes whose fewest-waves tile is the 256-wide blockwise tile (12 warps, the
# register re-split between warpgroups): one wave at 256 against two at 128, a
# ragged M, and a K split; 128x128 weight scales.
@pytest.mark.parametrize("M,N,K,log2", [(2048, 2048, 512, 0), (1100, 4096, 512, 0), (1024, 4096, 2048, 1)])
@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("group_n", [128, 1])
def test_blockscale_wide_tile(dev, oracle, M, N, K, log2, out_dtype, group_n):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    qa, sfa = oracle.quant_1x128(oracle.normal_rows(31, 0, M, K))
    if group_n == 128:
        qb, sfb = oracle.quant_128x128(oracle.normal_rows(32, 0, N, K))
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    else:
        qb, sfb = oracle.quant_1x128(oracle.normal_rows(32, 0, N, K))  # [K/128, N]
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, N, 1, 1)
    out = ops.gemm_a8w8_blockscale(T(qa, dev), T(qb, dev), T(sfa, dev), T(sfb, dev), group_n=group_n, out_dtype=od,
                                   log2_k_split=log2)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, od)


# ------------------------------------------------------------------ plain fp8 (fp8_gemm / flatmm)
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (100, 256, 512)])
def test_a8w8(dev, oracle, M, N, K):
    from gcnasm_b200 import ops
    x = oracle.normal_rows(21, 0, M, K)
    w = oracle.normal_rows(22, 0, N, K)
    qa = np.array([oracle.lib().orc_f32_to_e4m3(float(v)) for v in x.ravel()], np.uint8).reshape(M, K)
    qb = np.array([oracle.lib().orc_f32_to_e4m3(float(v)) for v in w.ravel()], np.uint8).reshape(N, K)
    ref = oracle.gemm_a8w8(qa, qb, M, N, K).astype(np.float64) * 0.5
    out = ops.gemm_a8w8(T(qa, dev), T(qb, dev), alpha=0.5, out_dtype=torch.float32)
    torch.cuda.synchronize()
    check_out(out, ref, torch.float32)
    # flat-mm form: B given [K, N] and preshuffled by the reference's shuffle_b
    b_kn = np.ascontiguousarray(qb.T)
    ref_kn = oracle.gemm_a8w8_kn(qa, b_kn, M, N, K).astype(np.float64)
    b_sh = T(oracle.flatmm_shuffle_b(b_kn, N, K).reshape(N, K), dev)
    out = ops.gemm_a8w8(T(qa, dev), b_sh, alpha=1.0, out_dtype=torch.bfloat16, b_preshuffled=True)
    torch.cuda.synchronize()
    check_out(out, ref_kn, torch.bfloat16)


def test_a8w8_batched(dev, oracle):
    from gcnasm_b200 import ops
    B, M, N, K = 3, 128, 256, 256
    x = oracle.normal_rows(31, 0, B * M, K).reshape(B, M, K)
    w = oracle.normal_rows(32, 0, B * N, K).reshape(B, N, K)
    enc = np.vectorize(lambda v: oracle.lib().orc_f32_to_e4m3(float(v)), otypes=[np.uint8])
    qa, qb = enc(x), enc(w)
    out = ops.gemm_a8w8(T(qa, dev), T(qb, dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    for b in range(B):
        ref = oracle.gemm_a8w8(qa[b], qb[b], M, N, K).astype(np.float64)
        check_out(out[b], ref, torch.float32)


@pytest.mark.parametrize("group_n", [128, 1])
def test_blockscale_batched_wide_tile(dev, oracle, group_n):
    """opus_gemm_kargs with batch = 2 (per-batch A, B, C and scale strides) on a shape
    whose fewest-waves tile is the 256-wide blockwise tile (2 x 9 x 16 tiles: two waves,
    against four at 128 wide), both weight-scale layouts, fp32 C."""
    from gcnasm_b200 import capi, ops
    Bt, M, N, K = 2, 1100, 4096, 256
    qas, sas, qbs, sbs, refs = [], [], [], [], []
    for b in range(Bt):
        qa, sa = oracle.quant_1x128(oracle.normal_rows(40 + b, 0, M, K))  # sa [K/128, M]
        if group_n == 128:
            qb, sb = oracle.quant_128x128(oracle.normal_rows(50 + b, 0, N, K))  # [N/128, K/128]
            refs.append(oracle.gemm_blockscale_f64(qa, qb, sa, sb, M, N, K, M, K // 128, 128, 0))
        else:
            qb, sb = oracle.quant_1x128(oracle.normal_rows(50 + b, 0, N, K))  # [K/128, N]
            refs.append(oracle.gemm_blockscale_f64(qa, qb, sa, sb, M, N, K, M, N, 1, 1))
        qas.append(qa); sas.append(sa); qbs.append(qb); sbs.append(sb)
    a, b_ = T(np.stack(qas), dev), T(np.stack(qbs), dev)
    sfa, sfb = T(np.stack(sas), dev), T(np.stack(sbs), dev)
    out = torch.full((Bt, M, N), float("nan"), dtype=torch.float32, device=dev)
    stride_sfb = K // 128 if group_n == 128 else N
    ka = ops.opus_kargs(a, b_, out, sfa[0], sfb[0], stride_sfa=M, stride_sfb=stride_sfb, batch=Bt,
                        stride_sfa_batch=sfa.stride(0), stride_sfb_batch=sfb.stride(0))
    capi.check(capi.lib().b2g_gemm_a8w8_blockscale(C.byref(ka), group_n, capi.OUT_F32, 0, None), "blockscale")
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for b in range(Bt):
        check_out(out[b], refs[b], torch.float32)


# ------------------------------------------------------------------ full-size property check
def test_mxfp8_8192_sampled_rows(dev, oracle):
    """The headline 8192^3 MXFP8 GEMM on the GPU; 64 sampled rows recomputed by the oracle."""
    from gcnasm_b200 import ops
    M = N = K = 8192
    x = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(1234))
    w = torch.randn(N, K, device=dev, generator=torch.Generator(device=dev).manual_seed(5678))
    qa, sa = ops.quant_mxfp8(x, "rowmajor")
    qb, sb = ops.quant_mxfp8(w, "rowmajor")
    out = ops.mxfp8_gemm(qa, qb, ops.sf_rowmajor_to_tc(sa, K), ops.sf_rowmajor_to_tc(sb, K), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    rows = np.random.RandomState(0).choice(M, 64, replace=False)
    qa_h, sa_h = qa.cpu().numpy(), sa.cpu().numpy()
    ref = oracle.gemm_mx(np.ascontiguousarray(qa_h[rows]), qb.cpu().numpy(), np.ascontiguousarray(sa_h[rows]),
                         sb.cpu().numpy(), 64, N, K, acc_f64=True)
    check_out(out[torch.from_numpy(rows).to(dev)], ref, torch.bfloat16)


# ------------------------------------------------------------------ bounded waits (failure detection)
def test_bounded_wait_reports_timeout_and_context_survives(dev, oracle):
    """A test hook makes the MMA issuer wait on a barrier nothing arrives on; the
    wait gives up after its limit, the kernel retires cleanly, the status word
    says so, and the next launch on the same context is correct."""
    from gcnasm_b200 import capi, ops
    L = capi.lib()
    M, N, K = 128, 256, 256
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    args = (T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev))
    assert ops.device_status(clear=True) == 0
    L.b2g_set_wait_timeout_ms(200)
    L.b2g_debug_force_stall(1)
    try:
        ops.mxfp8_gemm(*args, out_dtype=torch.float32)
        st = C.c_int(0)
        rc = L.b2g_device_status(C.byref(st), 1)
        assert rc == capi.B2G_ERR_DEVICE_TIMEOUT and st.value == 2  # kDevTimeoutMma
    finally:
        L.b2g_debug_force_stall(0)
        L.b2g_set_wait_timeout_ms(4000)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    out = ops.mxfp8_gemm(*args, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, torch.float32)


# ------------------------------------------------------------------ single-CTA path at pair-sized shapes
_SINGLE_CTA_SCRIPT = r'''
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from oracle import oracle as O
from gcnasm_b200 import ops
dev = torch.device("cuda:0")
for (M, N, K, pre) in ((512, 512, 512, False), (300, 1024, 1024, True), (64, 1024, 512, False), (1, 512, 256, True)):
    qa, sa = O.quant_mx(O.normal_rows(1234, 0, M, K)); qb, sb = O.quant_mx(O.normal_rows(5678, 0, N, K))
    ref = O.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    b = O.shuffle_weight_16x16(qb, N, K).reshape(N, K) if pre else qb
    out = ops.mxfp8_gemm(torch.from_numpy(qa).to(dev), torch.from_numpy(b).to(dev),
                         torch.from_numpy(O.sf_to_tc_layout(sa)).to(dev), torch.from_numpy(O.sf_to_tc_layout(sb)).to(dev),
                         out_dtype=torch.bfloat16, b_preshuffled=pre)
    torch.cuda.synchronize()
    r = O.check_bf16(out.float().cpu().numpy(), ref)
    assert r <= 1.0, (M, N, K, pre, r)
print("single-cta ok")
'''


def test_single_cta_path_when_pairs_disabled(dev):
    """B2G_DISABLE_PAIR=1 / B2G_DISABLE_SKINNY=1 route every shape to the single-CTA kernel."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, B2G_DISABLE_PAIR="1", B2G_DISABLE_SKINNY="1")
    r = subprocess.run([sys.executable, "-c", _SINGLE_CTA_SCRIPT, root], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "single-cta ok" in r.stdout


_FOLD_SCRIPT = r'''
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from oracle import oracle as O
from gcnasm_b200 import ops
dev = torch.device("cuda:0")
outs = []
for (M, N, K) in ((16, 4096, 14336), (1, 4096, 14336), (16, 2048, 4096)):
    qa, sa = O.quant_mx(O.normal_rows(31, 0, M, K)); qb, sb = O.quant_mx(O.normal_rows(32, 0, N, K))
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    for od in (torch.float32, torch.bfloat16):
        out = ops.mxfp8_gemm(T(qa), T(qb), T(O.sf_to_tc_layout(sa)), T(O.sf_to_tc_layout(sb)), out_dtype=od)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        outs.append(out.view(torch.uint8).cpu().numpy().ravel())
np.save(sys.argv[2], np.concatenate(outs))
'''


def test_decode_cluster_fold_matches_l2_fold(dev, tmp_path):
    """Decode shapes whose every tile is split into equal pieces, one per CTA
    (16 x 4096 x 14336: 32 tiles x 4 pieces on 128 CTAs), run in clusters whose
    pieces meet in shared memory; with B2G_CLUSTER_FOLD=0 they meet through L2
    slots and counters.  Both add the pieces in the same order, so C is bit for bit
    the same (fp32 and bf16)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = {}
    for mode in ("1", "0"):
        f = str(tmp_path / f"fold{mode}.npy")
        env = dict(os.environ, B2G_CLUSTER_FOLD=mode)
        r = subprocess.run([sys.executable, "-c", _FOLD_SCRIPT, root, f], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        res[mode] = np.load(f)
    assert np.array_equal(res["1"], res["0"])


def test_bounded_wait_pair_kernel(dev, oracle):
    """The stall hook on the CTA-pair kernel: the leader's MMA wait gives up, both
    CTAs retire through their bounded waits, and the context stays usable."""
    from gcnasm_b200 import capi, ops
    L = capi.lib()
    M, N, K = 512, 512, 256
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    args = (T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev))
    assert ops.device_status(clear=True) == 0
    L.b2g_set_wait_timeout_ms(200)
    L.b2g_debug_force_stall(1)
    try:
        ops.mxfp8_gemm(*args, out_dtype=torch.float32)
        st = C.c_int(0)
        assert L.b2g_device_status(C.byref(st), 1) == capi.B2G_ERR_DEVICE_TIMEOUT and st.value != 0
    finally:
        L.b2g_debug_force_stall(0)
        L.b2g_set_wait_timeout_ms(4000)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    out = ops.mxfp8_gemm(*args, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, torch.float32)


@pytest.mark.parametrize("M", [1, 16, 64, 128])
@pytest.mark.parametrize("bpre", [False, True])
def test_skinny_decode_shapes(dev, oracle, M, bpre):
    """Decode shapes (C4: N=28672, K=4096) on the transposed stream-K kernel, fp32 C."""
    from gcnasm_b200 import ops
    N, K = 28672, 4096
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    b = T(oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K), dev) if bpre else T(qb, dev)
    out = ops.mxfp8_gemm(T(qa, dev), b, T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev),
                         out_dtype=torch.float32, b_preshuffled=bpre)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, torch.float32)


@pytest.mark.parametrize("M", [1, 16, 64])
@pytest.mark.parametrize("bpre", [False, True])
def test_skinny_decode_shapes_long_k(dev, oracle, M, bpre):
    """The second C4 decode shape (N=4096, K=14336), fp32 C: 32 weight tiles for
    148 CTAs, so every tile's 56 K units are split over about five CTAs and no CTA
    owns a whole tile."""
    from gcnasm_b200 import ops
    N, K = 4096, 14336
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    b = T(oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K), dev) if bpre else T(qb, dev)
    args = (T(qa, dev), b, T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev))
    out = ops.mxfp8_gemm(*args, out_dtype=torch.float32, b_preshuffled=bpre)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, torch.float32)
    again = ops.mxfp8_gemm(*args, out_dtype=torch.float32, b_preshuffled=bpre)
    torch.cuda.synchronize()
    assert torch.equal(out, again)  # the split-tile partials are folded in a fixed order


# Split-tile fixup of the skinny kernel: a tile's K range shared by several CTAs
# (up to 64 segments when N is small and K large), K not a multiple of 256 (one
# K block per ring stage) or of 128 (plain (K, rows) maps with a zero-filled
# tail), every padded M, both output types.  The last two have more tiles than
# 1.5 CTAs' worth: every CTA also owns whole tiles after its stream-K units (two
# each for N = 449 tiles with a ragged K; one for 297 tiles, where a second would
# leave each CTA under half a tile of stream-K work).
SKINNY_SPLIT = [(16, 256, 16384, "f32"), (5, 384, 8320, "bf16"), (16, 512, 4000, "f32"),
                (64, 1024, 8192, "bf16"), (128, 640, 4096, "f32"), (33, 4096, 2048, "bf16"),
                (7, 57472, 1056, "bf16"), (20, 38016, 2048, "f32")]


@pytest.mark.parametrize("M,N,K,out", SKINNY_SPLIT)
def test_skinny_split_tiles(dev, oracle, M, N, K, out):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out == "bf16" else torch.float32
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    args = (T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev))
    first = ops.mxfp8_gemm(*args, out_dtype=od)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(first, ref, od)
    # the partials are added in segment order: a repeat is bit-identical, also
    # after a call of another shape has used the same tile counters
    qa2, sa2, qb2, sb2 = mx_operands(oracle, 7, 256, 8192, seed_a=11, seed_b=12)
    ops.mxfp8_gemm(T(qa2, dev), T(qb2, dev), T(oracle.sf_to_tc_layout(sa2), dev),
                   T(oracle.sf_to_tc_layout(sb2), dev), out_dtype=torch.float32)
    again = ops.mxfp8_gemm(*args, out_dtype=od)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_skinny_plain_fp8_split_tiles(dev, oracle):
    """Plain FP8 (alpha only) on the skinny kernel, split tiles, bf16 out."""
    from gcnasm_b200 import ops
    M, N, K = 9, 384, 6144
    qa, _ = oracle.quant_1x128(oracle.normal_rows(41, 0, M, K))  # E4M3 bytes; scales unused
    qb, _ = oracle.quant_1x128(oracle.normal_rows(42, 0, N, K))
    ref = oracle.gemm_a8w8(qa, qb, M, N, K).astype(np.float64) * 0.25
    out = ops.gemm_a8w8(T(qa, dev), T(qb, dev), alpha=0.25, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, torch.bfloat16)


def test_skinny_cuda_graph_replay(dev, oracle):
    """Decode loops replay captured launches: the tile counters are left at zero
    by every launch, so each replay of the same captured launches (same counter
    tag) recomputes the same bits."""
    from gcnasm_b200 import ops
    M, N, K = 16, 768, 8192  # 6 tiles over many CTAs: every tile split
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    args = (T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev))
    out = torch.empty((M, N), dtype=torch.float32, device=dev)
    eager = ops.mxfp8_gemm(*args, out_dtype=torch.float32)  # also the warm-up before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.mxfp8_gemm(*args, out=out)
        ops.mxfp8_gemm(*args, out=out)
    for _ in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert ops.device_status() == 0
    check_out(out, ref, torch.float32)


# Blockwise scales with M <= 32 rows and more 128-row tiles than SMs run on the
# stream-K decode kernel that folds each 128-K block into registers (M=16/32: one
# or two K blocks per stage, split tiles, both scale layouts, both output types);
# M=7 (scale rows not 16-byte aligned) and the smaller shapes exercise the
# single-CTA kernel's small-M path.
SKINNY_BLK = [(16, 19200, 1536, 128, "f32"), (12, 19328, 2048, 128, "bf16"), (16, 19456, 640, 1, "bf16"),
              (32, 19200, 1280, 1, "f32"), (7, 19200, 768, 128, "bf16"), (1, 256, 8192, 128, "f32"),
              (64, 384, 6144, 1, "f32"), (128, 7168, 2048, 128, "bf16")]


@pytest.mark.parametrize("M,N,K,group_n,out", SKINNY_BLK)
def test_blockscale_skinny(dev, oracle, M, N, K, group_n, out):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out == "bf16" else torch.float32
    qa, sfa = oracle.quant_1x128(oracle.normal_rows(71, 0, M, K))
    if group_n == 128:
        qb, sfb = oracle.quant_128x128(oracle.normal_rows(72, 0, N, K))
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    else:
        qb, sfb = oracle.quant_1x128(oracle.normal_rows(72, 0, N, K))  # [K/128, N]
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, N, 1, 1)
    args = (T(qa, dev), T(qb, dev), T(sfa, dev), T(sfb, dev))
    first = ops.gemm_a8w8_blockscale(*args, group_n=group_n, out_dtype=od)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(first, ref, od)
    again = ops.gemm_a8w8_blockscale(*args, group_n=group_n, out_dtype=od)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_static_weights_decode_waits_for_activations(dev, oracle):
    """With static weights on, a decode GEMM streams B before the preceding kernel
    ends but must still read A after it: A is overwritten by an elementwise kernel
    (not a memcpy, so the GEMM is launched as its programmatic dependent) right
    before each GEMM on the same stream, eagerly and in a replayed CUDA graph, and
    every result is the GEMM of the new A."""
    from gcnasm_b200 import ops
    M, N, K = 16, 4096, 4096
    qa1, sa1, qb, sb = mx_operands(oracle, M, N, K)
    qa2, _, _, _ = mx_operands(oracle, M, N, K, seed_a=4321)
    sfb = T(oracle.sf_to_tc_layout(sb), dev)
    sfa = T(oracle.sf_to_tc_layout(sa1), dev)  # kept for both: only the bytes of A change
    b = T(qb, dev)
    a_src = [T(qa1, dev), T(qa2, dev)]
    want = [ops.mxfp8_gemm(x, b, sfa, sfb, out_dtype=torch.float32) for x in a_src]
    assert not torch.equal(want[0], want[1])
    a = torch.empty_like(a_src[0])
    out = torch.empty((M, N), dtype=torch.float32, device=dev)
    ops.set_static_weights(True)
    try:
        for i in range(6):
            torch.bitwise_or(a_src[i % 2], 0, out=a)
            ops.mxfp8_gemm(a, b, sfa, sfb, out=out)
            torch.cuda.synchronize()
            assert torch.equal(out, want[i % 2]), i
        outs = [torch.empty_like(out) for _ in range(4)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(4):
                torch.bitwise_or(a_src[i % 2], 0, out=a)
                ops.mxfp8_gemm(a, b, sfa, sfb, out=outs[i])
        for _ in range(2):
            g.replay()
            torch.cuda.synchronize()
            for i in range(4):
                assert torch.equal(outs[i], want[i % 2]), i
    finally:
        ops.set_static_weights(False)
    assert ops.device_status() == 0


# ------------------------------------------------------------------ fused epilogue terms
# D = alpha * A . B^T + beta * C + bias[n] (b2g_gemm_mxfp8_ex): the reference CPU GEMM's
# v = alpha * acc; v += beta * C (f4gemm_ref.hpp:179-210), then the split-K reduce's
# per-column bias (splitk_reduce_gfx950.cuh:49-60), each in fp32.  Routes: CTA pair
# (M > 128), decode kernel (M <= 128), split-K through the workspace and the reduce.
@pytest.mark.parametrize("M,N,K,log2", [(512, 512, 1024, 0), (16, 4096, 1024, 0), (300, 1024, 2048, 2),
                                        (200, 768, 512, 0)])
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("in_place", [False, True])
def test_mxfp8_epilogue_beta_bias(dev, oracle, M, N, K, log2, out, in_place):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out == "bf16" else torch.float32
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    alpha, beta = 0.5, -0.75
    acc = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    c_in = torch.from_numpy(oracle.normal_rows(77, 0, M, N)).to(od)
    bias = torch.from_numpy(oracle.normal_rows(78, 0, 1, N)[0] * 4).to(od)
    v = np.float32(alpha) * acc.astype(np.float32)
    v = (v + np.float32(beta) * c_in.float().numpy()).astype(np.float32)
    ref = (v + bias.float().numpy()[None, :]).astype(np.float64)
    dC = c_in.to(dev)
    out_t = dC if in_place else torch.full((M, N), float("nan"), dtype=od, device=dev)
    ops.mxfp8_gemm(T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev),
                   out=out_t, alpha=alpha, log2_k_split=log2, c=dC, beta=beta, bias=bias.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out_t, ref, od)


def test_mxfp8_epilogue_bias_only(dev, oracle):
    """bias without a C term, bf16 output, ragged M and N"""
    from gcnasm_b200 import ops
    M, N, K = 333, 1040, 512
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    bias = torch.from_numpy(oracle.normal_rows(5, 0, 1, N)[0]).to(torch.bfloat16)
    ref = (oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True).astype(np.float32)
           + bias.float().numpy()[None, :]).astype(np.float64)
    got = ops.mxfp8_gemm(T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev),
                         T(oracle.sf_to_tc_layout(sb), dev), out_dtype=torch.bfloat16, bias=bias.to(dev))
    torch.cuda.synchronize()
    check_out(got, ref, torch.bfloat16)


@pytest.mark.parametrize("M,N,K,out,n_peers,self_index", [(512, 1024, 512, "bf16", 4, 1), (300, 768, 1024, "f32", 3, 2),
                                                          (100, 512, 256, "bf16", 2, 0)])
def test_mxfp8_a2a_out_local_peers(dev, oracle, M, N, K, out, n_peers, self_index):
    """b2g_gemm_mxfp8_a2a_out with every "peer" window a separate buffer on this GPU:
    column shard q of C lands in window q's rows [self * M, (self + 1) * M) and
    nothing else in any window is written (the pair, single-CTA and ragged-M routes)."""
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out == "bf16" else torch.float32
    qa, sa, qb, sb = mx_operands(oracle, M, N, K)
    ref = oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True)
    shard = N // n_peers
    wins = [torch.full((n_peers * M, shard), float("nan"), dtype=od, device=dev) for _ in range(n_peers)]
    ops.mxfp8_gemm_a2a_out(T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev),
                           T(oracle.sf_to_tc_layout(sb), dev), wins[self_index],
                           [w.data_ptr() for w in wins], self_index)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for q, w in enumerate(wins):
        block = w[self_index * M:(self_index + 1) * M]
        check_out(block, ref[:, q * shard:(q + 1) * shard], od)
        rest = torch.cat([w[:self_index * M], w[(self_index + 1) * M:]])
        assert torch.isnan(rest.float()).all()


# ------------------------------------------------------------------ blockwise, 32 < M <= 128: untransposed stream-K
@pytest.mark.parametrize("M,N,K", [(128, 7168, 2048), (100, 1024, 4096), (64, 4096, 7168), (40, 512, 1024),
                                   (128, 256, 128), (24, 2048, 1024)])
@pytest.mark.parametrize("group_n", [128, 1])
@pytest.mark.parametrize("out_dtype", ["bf16", "f32"])
def test_blockscale_stream_k_untransposed(dev, oracle, monkeypatch, M, N, K, group_n, out_dtype):
    """Rows of A on the MMA's M, every SM on a stream-K share of (tile, K block)
    units, split tiles folded in the kernel (forced with B2G_BLK_NT=1, which the
    default routing picks for long K only): ragged M, tiles cut into many pieces
    (K=7168 over 32 tiles), few units (one tile), both weight-scale layouts."""
    from gcnasm_b200 import ops
    monkeypatch.setenv("B2G_BLK_NT", "1")
    od = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    qa, sfa = oracle.quant_1x128(oracle.normal_rows(61, 0, M, K))
    if group_n == 128:
        qb, sfb = oracle.quant_128x128(oracle.normal_rows(62, 0, N, K))
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    else:
        qb, sfb = oracle.quant_1x128(oracle.normal_rows(62, 0, N, K))  # [K/128, N]
        ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, N, 1, 1)
    args = (T(qa, dev), T(qb, dev), T(sfa, dev), T(sfb, dev))
    for _ in range(2):  # twice: the tile counters are back at zero after a launch
        out = ops.gemm_a8w8_blockscale(*args, group_n=group_n, out_dtype=od)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        check_out(out, ref, od)


@pytest.mark.parametrize("nt", ["1", "0"])
def test_bounded_wait_blockwise_decode_kernel(dev, oracle, monkeypatch, nt):
    """The stall hook on the blockwise decode kernel (untransposed, and transposed at
    M=16 over more weight tiles than SMs): the MMA issuer's wait gives up, every
    epilogue warp leaves through its bounded waits and the per-segment agreement,
    the status word reports it, and the next call on the context is correct."""
    from gcnasm_b200 import capi, ops
    monkeypatch.setenv("B2G_BLK_NT", nt)
    L = capi.lib()
    M, N, K = (100, 1024, 2048) if nt == "1" else (16, 160 * 128, 512)
    qa, sfa = oracle.quant_1x128(oracle.normal_rows(71, 0, M, K))
    qb, sfb = oracle.quant_128x128(oracle.normal_rows(72, 0, N, K))
    args = (T(qa, dev), T(qb, dev), T(sfa, dev), T(sfb, dev))
    assert ops.device_status(clear=True) == 0
    L.b2g_set_wait_timeout_ms(200)
    L.b2g_debug_force_stall(1)
    try:
        ops.gemm_a8w8_blockscale(*args, group_n=128, out_dtype=torch.float32)
        st = C.c_int(0)
        assert L.b2g_device_status(C.byref(st), 1) == capi.B2G_ERR_DEVICE_TIMEOUT and st.value != 0
    finally:
        L.b2g_debug_force_stall(0)
        L.b2g_set_wait_timeout_ms(4000)
    ref = oracle.gemm_blockscale_f64(qa, qb, sfa, sfb, M, N, K, M, K // 128, 128, 0)
    out = ops.gemm_a8w8_blockscale(*args, group_n=128, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(out, ref, torch.float32)
