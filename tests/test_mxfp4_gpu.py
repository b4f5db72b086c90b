"""GPU parity of the MXFP4 path (packed E2M1 operands, UE8M0 1x32 scales: the
reference's own f4gemm element type) through the C ABI against the CPU oracle.

Operands follow the reference's data recipe (make_operand,
asm_f4gemm/f4gemm_ref.hpp:150-177: uniform nibbles, exponents 124..130); the
reference GEMM is the oracle's f64-accumulate restatement of reference_gemm
(f4gemm_ref.hpp:181-222), pinned bit-exactly to the reference's golden output.

Tolerances (as asserted):
  * bf16 C:  max |err| <= 2^-7 * max_n |ref[m, n]|     per row   (check_bf16 <= 1)
  * fp32 C:  |err| / max(|ref|, 2^-7 * rowmax) <= 1e-3            (check_f32 <= 1e-3)
"""
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gcnasm_b200 import build
    build.build()
    return torch.device("cuda:0")


def T(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def fp4_operands(oracle, M, N, K, seed_a=1234, seed_b=5678):
    pa, sa = oracle.fp4_operand(M, K, seed_a)
    pb, sb = oracle.fp4_operand(N, K, seed_b)
    return pa, sa, pb, sb


def check_out(out, ref, od):
    got = out.float().cpu().numpy()
    if od == torch.bfloat16:
        from oracle import oracle as O
        r = O.check_bf16(got, ref)
        assert r <= 1.0, f"bf16 error ratio {r}"
    else:
        from oracle import oracle as O
        r = O.check_f32(got, ref)
        assert r <= 1e-3, f"fp32 relative error {r}"


# pair kernel (M > 128), skinny decode kernel (M <= 128, split tiles), ragged M / N edges
MX4_SHAPES = [(512, 512, 512), (300, 1024, 1024), (256, 768, 2048), (16, 4096, 1024), (1, 2048, 4096),
              (77, 640, 768), (128, 28672, 512)]


@pytest.mark.parametrize("M,N,K", MX4_SHAPES)
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_mxfp4_native(dev, oracle, M, N, K, out):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out == "bf16" else torch.float32
    pa, sa, pb, sb = fp4_operands(oracle, M, N, K)
    ref = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    got = ops.mxfp4_gemm(T(pa, dev), T(pb, dev), T(oracle.sf_to_tc_layout(sa), dev),
                         T(oracle.sf_to_tc_layout(sb), dev), out_dtype=od)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    check_out(got, ref, od)


@pytest.mark.parametrize("M,N,K", [(256, 512, 512), (16, 2048, 1024)])
def test_mxfp4_native_preshuffled_b_alpha(dev, oracle, M, N, K):
    """B through the reference's 16x16 byte preshuffle, alpha applied in the epilogue."""
    from gcnasm_b200 import ops
    pa, sa, pb, sb = fp4_operands(oracle, M, N, K)
    ref = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, alpha=0.5, acc_f64=True)
    b = oracle.shuffle_weight_16x16(pb, N, K // 2).reshape(N, K // 2)
    got = ops.mxfp4_gemm(T(pa, dev), T(b, dev), T(oracle.sf_to_tc_layout(sa), dev),
                         T(oracle.sf_to_tc_layout(sb), dev), out_dtype=torch.float32, alpha=0.5,
                         b_preshuffled=True)
    torch.cuda.synchronize()
    check_out(got, ref, torch.float32)


@pytest.mark.parametrize("log2", [1, 2])
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_mxfp4_splitk(dev, oracle, log2, out):
    from gcnasm_b200 import ops
    od = torch.bfloat16 if out == "bf16" else torch.float32
    M, N, K = 256, 1024, 4096
    pa, sa, pb, sb = fp4_operands(oracle, M, N, K)
    ref = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    got = ops.mxfp4_gemm(T(pa, dev), T(pb, dev), T(oracle.sf_to_tc_layout(sa), dev),
                         T(oracle.sf_to_tc_layout(sb), dev), out_dtype=od, log2_k_split=log2)
    torch.cuda.synchronize()
    check_out(got, ref, od)


# asm_f4gemm/run_tests.sh-style shapes through the reference's kernarg block
F4_SHAPES = [(128, 1024, 1024), (300, 2048, 1024), (1, 4096, 2048), (17, 512, 256), (512, 1024, 2048)]


@pytest.mark.parametrize("M,N,K", F4_SHAPES)
@pytest.mark.parametrize("bpre", [1, 0])
def test_mxfp4_f4gemm_abi(dev, oracle, M, N, K, bpre):
    """The reference's own launch: packed E2M1 A/B padded to 256 rows, scales padded +
    shuffled (shuffle_scale), B optionally through shuffle_weight_16x16 over its bytes,
    strides in E2M1 elements as fill_args writes them."""
    from gcnasm_b200 import f4gemm
    sh = f4gemm.Shape(M, N, K)
    pa, sa, pb, sb = fp4_operands(oracle, M, N, K)
    ref = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    hA = np.zeros((sh.a_rows_pad(), K // 2), np.uint8); hA[:M] = pa
    hB = np.zeros((sh.b_rows_pad(), K // 2), np.uint8)
    hB[:N] = oracle.shuffle_weight_16x16(pb, N, K // 2).reshape(N, K // 2) if bpre else pb
    hSA = oracle.shuffle_scale(sa, M, sh.Ks(), sh.scale_a_rows(), sh.scale_cols())
    hSB = oracle.shuffle_scale(sb, N, sh.Ks(), sh.scale_b_rows(), sh.scale_cols())
    dA, dB, dSA, dSB = T(hA, dev), T(hB, dev), T(hSA, dev), T(hSB, dev)
    dD = torch.zeros((sh.d_rows_pad(), N), dtype=torch.bfloat16, device=dev)
    args = f4gemm.fill_args(dD.data_ptr(), None, dA.data_ptr(), dB.data_ptr(), dSA.data_ptr(), dSB.data_ptr(),
                            M, N, K, N, sh.scale_cols(), sh.scale_cols(), 1.0, 0.0, 0)
    f4gemm.launch(args, bpre, fp4=True)
    torch.cuda.synchronize()
    check_out(dD[:M], ref, torch.bfloat16)


def test_mxfp4_f4gemm_abi_splitk_beta(dev, oracle):
    """Split K (log2 2) and D = alpha * A . B^T + beta * C with C = D (in place)."""
    from gcnasm_b200 import capi, f4gemm
    M, N, K = 256, 1024, 4096
    sh = f4gemm.Shape(M, N, K)
    pa, sa, pb, sb = fp4_operands(oracle, M, N, K)
    alpha, beta = 0.75, -1.25
    acc = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    c_in = torch.from_numpy(oracle.normal_rows(99, 0, M, N))
    ref = (np.float32(alpha) * acc).astype(np.float64) + np.float64(np.float32(beta)) * c_in.numpy()
    dA = T(pa, dev)
    dB = T(oracle.shuffle_weight_16x16(pb, N, K // 2).reshape(N, K // 2), dev)
    dSA = T(oracle.shuffle_scale(sa, M, sh.Ks(), sh.scale_a_rows(), sh.scale_cols()), dev)
    dSB = T(oracle.shuffle_scale(sb, N, sh.Ks(), sh.scale_b_rows(), sh.scale_cols()), dev)
    dD = c_in.to(dev)
    args = f4gemm.fill_args(dD.data_ptr(), dD.data_ptr(), dA.data_ptr(), dB.data_ptr(), dSA.data_ptr(),
                            dSB.data_ptr(), M, N, K, N, sh.scale_cols(), sh.scale_cols(), alpha, beta, 2)
    f4gemm.launch(args, 1, capi.OUT_F32, fp4=True)
    torch.cuda.synchronize()
    check_out(dD, ref, torch.float32)


def test_mxfp4_reference_golden_on_device(dev, oracle, golden):
    """The reference's own make_operand data (8x64 . 4x64) on the device kernel,
    against the reference's own reference_gemm output."""
    from gcnasm_b200 import ops
    pa = golden["op_a_packed"].reshape(8, 32); sa = golden["op_a_scales"].reshape(8, 2)
    pb = golden["op_b_packed"].reshape(4, 32); sb = golden["op_b_scales"].reshape(4, 2)
    ref = golden["ref_gemm_D"].reshape(8, 4).astype(np.float64)
    # K = 64 is below the kernel's 256-element granule: pad K with zero codes (value 0)
    K = 256
    hA = np.zeros((8, K // 2), np.uint8); hA[:, :32] = pa
    hB = np.zeros((16, K // 2), np.uint8); hB[:4, :32] = pb
    hSA = np.full((8, K // 32), 127, np.uint8); hSA[:, :2] = sa
    hSB = np.full((16, K // 32), 127, np.uint8); hSB[:4, :2] = sb
    got = ops.mxfp4_gemm(T(hA, dev), T(hB, dev), T(oracle.sf_to_tc_layout(hSA), dev),
                         T(oracle.sf_to_tc_layout(hSB), dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    check_out(got[:, :4], ref, torch.float32)


_SINGLE_CTA_MX4 = r'''
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from oracle import oracle as O
from gcnasm_b200 import ops
dev = torch.device("cuda:0")
for (M, N, K, pre) in ((512, 512, 512, False), (300, 1024, 1024, True), (64, 1024, 512, False), (1, 512, 256, True)):
    pa, sa = O.fp4_operand(M, K, 1234); pb, sb = O.fp4_operand(N, K, 5678)
    ref = O.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    b = O.shuffle_weight_16x16(pb, N, K // 2).reshape(N, K // 2) if pre else pb
    out = ops.mxfp4_gemm(torch.from_numpy(pa).to(dev), torch.from_numpy(b).to(dev),
                         torch.from_numpy(O.sf_to_tc_layout(sa)).to(dev), torch.from_numpy(O.sf_to_tc_layout(sb)).to(dev),
                         out_dtype=torch.bfloat16, b_preshuffled=pre)
    torch.cuda.synchronize()
    r = O.check_bf16(out.float().cpu().numpy(), ref)
    assert r <= 1.0, (M, N, K, pre, r)
print("single-cta mx4 ok")
'''


def test_mxfp4_single_cta_path(dev):
    """B2G_DISABLE_PAIR=1 / B2G_DISABLE_SKINNY=1: MXFP4 on the single-CTA kernel."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, B2G_DISABLE_PAIR="1", B2G_DISABLE_SKINNY="1")
    r = subprocess.run([sys.executable, "-c", _SINGLE_CTA_MX4, root], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "single-cta mx4 ok" in r.stdout


@pytest.mark.parametrize("M,log2", [(512, 0), (16, 0), (256, 2)])
def test_mxfp4_epilogue_beta_bias(dev, oracle, M, log2):
    """b2g_gemm_mxfp4_ex: D = alpha * A . B^T + beta * C + bias[n], C = D in place."""
    from gcnasm_b200 import ops
    N, K = 1024, 2048
    pa, sa, pb, sb = fp4_operands(oracle, M, N, K)
    alpha, beta = 0.25, 1.5
    acc = oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True)
    c_in = torch.from_numpy(oracle.normal_rows(7, 0, M, N))
    bias = torch.from_numpy(oracle.normal_rows(8, 0, 1, N)[0])
    v = (np.float32(alpha) * acc.astype(np.float32) + np.float32(beta) * c_in.numpy()).astype(np.float32)
    ref = (v + bias.numpy()[None, :]).astype(np.float64)
    dC = c_in.to(dev)
    ops.mxfp4_gemm(T(pa, dev), T(pb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev),
                   out=dC, alpha=alpha, log2_k_split=log2, c=dC, beta=beta, bias=bias.to(dev))
    torch.cuda.synchronize()
    check_out(dC, ref, torch.float32)
