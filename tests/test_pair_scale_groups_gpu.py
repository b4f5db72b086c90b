"""GPU parity of the CTA-pair kernel's scale-atom ring at the K lengths that stress it.

The pair kernel's MX kinds load the scale atoms of four consecutive 128-byte K blocks
per TMA box into a two-slot ring and copy them into TMEM one group at a time; a
unit's last group is shorter when its K-block count is not a multiple of four, a
K split starts groups at the split's first block, and a CTA pair that owns more
than one tile keeps loading one group ahead across the tile boundary.  These cases
run the pair tile forced (B2G_FORCE_TILE, the reference host's `--kernel` analogue)
against the oracle: K of 1, 3, 5, 7 and 9 blocks, K splits whose pieces are 2-5
blocks long, and 80 tiles on the 74 pairs.

Tolerances (as in the other parity tests):
  * bf16 C:  max |err| <= 2^-7 * max_n |ref[m, n]| per row   (check_bf16 <= 1)
  * fp32 C:  |err| / max(|ref|, 2^-7 * rowmax) <= 1e-3          (check_f32 <= 1e-3)
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

PAIR = "b2g_sm100a_fp8_pair_256x256"


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gcnasm_b200 import build
    build.build()
    return torch.device("cuda:0")


def T(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


_REFS = {}  # oracle results per operand set (each shape runs with both output types)


def _mx(oracle, M, N, K):
    key = ("mx", M, N, K)
    if key not in _REFS:
        qa, sa = oracle.quant_mx(oracle.normal_rows(1234, 0, M, K))
        qb, sb = oracle.quant_mx(oracle.normal_rows(5678, 0, N, K))
        _REFS[key] = (qa, sa, qb, sb, oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True))
    return _REFS[key]


def _mx4(oracle, M, N, K):
    key = ("mx4", M, N, K)
    if key not in _REFS:
        pa, sa = oracle.fp4_operand(M, K, 1234)
        pb, sb = oracle.fp4_operand(N, K, 5678)
        _REFS[key] = (pa, sa, pb, sb, oracle.gemm_mxfp4(pa, pb, sa, sb, M, N, K, acc_f64=True))
    return _REFS[key]


def _check(oracle, out, ref, od):
    got = out.float().cpu().numpy()
    if od == torch.bfloat16:
        r = oracle.check_bf16(got, ref)
        assert r <= 1.0, f"bf16 error ratio {r}"
    else:
        r = oracle.check_f32(got, ref)
        assert r <= 1e-3, f"fp32 relative error {r}"


# (M, N, K elements, log2 K split): K blocks of 128 bytes = K / 128 for FP8
MX_CASES = [(300, 512, 128, 0), (256, 256, 384, 0), (512, 768, 640, 0), (384, 512, 896, 0),
            (2048, 2560, 640, 0), (256, 1024, 1152, 1), (256, 1024, 1152, 2), (512, 512, 1408, 2)]


@pytest.mark.parametrize("M,N,K,log2", MX_CASES)
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_pair_mxfp8_scale_groups(dev, oracle, monkeypatch, M, N, K, log2, out):
    from gcnasm_b200 import ops
    monkeypatch.setenv("B2G_FORCE_TILE", PAIR)
    od = torch.bfloat16 if out == "bf16" else torch.float32
    qa, sa, qb, sb, ref = _mx(oracle, M, N, K)
    got = ops.mxfp8_gemm(T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev),
                         out_dtype=od, log2_k_split=log2)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    _check(oracle, got, ref, od)


# (M, N, K elements, log2 K split): K blocks of 128 bytes = K / 256 for packed E2M1
MX4_CASES = [(300, 512, 256, 0), (256, 256, 768, 0), (512, 768, 1280, 0), (2048, 2560, 1280, 0),
             (256, 1024, 2304, 1), (256, 512, 2816, 2)]


@pytest.mark.parametrize("M,N,K,log2", MX4_CASES)
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_pair_mxfp4_scale_groups(dev, oracle, monkeypatch, M, N, K, log2, out):
    from gcnasm_b200 import ops
    monkeypatch.setenv("B2G_FORCE_TILE", PAIR)
    od = torch.bfloat16 if out == "bf16" else torch.float32
    pa, sa, pb, sb, ref = _mx4(oracle, M, N, K)
    got = ops.mxfp4_gemm(T(pa, dev), T(pb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev),
                         out_dtype=od, log2_k_split=log2)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    _check(oracle, got, ref, od)


def test_pair_mxfp8_scale_groups_repeat_calls(dev, oracle, monkeypatch):
    """Two calls in a row on the same buffers give bit-identical C (the ring and the
    TMEM scale sets carry nothing from one launch to the next)."""
    from gcnasm_b200 import ops
    monkeypatch.setenv("B2G_FORCE_TILE", PAIR)
    M, N, K = 2048, 2560, 896
    qa, sa = oracle.quant_mx(oracle.normal_rows(11, 0, M, K))
    qb, sb = oracle.quant_mx(oracle.normal_rows(12, 0, N, K))
    args = (T(qa, dev), T(qb, dev), T(oracle.sf_to_tc_layout(sa), dev), T(oracle.sf_to_tc_layout(sb), dev))
    a = ops.mxfp8_gemm(*args, out_dtype=torch.bfloat16)
    b = ops.mxfp8_gemm(*args, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    _check(oracle, a, oracle.gemm_mx(qa, qb, sa, sb, M, N, K, acc_f64=True), torch.bfloat16)
