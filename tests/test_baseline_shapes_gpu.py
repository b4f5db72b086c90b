"""GPU parity at the benchmark configurations' real sizes, and the reference's own
regression sweep (asm_f4gemm/run_tests.sh) case for case.

Sizes too large for the oracle to recompute whole are checked on 64 sampled rows
(the first, the last and 62 seeded ones): the oracle recomputes those rows from
the same quantised bytes the GPU consumed.  Tolerances as in the other parity
tests -- bf16 C: max|err| <= 2^-7 * max_n |ref[m, n]| per row; fp32 C:
|err| / max(|ref|, 2^-7 * row max) <= 1e-3.  The block-scale reference is the
f64 form of the reference's gemm_ref loop (pinned bit for bit in its fp32 form
to the reference's own compiled loop); the MX reference is the f64-accumulate
GEMM of the dequantised operands (asm_f4gemm/f4gemm_ref.hpp:181-222).
"""
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


def _rows(M, n=64, seed=0):
    if M <= n:
        return np.arange(M)
    mid = np.random.RandomState(seed).choice(np.arange(1, M - 1), n - 2, replace=False)
    return np.sort(np.concatenate([[0, M - 1], mid]))


def _randn(rows, cols, seed, dev):
    return torch.randn(rows, cols, device=dev, generator=torch.Generator(device=dev).manual_seed(seed))


def _check(oracle, got, ref, bf16):
    g = got.float().cpu().numpy()
    if bf16:
        r = oracle.check_bf16(g, ref)
        assert r <= BF16_TOL, f"bf16 error ratio {r}"
    else:
        r = oracle.check_f32(g, ref)
        assert r <= F32_TOL, f"fp32 relative error {r}"


# ------------------------------------------------------------------ C3: 1x128 block-scale GEMM, 12 shapes
C3_NK = [(7168, 2048), (4096, 7168), (7168, 18432)]
C3_M = [128, 1024, 4096, 16384]


@pytest.mark.parametrize("group_n", [128, 1])
@pytest.mark.parametrize("N,K", C3_NK)
@pytest.mark.parametrize("M", C3_M)
def test_c3_blockscale_sampled_rows(dev, oracle, M, N, K, group_n):
    """Every C3 shape, both weight-scale layouts, bf16 C: A 1x128 fp32 scales
    (amax/448 of N(0,1) rows), B 128x128 block scales (GROUP_N=128) or per-column
    scales over 1x128 (GROUP_N=1)."""
    from gcnasm_b200 import ops
    qa, sfa = ops.quant_1x128(_randn(M, K, 1000 + M, dev))           # sfa [K/128, M]
    w = _randn(N, K, 2000 + N + K, dev)
    if group_n == 128:
        qb, sfb = ops.quant_128x128(w)                                # [N/128, K/128]
    else:
        qb, sfb = ops.quant_1x128(w)                                  # [K/128, N]
    del w
    out = ops.gemm_a8w8_blockscale(qa, qb, sfa, sfb, group_n=group_n, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    rows = _rows(M)
    ri = torch.from_numpy(rows).to(dev)
    a_h = qa[ri].cpu().numpy()
    sfa_h = np.ascontiguousarray(sfa[:, ri].cpu().numpy())
    b_h, sfb_h = qb.cpu().numpy(), sfb.cpu().numpy()
    n = len(rows)
    stride_sfb = K // 128 if group_n == 128 else N
    ref = oracle.gemm_blockscale_f64(a_h, b_h, sfa_h, sfb_h, n, N, K, n, stride_sfb, group_n,
                                     0 if group_n == 128 else 1)
    _check(oracle, out[ri], ref, bf16=True)


# ------------------------------------------------------------------ C4: decode shapes, bf16 C
@pytest.mark.parametrize("N,K", [(28672, 4096), (4096, 14336)])
@pytest.mark.parametrize("M", [1, 16, 64])
def test_c4_decode_bf16(dev, oracle, M, N, K):
    """Every C4 decode shape with bf16 output (the fp32 form is in the decode tests):
    the stream-K decode kernel, all rows against the oracle."""
    from gcnasm_b200 import ops
    qa, sa = ops.quant_mxfp8(_randn(M, K, 3000 + M, dev), "rowmajor")
    qb, sb = ops.quant_mxfp8(_randn(N, K, 4000 + N, dev), "rowmajor")
    out = ops.mxfp8_gemm(qa, qb, ops.sf_rowmajor_to_tc(sa, K), ops.sf_rowmajor_to_tc(sb, K),
                         out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    ref = oracle.gemm_mx(qa.cpu().numpy(), qb.cpu().numpy(), sa.cpu().numpy(), sb.cpu().numpy(), M, N, K,
                         acc_f64=True)
    _check(oracle, out, ref, bf16=True)


# ------------------------------------------------------------------ C5: one shard of the sharded GEMM
def test_c5_shard_sampled_rows(dev, oracle):
    """One GPU's shard of C5 (M=65536 rows over 8 GPUs: 8192 x 28672 x 8192, bf16 C),
    64 sampled rows."""
    from gcnasm_b200 import ops
    M, N, K = 8192, 28672, 8192
    qa, sa = ops.quant_mxfp8(_randn(M, K, 5001, dev), "rowmajor")
    qb, sb = ops.quant_mxfp8(_randn(N, K, 5002, dev), "rowmajor")
    out = ops.mxfp8_gemm(qa, qb, ops.sf_rowmajor_to_tc(sa, K), ops.sf_rowmajor_to_tc(sb, K),
                         out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    rows = _rows(M)
    ri = torch.from_numpy(rows).to(dev)
    ref = oracle.gemm_mx(qa[ri].cpu().numpy(), qb.cpu().numpy(), sa[ri].cpu().numpy(), sb.cpu().numpy(),
                         len(rows), N, K, acc_f64=True)
    _check(oracle, out[ri], ref, bf16=True)


# ------------------------------------------------------------------ asm_f4gemm/run_tests.sh, case for case
def _f4gemm_run(dev, oracle, M, N, K, bpre, log2_split=0):
    """One run of the reference host (asm_f4gemm/main.cpp) through this library's
    f4gemm ABI: padded buffers, shuffled scales, B preshuffled when bpre, bf16 D."""
    from gcnasm_b200 import f4gemm
    sh = f4gemm.Shape(M, N, K)
    qa, sa = oracle.quant_mx(oracle.normal_rows(1234, 0, M, K))
    qb, sb = oracle.quant_mx(oracle.normal_rows(5678, 0, N, K))
    hA = np.zeros((sh.a_rows_pad(), K), np.uint8)
    hA[:M] = qa
    hB = np.zeros((sh.b_rows_pad(), K), np.uint8)
    hB[:N] = oracle.shuffle_weight_16x16(qb, N, K).reshape(N, K) if bpre else qb
    hSA = oracle.shuffle_scale(sa, M, sh.Ks(), sh.scale_a_rows(), sh.scale_cols())
    hSB = oracle.shuffle_scale(sb, N, sh.Ks(), sh.scale_b_rows(), sh.scale_cols())
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
    dA, dB, dSA, dSB = T(hA), T(hB), T(hSA), T(hSB)
    dD = torch.full((sh.d_rows_pad(), N), float("nan"), dtype=torch.bfloat16, device=dev)
    args = f4gemm.fill_args(dD.data_ptr(), None, dA.data_ptr(), dB.data_ptr(), dSA.data_ptr(), dSB.data_ptr(),
                            M, N, K, N, sh.scale_cols(), sh.scale_cols(), 1.0, 0.0, log2_split)
    f4gemm.launch(args, bpre)
    torch.cuda.synchronize()
    rows = _rows(M, 128)
    ref = oracle.gemm_mx(np.ascontiguousarray(qa[rows]), qb, np.ascontiguousarray(sa[rows]), sb, len(rows), N, K,
                         acc_f64=True)
    _check(oracle, dD[torch.from_numpy(rows).to(dev)], ref, bf16=True)


# run_tests.sh:39-44: the heuristic path over its eight shapes (B preshuffled, the host's default)
@pytest.mark.parametrize("M,N,K", [(128, 1024, 1024), (256, 2048, 2048), (300, 2048, 1024), (1, 4096, 2048),
                                   (17, 512, 256), (512, 1024, 2048), (2048, 8192, 1024), (4096, 4096, 512)])
def test_run_tests_heuristic_shapes(dev, oracle, M, N, K):
    _f4gemm_run(dev, oracle, M, N, K, bpre=1)


def _manifest_names():
    from gcnasm_b200 import f4gemm
    return [(c.knl_name, c.bpreshuffle) for c in f4gemm.load_configs()]


# run_tests.sh:46-52: every kernel of the manifest at M=300 N=2048 K=1024, forced
# (the host's --kernel <co>, here B2G_FORCE_TILE), with the B layout it was built for
@pytest.mark.parametrize("name,bpre", _manifest_names())
def test_run_tests_every_manifest_kernel(dev, oracle, monkeypatch, name, bpre):
    monkeypatch.setenv("B2G_FORCE_TILE", name)
    _f4gemm_run(dev, oracle, 300, 2048, 1024, bpre=bpre)


# run_tests.sh:54-59: split-K 1..4 at M=256 N=1024 K=4096 on the two widest
# preshuffled tiles (the reference's 256x256 and 128x512; here the pair 256x256
# and the single-CTA 128x256)
@pytest.mark.parametrize("split", [1, 2, 3, 4])
@pytest.mark.parametrize("name", ["b2g_sm100a_fp8_pair_256x256_bpreshuffle", "b2g_sm100a_fp8_128x256_bpreshuffle"])
def test_run_tests_splitk(dev, oracle, monkeypatch, name, split):
    monkeypatch.setenv("B2G_FORCE_TILE", name)
    _f4gemm_run(dev, oracle, 256, 1024, 4096, bpre=1, log2_split=split)


def test_force_tile_rejects_unknown_name_and_wrong_layout(dev, oracle, monkeypatch):
    from gcnasm_b200 import capi
    monkeypatch.setenv("B2G_FORCE_TILE", "no_such_kernel")
    with pytest.raises(capi.B2GError):
        _f4gemm_run(dev, oracle, 300, 256, 256, bpre=1)
    monkeypatch.setenv("B2G_FORCE_TILE", "b2g_sm100a_fp8_128x256")  # built for row-major B
    with pytest.raises(capi.B2GError):
        _f4gemm_run(dev, oracle, 300, 256, 256, bpre=1)
