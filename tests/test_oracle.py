"""The CPU oracle, pinned against the reference's own code (golden fixtures made
from oracle/_ref, and oracle/_ref itself where it was built) and against
independent decoders (std::mt19937_64 known answers, torch's float8 dtypes)."""
import numpy as np
import pytest
import torch


def test_e8m0_matches_reference(oracle, golden):
    mine = np.array([oracle.lib().orc_e8m0_to_f32(i) for i in range(256)], np.float32)
    ref = golden["e8m0"]
    assert np.array_equal(np.isnan(mine), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(mine[ok].view(np.uint32), ref[ok].view(np.uint32))
    assert np.array_equal(oracle.e8m0_decode(np.arange(256))[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_e4m3_decode_matches_torch(oracle):
    t = oracle.e4m3_table()
    tt = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(t), np.isnan(tt))
    assert np.array_equal(t[~np.isnan(t)], tt[~np.isnan(tt)])
    assert t[0x7E] == 448.0 and t[0x01] == 2.0 ** -9 and t[0x08] == 2.0 ** -6


def test_e4m3_encode_rne_matches_torch(oracle):
    rs = np.random.RandomState(0)
    x = np.concatenate([np.clip(rs.randn(50000) * 100, -463, 463), rs.randn(50000) * 0.01,
                        [0.0, -0.0, 2 ** -10, 3 * 2 ** -11, 5 * 2 ** -11, 448.0, 463.9, -463.9]]).astype(np.float32)
    mine = np.array([oracle.lib().orc_f32_to_e4m3(float(v)) for v in x], np.uint8)
    th = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, th)
    # saturation (the reference's host casts are SATFINITE) and NaN
    assert oracle.lib().orc_f32_to_e4m3(1e6) == 0x7E and oracle.lib().orc_f32_to_e4m3(-1e6) == 0xFE
    assert oracle.lib().orc_f32_to_e4m3(float("nan")) == 0x7F


def test_mt19937_64_known_answers(oracle):
    # first outputs of std::mt19937_64 seeded 1234 (libstdc++), and the 10000th
    # output of the default seed 5489 (the C++ standard's required value)
    o = np.empty(1, np.uint64)
    oracle.lib().orc_mt19937_64(1234, o, 1)
    assert int(o[0]) == 17473339210090333472
    o = np.empty(10000, np.uint64)
    oracle.lib().orc_mt19937_64(5489, o, 10000)
    assert int(o[-1]) == 9981545732273789042


def test_normal_rows_reproducible_by_shard(oracle):
    full = oracle.normal_rows(1234, 0, 512, 96)
    part = oracle.normal_rows(1234, 256, 128, 96)
    assert np.array_equal(full[256:384], part)
    assert abs(float(full.mean())) < 0.02 and abs(float(full.std()) - 1.0) < 0.02


def test_mx_scale_rule(oracle):
    L = oracle.lib()
    for amax in [0.0, 1e-30, 0.5, 1.0, 447.9, 448.0, 448.1, 896.0, 3.5, 7.0, 1.75 * 2 ** 5]:
        e = L.orc_mx_scale_byte(amax)
        if amax == 0.0:
            assert e == 1
            continue
        s = 2.0 ** (e - 127)
        assert s * 448 >= amax * (1 - 1e-12) and (e == 1 or s / 2 * 448 < amax)


def test_quant_mx_roundtrip(oracle):
    x = oracle.normal_rows(1234, 0, 64, 256)
    q, sf = oracle.quant_mx(x)
    deq = oracle.e4m3_decode(q) * np.repeat(oracle.e8m0_decode(sf), 32, axis=1)
    rel = np.abs(deq - x) / np.maximum(np.abs(x), 1e-3)
    assert np.median(rel) < 0.04 and np.all(np.abs(deq) <= np.abs(x).max() * 1.07)
    # every block's max lands in the top binade of E4M3
    blk = np.abs(oracle.e4m3_decode(q)).reshape(64, 8, 32).max(axis=2)
    assert np.all(blk >= 224) and np.all(blk <= 448)  # amax/s in (224, 448], then RNE


def test_shuffle_weight_matches_reference(oracle, golden):
    N, Kp = golden["sw_shape"]
    mine = oracle.shuffle_weight_16x16(golden["sw_src"], int(N), int(Kp))
    assert np.array_equal(mine, golden["sw_dst"])


def test_shuffle_scale_matches_reference(oracle, golden):
    rows, cols, sm, sn = (int(v) for v in golden["ss_shape"])
    mine = oracle.shuffle_scale(golden["ss_src"], rows, cols, sm, sn)
    assert np.array_equal(mine, golden["ss_dst"])


def test_flatmm_shuffle_equals_f4gemm_layout(oracle):
    # one byte per E4M3 element: opus_fmm's shuffle_b of a [K, N] source equals
    # f4gemm's shuffle_weight_16x16 of the transposed [N, K] buffer
    rs = np.random.RandomState(3)
    K, N = 64, 48
    b_kn = rs.randint(0, 256, (K, N)).astype(np.uint8)
    a = oracle.flatmm_shuffle_b(b_kn, N, K)
    b = oracle.shuffle_weight_16x16(np.ascontiguousarray(b_kn.T), N, K)
    assert np.array_equal(a, b)


def test_reference_gemm_f64_matches_reference(oracle, golden):
    # reference_gemm (f4gemm_ref.hpp:181-222) on the reference's own make_operand
    # data: the oracle's f64 MX GEMM on the same dequantised values must agree
    A = golden["op_a_dequant"].reshape(8, 64)
    B = golden["op_b_dequant"].reshape(4, 64)
    ref = golden["ref_gemm_D"].reshape(8, 4)
    mine = (A.astype(np.float64) @ B.astype(np.float64).T).astype(np.float32)
    assert np.array_equal(mine, ref)


def test_mxfp4_oracle_matches_reference_golden(oracle, golden):
    # the reference's own MXFP4 operands (make_operand, f4gemm_ref.hpp:150-177):
    # the oracle's e2m1 decode reproduces its dequantised values and the oracle's
    # f64 GEMM over the packed bytes reproduces reference_gemm (f4gemm_ref.hpp:181-222)
    pa = golden["op_a_packed"].reshape(8, 32)
    sa = golden["op_a_scales"].reshape(8, 2)
    pb = golden["op_b_packed"].reshape(4, 32)
    sb = golden["op_b_scales"].reshape(4, 2)
    da = oracle.e2m1_decode(pa) * np.repeat(oracle.e8m0_decode(sa), 32, axis=1)
    db = oracle.e2m1_decode(pb) * np.repeat(oracle.e8m0_decode(sb), 32, axis=1)
    assert np.array_equal(da, golden["op_a_dequant"].reshape(8, 64))
    assert np.array_equal(db, golden["op_b_dequant"].reshape(4, 64))
    d = oracle.gemm_mxfp4(pa, pb, sa, sb, 8, 4, 64, acc_f64=True)
    assert np.array_equal(d, golden["ref_gemm_D"].reshape(8, 4))
    assert [oracle.lib().orc_e2m1_to_f32(i) for i in range(16)] == list(oracle.E2M1)


def test_mxfp4_oracle_f32_close_to_f64(oracle):
    pa, sa = oracle.fp4_operand(24, 512, 1)
    pb, sb = oracle.fp4_operand(40, 512, 2)
    f64 = oracle.gemm_mxfp4(pa, pb, sa, sb, 24, 40, 512, acc_f64=True)
    f32 = oracle.gemm_mxfp4(pa, pb, sa, sb, 24, 40, 512, acc_f64=False)
    da = oracle.e2m1_decode(pa).astype(np.float64) * np.repeat(oracle.e8m0_decode(sa), 32, axis=1)
    db = oracle.e2m1_decode(pb).astype(np.float64) * np.repeat(oracle.e8m0_decode(sb), 32, axis=1)
    np.testing.assert_allclose(f64, da @ db.T, rtol=1e-6, atol=1e-6)
    assert oracle.check_f32(f32, f64) < 1e-5


def test_e2m1_rounding_is_nearest_even(oracle):
    # the MXFP4 quantiser's element rounding against a brute-force search: nearest
    # value of the e2m1 grid, ties to the even code, saturation at 6, sign kept
    L = oracle.lib()
    grid = oracle.E2M1[:8].astype(np.float64)
    mids = (grid[1:] + grid[:-1]) / 2
    rs = np.random.RandomState(0)
    xs = np.concatenate([rs.uniform(-7, 7, 4000), grid, -grid, mids, -mids, [6.5, 100.0, -100.0, -0.1]])
    for x in xs.astype(np.float32):
        a = min(abs(float(x)), 6.0)
        d = np.abs(grid - a)
        best = np.flatnonzero(d == d.min())
        code = int(best[0]) if len(best) == 1 else int([b for b in best if b % 2 == 0][0])
        assert L.orc_f32_to_e2m1(float(x)) == code | (8 if np.signbit(x) else 0), x


def test_mxfp4_scale_rule(oracle):
    # s = 2^ceil(log2(amax / 6)): every |x / s| <= 6, and the next smaller power would overflow
    L = oracle.lib()
    for amax in [6.0, 6.0001, 5.999, 3.0, 0.75, 1e-3, 1.0, 12.0, 1e30]:
        e = L.orc_mxfp4_scale_byte(amax) - 127
        assert amax / 2.0 ** e <= 6.0 and (e - 1 + 127 < 1 or amax / 2.0 ** (e - 1) > 6.0), amax
    assert L.orc_mxfp4_scale_byte(0.0) == 1


def test_gemm_mx_oracle_consistent(oracle):
    x = oracle.normal_rows(1234, 0, 32, 128)
    w = oracle.normal_rows(5678, 0, 48, 128)
    qa, sa = oracle.quant_mx(x)
    qb, sb = oracle.quant_mx(w)
    f64 = oracle.gemm_mx(qa, qb, sa, sb, 32, 48, 128, acc_f64=True)
    f32 = oracle.gemm_mx(qa, qb, sa, sb, 32, 48, 128, acc_f64=False)
    da = oracle.e4m3_decode(qa) * np.repeat(oracle.e8m0_decode(sa), 32, axis=1)
    db = oracle.e4m3_decode(qb) * np.repeat(oracle.e8m0_decode(sb), 32, axis=1)
    np.testing.assert_allclose(f64, (da.astype(np.float64) @ db.T.astype(np.float64)), rtol=1e-6, atol=1e-6)
    assert oracle.check_f32(f32, f64) < 1e-5


def test_blockscale_refs_consistent(oracle):
    rs = np.random.RandomState(1)
    M, N, K = 16, 256, 256
    a = rs.randint(0, 0x7E, (M, K)).astype(np.uint8)
    b = rs.randint(0, 0x7E, (N, K)).astype(np.uint8) | (rs.randint(0, 2, (N, K)) * 0x80).astype(np.uint8)
    sfa = rs.uniform(0.8, 1.2, (K // 128, M)).astype(np.float32)
    sfb128 = rs.uniform(0.8, 1.2, (N // 128, K // 128)).astype(np.float32)
    sfb1 = rs.uniform(0.8, 1.2, (K // 128, N)).astype(np.float32)
    da, db = oracle.e4m3_decode(a).astype(np.float64), oracle.e4m3_decode(b).astype(np.float64)
    # independent numpy statement of gemm_ref (opus_gemm/block_scale_gemm/..._host.cc:66-90)
    exp128 = np.zeros((M, N))
    exp1 = np.zeros((M, N))
    for kg in range(K // 128):
        part = da[:, kg * 128:(kg + 1) * 128] @ db[:, kg * 128:(kg + 1) * 128].T
        exp128 += part * sfa[kg][:, None] * np.repeat(sfb128[:, kg], 128)[None, :]
        exp1 += part * sfa[kg][:, None] * sfb1[kg][None, :]
    c128 = oracle.gemm_blockscale(a, b, sfa, sfb128, M, N, K, M, K // 128, 128, 0)
    c1 = oracle.gemm_blockscale(a, b, sfa, sfb1, M, N, K, M, N, 1, 1)
    # fp32 running sums (the reference's loop) vs an f64 restatement
    assert oracle.check_f32(c128, exp128) < 1e-4
    assert oracle.check_f32(c1, exp1) < 1e-4
    f64 = oracle.gemm_blockscale_f64(a, b, sfa, sfb1, M, N, K, M, N, 1, 1)
    np.testing.assert_allclose(f64, exp1, rtol=1e-12, atol=1e-9)


def test_sf_tc_layout(oracle):
    rs = np.random.RandomState(2)
    rows, cols = 200, 9
    sf = rs.randint(1, 254, (rows, cols)).astype(np.uint8)
    tc = oracle.sf_to_tc_layout(sf)
    assert tc.size == 2 * 3 * 512
    for r in (0, 31, 32, 127, 128, 199):
        for c in (0, 3, 4, 8):
            off = ((r // 128) * 3 + c // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + c % 4
            assert tc[off] == sf[r, c]
    assert tc[(1 * 3 + 2) * 512 + (80 % 32) * 16 + 2 * 4 + 3] == 0x7F  # padded row 208, col 11


@pytest.mark.skipif(__import__("oracle.oracle", fromlist=["x"]).ref_lib() is None,
                    reason="oracle/_ref not built (reference tree absent)")
def test_against_live_reference(oracle):
    R = oracle.ref_lib()
    rs = np.random.RandomState(9)
    for N, Kp in ((16, 32), (64, 256), (32, 4096)):
        src = rs.randint(0, 256, N * Kp).astype(np.uint8)
        d = np.empty_like(src)
        R.ref_shuffle_weight_16x16(src, d, N, Kp)
        assert np.array_equal(d, oracle.shuffle_weight_16x16(src, N, Kp))
    for rows, cols in ((1, 1), (300, 32), (257, 13)):
        sm, sn = oracle.round_up(rows, 256), oracle.round_up(cols, 8)
        src = rs.randint(0, 256, rows * cols).astype(np.uint8)
        d = np.empty(sm * sn, np.uint8)
        R.ref_shuffle_scale(src, rows, cols, sm, sn, d)
        assert np.array_equal(d, oracle.shuffle_scale(src, rows, cols, sm, sn))


# ------------------------------------------------------------ opus gemm_ref loops, pinned
def _golden_opus_cases():
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "opus_gemm_ref_golden.npz")
    g = np.load(path)
    out = []
    for i, spec in enumerate(g["cases"]):
        loop, recipe, M, N, K, seed = str(spec).split("|")
        M, N, K = int(M), int(N), int(K)
        case = {"loop": loop, "M": M, "N": N, "K": K, "group_n": 1 if loop == "blockscale_1x128x1" else 128,
                "a": g[f"{i}_a"], "b": g[f"{i}_b"]}
        if loop.startswith("blockscale"):
            case["sfa"], case["sfb"] = g[f"{i}_sfa"], g[f"{i}_sfb"]
            case["stride_sfa"] = M
            case["stride_sfb"] = K // 128 if case["group_n"] == 128 else N
        out.append((f"{loop}|{recipe}", case, g[f"{i}_c"]))
    return out, g


def test_opus_oracle_matches_reference_golden(oracle):
    """orc_gemm_blockscale / _1x128x1 / orc_gemm_a8w8 / orc_gemm_a8w8_kn equal, bit for
    bit, the outputs of the reference's own gemm_ref loops (compiled from its
    sources by oracle/Makefile; fixtures from tests/golden/make_golden_opus.py)."""
    cases, _ = _golden_opus_cases()
    assert len(cases) == 10
    for name, case, ref in cases:
        got = oracle.run_opus_case(case, "oracle")
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name


def test_opus_e4m3_stand_in_matches_torch(oracle):
    """The stand-in for __hip_fp8_e4m3's conversion the reference loops were compiled
    with decodes like torch's float8_e4m3fn and the oracle's table."""
    _, g = _golden_opus_cases()
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    mine = oracle.e4m3_table()
    for table in (g["e4m3"], mine):
        assert np.array_equal(np.isnan(table), np.isnan(t))
        ok = ~np.isnan(t)
        assert np.array_equal(table[ok].view(np.uint32), t[ok].view(np.uint32))


@pytest.mark.skipif(__import__("oracle.oracle", fromlist=["x"]).opus_ref_lib() is None,
                    reason="oracle/_ref/libopus_ref.so not built (reference tree absent)")
@pytest.mark.parametrize("loop", ["blockscale", "blockscale_1x128x1", "fp8_gemm", "flatmm"])
def test_opus_oracle_matches_live_reference(oracle, loop):
    """The same pin against the live compiled reference on more shapes and seeds:
    ragged M, several K groups, each data recipe."""
    recipes = ["uniform", "bytes"] + (["normal"] if loop.startswith("blockscale") else [])
    for recipe in recipes:
        for (M, N, K), seed in (((1, 128, 128), 1), ((37, 256, 640), 2), ((64, 384, 1024), 3)):
            case = oracle.opus_case(loop, recipe, M, N, K, seed)
            got = oracle.run_opus_case(case, "oracle")
            ref = oracle.run_opus_case(case, "reference")
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (recipe, M, N, K)
