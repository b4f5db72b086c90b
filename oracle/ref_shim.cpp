/*
 * ref_shim.cpp -- C entry points over the reference's own f4gemm host code,
 * compiled from the reference sources where they lie (asm_f4gemm/f4gemm_ref.hpp
 * and asm_f4gemm/f4gemm.hpp) into oracle/_ref/libf4gemm_ref.so.
 *
 * TEST INFRASTRUCTURE ONLY: the parity tests and tests/golden/make_golden.py
 * use it to pin the oracle restatement and the product's host logic against
 * the real reference.  Nothing here is part of the product library.
 */
#include "f4gemm.hpp"
#include "f4gemm_ref.hpp"

#include <cstring>
#include <vector>

using namespace f4gemm;

extern "C" {

float ref_e8m0_to_f32(uint8_t e) { return e8m0_to_f32(e); }

void ref_shuffle_weight_16x16(const uint8_t* src, uint8_t* dst, int N, int Kp)
{
    std::vector<uint8_t> s(src, src + (size_t)N * Kp);
    std::vector<uint8_t> d = shuffle_weight_16x16(s, N, Kp);
    memcpy(dst, d.data(), d.size());
}

void ref_shuffle_scale(const uint8_t* src, int rows, int cols, int sm, int sn, uint8_t* dst)
{
    std::vector<uint8_t> s(src, src + (size_t)rows * cols);
    std::vector<uint8_t> d = shuffle_scale(s, rows, cols, sm, sn);
    memcpy(dst, d.data(), d.size());
}

/* Shape helpers, f4gemm_ref.hpp:61-73 */
void ref_shape(int M, int N, int K, int* out7)
{
    Shape sh{M, N, K};
    out7[0] = sh.Kp(); out7[1] = sh.Ks(); out7[2] = sh.scale_cols(); out7[3] = sh.a_rows_pad();
    out7[4] = sh.b_rows_pad(); out7[5] = sh.scale_a_rows(); out7[6] = sh.d_rows_pad();
}

/* make_operand, f4gemm_ref.hpp:145-176 */
void ref_make_operand(int rows, int K, uint32_t seed, uint8_t* packed, uint8_t* scales, float* dequant)
{
    Operand op = make_operand(rows, K, seed);
    memcpy(packed, op.packed.data(), op.packed.size());
    memcpy(scales, op.scales.data(), op.scales.size());
    memcpy(dequant, op.dequant.data(), op.dequant.size() * sizeof(float));
}

/* reference_gemm, f4gemm_ref.hpp:181-222 (beta = 0, no C) */
void ref_reference_gemm(const float* A, const float* B, int M, int N, int K, float alpha, float* D)
{
    std::vector<float> a(A, A + (size_t)M * K), b(B, B + (size_t)N * K);
    std::vector<float> d = reference_gemm(a, b, M, N, K, alpha, {}, 0.0f);
    memcpy(D, d.data(), d.size() * sizeof(float));
}

/* select_kernel, f4gemm.hpp:210-267, over a manifest given as parallel arrays */
void ref_select_kernel(int M, int N, int K, int num_cu, int log2_k_split, int bpreshuffle,
                       int ncfg, const int* tile_m, const int* tile_n, const int* splitk, const int* bps,
                       int* out_idx, int* out_log2)
{
    std::vector<Config> cfgs(ncfg);
    for (int i = 0; i < ncfg; ++i) {
        cfgs[i].tile_M = tile_m[i]; cfgs[i].tile_N = tile_n[i];
        cfgs[i].splitK = splitk[i]; cfgs[i].bpreshuffle = bps[i];
        cfgs[i].knl_name = "k" + std::to_string(i); cfgs[i].co_name = "k" + std::to_string(i) + ".co";
    }
    auto r = select_kernel(M, N, K, num_cu, log2_k_split, bpreshuffle, cfgs);
    *out_idx = r.first;
    *out_log2 = r.second;
}

/* make_launch, f4gemm.hpp:329-349.  Returns 0, or 1 when the reference would exit
 * (K % (1 << log2_k_split) != 0); out5 = gdx, gdy, gdz, log2_k_split, zero_out. */
int ref_make_launch(int tile_m, int tile_n, int splitk, int M, int N, int K, int log2_k_split, int* out5)
{
    if (splitk == 1 && K % (1 << log2_k_split) != 0) return 1;
    Config c; c.tile_M = tile_m; c.tile_N = tile_n; c.splitK = splitk;
    LaunchDesc d = make_launch(c, M, N, K, log2_k_split);
    out5[0] = d.gdx; out5[1] = d.gdy; out5[2] = d.gdz; out5[3] = d.log2_k_split; out5[4] = d.zero_out ? 1 : 0;
    return 0;
}

/* fill_args, f4gemm.hpp:355-392: the packed 0x174-byte kernarg block */
int ref_kernel_args_size(void) { return (int)sizeof(KernelArgs); }

void ref_fill_args(void* out, void* d_D, void* d_C, void* d_A, void* d_B, void* d_SA, void* d_SB,
                   int M, int N, int K, int stride_D0, int stride_SA0, int stride_SB0,
                   float alpha, float beta, int log2_k_split)
{
    KernelArgs a;
    fill_args(a, d_D, d_C, d_A, d_B, d_SA, d_SB, M, N, K, stride_D0, stride_SA0, stride_SB0,
              alpha, beta, log2_k_split);
    memcpy(out, &a, sizeof(a));
}

/* load_configs, f4gemm.hpp:141-200 (exits the process on a missing file, like the reference) */
int ref_load_configs(const char* path, int cap, int* tile_m, int* tile_n, int* splitk, int* bps)
{
    std::vector<Config> c = load_configs(path);
    int n = (int)c.size();
    for (int i = 0; i < n && i < cap; ++i) {
        tile_m[i] = c[i].tile_M; tile_n[i] = c[i].tile_N; splitk[i] = c[i].splitK; bps[i] = c[i].bpreshuffle;
    }
    return n;
}

} // extern "C"
