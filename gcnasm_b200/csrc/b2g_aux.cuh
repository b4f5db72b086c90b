// b2g_aux.cuh -- memory-bound helper kernels around the GEMM:
//   * split-K reduce + cast (fp32 workspace -> bf16 / fp32 C)
//   * scale-factor layout conversion between the reference's f4gemm shuffled
//     layout, plain row-major UE8M0 and the sm_100 tensor-core atom layout
//   * the reference's 16x16 B preshuffle (and its inverse) on device
//   * MXFP8 / MXFP4 / 1x128 / 128x128 quantisers (fp32 or bf16 input for the MX and
//     1x128 forms; the data recipe of the benchmark configs)
// All of them are byte/integer work bound by HBM: grid-stride loops, 16-byte
// accesses where the layout allows, grids sized in multiples of the SM count.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "b2g_epi.cuh"

namespace b2g {

// ---------------------------------------------------------------------------
// split-K reduce: C[b][m][n] = cast(sum_s ws[s][b][m][n] + beta * Cin + bias[n])
// (opus_gemm_dist/opus_gemm_mem_gemm_a2a/include/gfx950/splitk_reduce_gfx950.cuh:68-259
//  sums the split slices of an fp32 workspace, adds the optional per-column bias in
//  fp32 and casts to D_OUT; N % 4 == 0 here).  Cin may be the output itself.
// ---------------------------------------------------------------------------
template <bool kOutF32>
__global__ void b2g_splitk_reduce_kernel(const float* __restrict__ ws, void* c, int S, int batch,
                                         int M, int N, long long ldc, long long c_bstride, EpiTerms epi) {
  const long long n4 = N / 4;
  const long long total = static_cast<long long>(batch) * M * n4;
  const long long slice = static_cast<long long>(batch) * M * N;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / n4;  // b * M + m
    const int col = static_cast<int>(i - row * n4) * 4;
    const float* src = ws + row * N + col;
    float4 acc = __ldg(reinterpret_cast<const float4*>(src));
    for (int s = 1; s < S; ++s) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + s * slice));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const int b = static_cast<int>(row / M);
    const int m = static_cast<int>(row - static_cast<long long>(b) * M);
    if (epi_any(epi)) epi_apply4<kOutF32>(epi, b, m, col, acc.x, acc.y, acc.z, acc.w);
    if (kOutF32) {
      float* dst = reinterpret_cast<float*>(c) + b * c_bstride + m * ldc + col;
      *reinterpret_cast<float4*>(dst) = acc;
    } else {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(c) + b * c_bstride + m * ldc + col;
      __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
      __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(dst) = pk;
    }
  }
}

// ---------------------------------------------------------------------------
// scale-factor layouts
//   tc atom layout: atoms of 128 rows x 4 scale columns (512 B), byte
//   (r%32)*16 + ((r/32)%4)*4 + (c%4); atoms [ceil(rows/128)][ceil(cols/4)].
// ---------------------------------------------------------------------------
__device__ __forceinline__ long long tc_atom_offset(int r, int c, int cb_n) {
  return (static_cast<long long>(r >> 7) * cb_n + (c >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
}

// plain row-major [rows, cols] (leading dim ld) -> tc layout; pad = 0x7F (1.0)
__global__ void b2g_sf_rowmajor_to_tc_kernel(const uint8_t* __restrict__ src, int rows, int cols, long long ld,
                                             uint8_t* __restrict__ dst) {
  const int rb_n = (rows + 127) / 128, cb_n = (cols + 3) / 4;
  const long long total = static_cast<long long>(rb_n) * cb_n * 512;
  for (long long o = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long atom = o >> 9;
    const int in = static_cast<int>(o & 511);
    const int rb = static_cast<int>(atom / cb_n), cb = static_cast<int>(atom - static_cast<long long>(rb) * cb_n);
    const int r = rb * 128 + (in >> 4) + ((in >> 2) & 3) * 32;
    const int c = cb * 4 + (in & 3);
    dst[o] = (r < rows && c < cols) ? src[static_cast<long long>(r) * ld + c] : uint8_t(0x7F);
  }
}

// f4gemm shuffled scales (asm_f4gemm/f4gemm_ref.hpp:101-130: padded [sm, sn],
// view(sm/32, 2, 16, sn/8, 2, 4).permute(0, 3, 5, 2, 4, 1)) -> tc layout for the
// first `rows` rows and `cols` columns.
__device__ __forceinline__ long long f4gemm_scale_offset(int r, int c, int sn) {
  const int d0 = r >> 5, d1 = (r >> 4) & 1, d2 = r & 15;
  const int d3 = c >> 3, d4 = (c >> 2) & 1, d5 = c & 3;
  return ((((static_cast<long long>(d0) * (sn >> 3) + d3) * 4 + d5) * 16 + d2) * 2 + d4) * 2 + d1;
}

__global__ void b2g_sf_f4gemm_to_tc_kernel(const uint8_t* __restrict__ src, int rows, int cols, int sn,
                                           uint8_t* __restrict__ dst) {
  const int rb_n = (rows + 127) / 128, cb_n = (cols + 3) / 4;
  const long long total = static_cast<long long>(rb_n) * cb_n * 512;
  for (long long o = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long atom = o >> 9;
    const int in = static_cast<int>(o & 511);
    const int rb = static_cast<int>(atom / cb_n), cb = static_cast<int>(atom - static_cast<long long>(rb) * cb_n);
    const int r = rb * 128 + (in >> 4) + ((in >> 2) & 3) * 32;
    const int c = cb * 4 + (in & 3);
    dst[o] = (r < rows && c < cols) ? src[f4gemm_scale_offset(r, c, sn)] : uint8_t(0x7F);
  }
}

// plain row-major [rows, cols] -> f4gemm shuffled layout [sm, sn] (pad 0x7F),
// the device form of asm_f4gemm/f4gemm_ref.hpp:108-130 (shuffle_scale).
__global__ void b2g_shuffle_scale_kernel(const uint8_t* __restrict__ src, int rows, int cols, int sm, int sn,
                                         uint8_t* __restrict__ dst) {
  const long long total = static_cast<long long>(sm) * sn;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / sn), c = static_cast<int>(i - static_cast<long long>(r) * sn);
    dst[f4gemm_scale_offset(r, c, sn)] = (r < rows && c < cols) ? src[static_cast<long long>(r) * cols + c] : uint8_t(0x7F);
  }
}

// ---------------------------------------------------------------------------
// 16x16 B preshuffle (asm_f4gemm/f4gemm_ref.hpp:78-96 on bytes; with one byte per
// E4M3 element it is also opus_fmm/flatmm_a8w8_gfx950.cc:638-681's layout):
// row n, 16-byte K chunk kc  <->  16-byte block ((n/16)*(Kp/16) + kc)*16 + n%16.
// ---------------------------------------------------------------------------
template <bool kInverse>
__global__ void b2g_shuffle_weight_16x16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int N,
                                                int kc_n /* Kp / 16 */) {
  const long long total = static_cast<long long>(N) * kc_n;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / kc_n), kc = static_cast<int>(i - static_cast<long long>(n) * kc_n);
    const long long shuf = (static_cast<long long>(n >> 4) * kc_n + kc) * 16 + (n & 15);
    if (kInverse) dst[i] = src[shuf];
    else dst[shuf] = src[i];
  }
}

// ---------------------------------------------------------------------------
// quantisers (bit-exact with oracle/b2g_oracle.c orc_quant_*)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint8_t f32_to_e4m3_sat(float x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(x));
  return static_cast<uint8_t>(r & 0xFF);
}

__device__ __forceinline__ uint32_t f32x4_to_e4m3x4_sat(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// smallest e with 2^e * 448 >= amax, biased and clamped to [1, 254]; 1 for amax == 0
__device__ __forceinline__ uint8_t mx_scale_byte(float amax) {
  if (!(amax > 0.f)) return 1;
  int ex;
  const float mant = frexpf(amax, &ex);
  int b = ((mant <= 0.875f) ? ex - 9 : ex - 8) + 127;
  b = b < 1 ? 1 : (b > 254 ? 254 : b);
  return static_cast<uint8_t>(b);
}

// MXFP4 element: round to nearest with ties to the even code onto the e2m1 grid
// {0, 0.5, 1, 1.5, 2, 3, 4, 6} (the midpoints are exact fp32 values), saturating
// at 6; sign from the sign bit of x; NaN -> 7 | sign.  Nibble code, bit 3 = sign.
__device__ __forceinline__ uint32_t f32_to_e2m1(float x) {
  const uint32_t sign = (__float_as_uint(x) >> 28) & 8u;
  const float a = fabsf(x);
  uint32_t c = (a <= 0.25f) ? 0u : (a < 0.75f) ? 1u : (a <= 1.25f) ? 2u : (a < 1.75f) ? 3u
             : (a <= 2.5f) ? 4u : (a < 3.5f) ? 5u : (a <= 5.0f) ? 6u : 7u;
  if (a != a) c = 7u;
  return sign | c;
}

// smallest e with 2^e * 6 >= amax (the MX scale rule with e2m1's largest value),
// biased and clamped to [1, 254]; 1 for amax == 0
__device__ __forceinline__ uint8_t mxfp4_scale_byte(float amax) {
  if (!(amax > 0.f)) return 1;
  int ex;
  const float mant = frexpf(amax, &ex);
  int b = ((mant <= 0.75f) ? ex - 3 : ex - 2) + 127;
  b = b < 1 ? 1 : (b > 254 ? 254 : b);
  return static_cast<uint8_t>(b);
}

// eight consecutive input elements as fp32 (bf16 widens exactly); 16-byte aligned
__device__ __forceinline__ void load8_f32(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8_f32(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 t = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = __uint_as_float(w[j] << 16);
    v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}

// MX quantiser (kFp4: MXFP4 packed e2m1, else MXFP8 E4M3): one thread per 8
// consecutive elements, 4 threads per 1x32 block.  K % 32 == 0.  q: E4M3 bytes
// [rows][ldq] or packed e2m1 (element 2i in the low nibble) [rows][ldq bytes].
// sf_tc (tc atom layout, may be null) and/or sf_rm (row-major [rows, K/32], may
// be null) receive the scales.
template <bool kFp4, typename In>
__global__ void b2g_quant_mx_kernel(const In* __restrict__ x, int rows, int K, long long ldx,
                                    uint8_t* __restrict__ q, long long ldq, uint8_t* __restrict__ sf_tc,
                                    uint8_t* __restrict__ sf_rm) {
  const int groups = K / 8;
  const long long total = static_cast<long long>(rows) * groups;
  const int cb_n = (K / 32 + 3) / 4;
  // the grid-stride step is a multiple of 4 so the 4 threads of a block stay in one warp
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i - (threadIdx.x & 31) < total; i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const bool live = i < total;
    const long long r = live ? i / groups : 0;
    const int g = live ? static_cast<int>(i - r * groups) : 0;
    float v[8];
    if (live) {
      load8_f32(x + r * ldx + g * 8, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    if (!live) continue;
    const uint8_t e = kFp4 ? mxfp4_scale_byte(amax) : mx_scale_byte(amax);
    const float inv = __int_as_float((254 - e) << 23);  // 2^(127 - e), exact
    if (kFp4) {
      uint32_t pk = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) pk |= f32_to_e2m1(v[j] * inv) << (4 * j);
      *reinterpret_cast<uint32_t*>(q + r * ldq + g * 4) = pk;
    } else {
      uint2 pk;
      pk.x = f32x4_to_e4m3x4_sat(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
      pk.y = f32x4_to_e4m3x4_sat(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
      *reinterpret_cast<uint2*>(q + r * ldq + g * 8) = pk;
    }
    if ((g & 3) == 0) {
      const int c = g >> 2;
      if (sf_tc) sf_tc[tc_atom_offset(static_cast<int>(r), c, cb_n)] = e;
      if (sf_rm) sf_rm[r * (K / 32) + c] = e;
    }
  }
}

// 1x128 (fp32 scale = amax/448 per 128 elements of a row): one warp per block;
// sf laid out [K/128, rows].
__device__ __forceinline__ float4 load4_f32(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 load4_f32(const __nv_bfloat16* p) {
  const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
  return make_float4(__uint_as_float(t.x << 16), __uint_as_float(t.x & 0xFFFF0000u), __uint_as_float(t.y << 16),
                     __uint_as_float(t.y & 0xFFFF0000u));
}

template <typename In>
__global__ void b2g_quant_1x128_kernel(const In* __restrict__ x, int rows, int K, uint8_t* __restrict__ q,
                                       float* __restrict__ sf) {
  const int nb = K / 128;
  const long long total = static_cast<long long>(rows) * nb;
  const int lane = threadIdx.x & 31;
  for (long long w = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5; w < total;
       w += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const long long r = w / nb;
    const int b = static_cast<int>(w - r * nb);
    const float4 v = load4_f32(x + r * K + b * 128 + lane * 4);
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = amax > 0.f ? __fdiv_rn(amax, 448.f) : 1.f;
    *reinterpret_cast<uint32_t*>(q + r * K + b * 128 + lane * 4) =
        f32x4_to_e4m3x4_sat(__fdiv_rn(v.x, s), __fdiv_rn(v.y, s), __fdiv_rn(v.z, s), __fdiv_rn(v.w, s));
    if (lane == 0) sf[static_cast<long long>(b) * rows + r] = s;
  }
}

// 128x128 (one fp32 scale per 128x128 tile of a [N, K] weight): one block of
// 256 threads per tile; sf laid out [N/128, K/128].
__global__ void b2g_quant_128x128_kernel(const float* __restrict__ x, int N, int K, uint8_t* __restrict__ q,
                                         float* __restrict__ sf) {
  __shared__ float red[8];
  const int nbk = K / 128;
  const int tiles = (N / 128) * nbk;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int bn = t / nbk, bk = t - bn * nbk;
    float amax = 0.f;
    for (int i = threadIdx.x; i < 128 * 32; i += blockDim.x) {
      const int rr = i >> 5, cc = (i & 31) * 4;
      const float4 v = __ldg(reinterpret_cast<const float4*>(x + static_cast<long long>(bn * 128 + rr) * K + bk * 128 + cc));
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int j = 1; j < static_cast<int>(blockDim.x >> 5); ++j) amax = fmaxf(amax, red[j]);
    const float s = amax > 0.f ? __fdiv_rn(amax, 448.f) : 1.f;
    for (int i = threadIdx.x; i < 128 * 32; i += blockDim.x) {
      const int rr = i >> 5, cc = (i & 31) * 4;
      const long long off = static_cast<long long>(bn * 128 + rr) * K + bk * 128 + cc;
      const float4 v = __ldg(reinterpret_cast<const float4*>(x + off));
      *reinterpret_cast<uint32_t*>(q + off) =
          f32x4_to_e4m3x4_sat(__fdiv_rn(v.x, s), __fdiv_rn(v.y, s), __fdiv_rn(v.z, s), __fdiv_rn(v.w, s));
    }
    if (threadIdx.x == 0) sf[t] = s;
    __syncthreads();
  }
}

}  // namespace b2g
