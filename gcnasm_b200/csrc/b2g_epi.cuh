// b2g_epi.cuh -- extra epilogue terms: D = alpha * acc + beta * C + bias[n].
//
// Order and rounding follow the reference: its CPU GEMM forms v = alpha * acc and
// then v += beta * C in fp32 (asm_f4gemm/f4gemm_ref.hpp:179-210); its split-K
// reduce adds a per-output-column bias in fp32 before the cast
// (opus_gemm_dist/opus_gemm_mem_gemm_a2a/include/gfx950/splitk_reduce_gfx950.cuh:49-60,
// bias [N] or [batch, N]).  Each step is one fp32 operation rounded to nearest;
// the cast to D's type comes last.  C and the bias have D's element type.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace b2g {

struct EpiTerms {
  const void* cin;  // C input at cin + b * cin_bstride + m * ldcin + n; null: no beta term
  long long ldcin, cin_bstride;
  float beta;
  const void* bias;  // bias at bias + b * bias_bstride + n; null: none
  long long bias_bstride;
};

__host__ __device__ __forceinline__ bool epi_any(const EpiTerms& e) { return e.cin != nullptr || e.bias != nullptr; }

// Four consecutive elements as fp32 (16-byte aligned for fp32, 8-byte for bf16).
// C may be the output itself: a plain load, read before the same thread (or its
// warp's TMA store) writes the element.
template <bool kF32>
__device__ __forceinline__ void epi_ld4(const void* base, long long i, float& a, float& b, float& c, float& d) {
  if (kF32) {
    const float4 t = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
    a = t.x; b = t.y; c = t.z; d = t.w;
  } else {
    // bf16 -> fp32 is exact: the 16 bits become the upper half of the fp32 word
    const uint2 t = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + i);
    a = __uint_as_float(t.x << 16);
    b = __uint_as_float(t.x & 0xFFFF0000u);
    c = __uint_as_float(t.y << 16);
    d = __uint_as_float(t.y & 0xFFFF0000u);
  }
}

// x[0..3] are columns n .. n+3 of row m, batch bi, already alpha * acc in fp32
template <bool kF32>
__device__ __forceinline__ void epi_apply4(const EpiTerms& e, int bi, long long m, long long n, float& x0, float& x1,
                                           float& x2, float& x3) {
  if (e.cin) {
    float c0, c1, c2, c3;
    epi_ld4<kF32>(e.cin, bi * e.cin_bstride + m * e.ldcin + n, c0, c1, c2, c3);
    x0 = __fadd_rn(x0, __fmul_rn(e.beta, c0));
    x1 = __fadd_rn(x1, __fmul_rn(e.beta, c1));
    x2 = __fadd_rn(x2, __fmul_rn(e.beta, c2));
    x3 = __fadd_rn(x3, __fmul_rn(e.beta, c3));
  }
  if (e.bias) {
    float b0, b1, b2, b3;
    epi_ld4<kF32>(e.bias, bi * e.bias_bstride + n, b0, b1, b2, b3);
    x0 = __fadd_rn(x0, b0);
    x1 = __fadd_rn(x1, b1);
    x2 = __fadd_rn(x2, b2);
    x3 = __fadd_rn(x3, b3);
  }
}

// one element, output type chosen at run time (the decode kernel's scalar stores)
__device__ __forceinline__ float epi_ld1(const void* base, long long i, bool f32) {
  return f32 ? static_cast<const float*>(base)[i] : __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}

__device__ __forceinline__ float epi_apply1(const EpiTerms& e, float v, long long m, long long n, bool f32) {
  if (e.cin) v = __fadd_rn(v, __fmul_rn(e.beta, epi_ld1(e.cin, m * e.ldcin + n, f32)));
  if (e.bias) v = __fadd_rn(v, epi_ld1(e.bias, n, f32));
  return v;
}

}  // namespace b2g
