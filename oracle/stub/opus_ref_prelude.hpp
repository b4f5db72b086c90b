/*
 * Stand-ins for the two types the reference's opus gemm_ref loops use, so that
 * those loops compile with g++ exactly as written (oracle/extract_gemm_ref.py,
 * oracle/opus_ref_shim.cpp).  TEST INFRASTRUCTURE ONLY.
 *
 *   fp32_t      -- float (opus::fp32_t, and the hosts' `using fp32_t = float`).
 *   host_fp8_t  -- one byte of OCP E4M3 ("fn": bias 7, no infinities, S.1111.111
 *                  is NaN, largest finite 448), the format of gfx950's
 *                  __hip_fp8_e4m3 that the reference hosts alias it to; only its
 *                  conversion to float is needed.  The decode here builds the
 *                  fp32 bit pattern directly (normal numbers) or scales the
 *                  mantissa by 2^-9 (subnormals), independently of the oracle's
 *                  own table.
 */
#pragma once
#include <cstdint>
#include <cstring>

using fp32_t = float;

struct host_fp8_t {
  uint8_t bits;

  explicit operator float() const {
    const uint32_t sign = static_cast<uint32_t>(bits & 0x80u) << 24;
    const uint32_t exp = (bits >> 3) & 0xFu;
    const uint32_t man = bits & 0x7u;
    uint32_t u;
    if (exp == 0xFu && man == 0x7u) {
      u = sign | 0x7FC00000u;  // NaN
    } else if (exp == 0) {
      float f = static_cast<float>(man) * (1.0f / 512.0f);  // m * 2^-9, exact
      std::memcpy(&u, &f, 4);
      u |= sign;
    } else {
      u = sign | ((exp + 120u) << 23) | (man << 20);  // 2^(e-7) * (1 + m/8)
    }
    float out;
    std::memcpy(&out, &u, 4);
    return out;
  }
};
static_assert(sizeof(host_fp8_t) == 1, "host_fp8_t must be one byte");
