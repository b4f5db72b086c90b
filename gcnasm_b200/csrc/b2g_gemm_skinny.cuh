// b2g_gemm_skinny.cuh -- GEMM for few rows of A (M <= 128: decode / small batch).
//
//   C[m, n] = alpha * sum_k A[m, k] * B[n, k]          m < M <= 128, B = weights
//
// The product is computed transposed: the MMA's M = 128 runs over 128 rows of
// B (weights) and its N = MP (M rounded up to 16/32/64/128) over the rows of A,
// so no tensor-core rows are spent on padding.  The work -- (128-row B tile,
// 128-K block) units -- is split evenly over the persistent CTAs (stream-K):
// CTA c takes units [c*W/G, (c+1)*W/G), which may begin or end inside a B tile.
// Every contiguous run of units of one tile ("segment") accumulates in TMEM and
// is added to C (zeroed by the caller) with fp32 vector reductions; with at
// most two segments per tile the sum is order-independent.  Decode GEMMs are
// bound by streaming B from HBM, so the ring is deep (8 stages of 16 KB of B)
// and every SM streams an equal share of B.
// Modes: kModePlain (alpha only) and kModeMX (UE8M0 1x32 scales; the weights'
// scale atoms are the MMA's A scales, the activations' its B scales).
#pragma once

#include "b2g_gemm.cuh"

namespace b2g {

template <int kMode_, int kMP_, bool kBPre_>
struct SkinnyCfg {
  static constexpr int kMode = kMode_;
  static constexpr int kMP = kMP_;  // padded A rows = MMA N
  static constexpr bool kBPre = kBPre_;
  static constexpr int kThreads = 192;  // producer, MMA, 4 epilogue warps
  static constexpr int kWBytes = 128 * 128;         // one 128 x 128 B (weight) tile
  static constexpr int kABytes = kMP * 128;         // the A rows of one 128-K block
  static constexpr int kSfBytes = kMode == kModeMX ? 512 : 0;  // one atom each
  static constexpr int kStageBytes = kWBytes + kABytes + 2 * kSfBytes;
  static constexpr int kStages = kMP <= 32 ? 10 : (kMP == 64 ? 8 : 6);
  static constexpr int kAccStages = 2;
  static constexpr int kAccStride = kMP < 32 ? 32 : kMP;  // accumulator stages start 32-column aligned
  static constexpr int kSfCols = kMode == kModeMX ? 8 : 0;  // weight atom (4) + activation atom (4)
  static constexpr int kSfCol = kAccStages * kAccStride;     // two alternating scale sets follow
  static constexpr int kColsUsed = kSfCol + 2 * kSfCols;
  static constexpr int kTmemCols = kColsUsed <= 32 ? 32 : kColsUsed <= 64 ? 64 : kColsUsed <= 128 ? 128
                                   : kColsUsed <= 256 ? 256 : 512;

  static constexpr int kOffW = 0;
  static constexpr int kOffA = kOffW + kStages * kWBytes;
  static constexpr int kOffSfw = kOffA + kStages * kABytes;
  static constexpr int kOffSfa = kOffSfw + kStages * kSfBytes;
  static constexpr int kOffBar = (kOffSfa + kStages * kSfBytes + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2;
  static constexpr int kOffCtl = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffCtl + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kMP == 16 || kMP == 32 || kMP == 64 || kMP == 128, "padded M");
  static_assert(kABytes % 1024 == 0 || kMP == 16, "A stage alignment");
};

struct SkinnyParams {
  int M, N, K;
  float* c;          // fp32 [M][ldc], zeroed by the caller; partial sums are added
  long long ldc;
  float alpha;
  const uint8_t* sfw;  // weight (B) scales, tensor-core atom layout, atoms [n_block][k_block]
  const uint8_t* sfa;  // activation (A) scales, same layout (one row block)
  long long sf_rb;     // bytes between row blocks of either scale buffer
  int NT, KB;          // 128-row weight tiles, 128-K blocks
  long long units;     // NT * KB
  int* status;
  unsigned long long timeout_ns;
  int debug_stall;
};

// contiguous unit range of CTA `c` out of `g`
__device__ __forceinline__ void skinny_range(long long units, int c, int g, long long* lo, long long* hi) {
  *lo = units * c / g;
  *hi = units * (c + 1) / g;
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    b2g_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                           const __grid_constant__ SkinnyParams p) {
  constexpr int kMode = Cfg::kMode;
  constexpr int ST = Cfg::kStages;
  constexpr int AS = Cfg::kAccStages;
  constexpr int MP = Cfg::kMP;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* acc_full = bars + 2 * ST;
  uint64_t* acc_empty = bars + 2 * ST + AS;
  uint64_t* fin = bars + 2 * ST + 2 * AS;
  uint64_t* never = fin + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffCtl + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (kMode == kModeMX) {
    for (int i = threadIdx.x; i < ST * 2 * Cfg::kSfBytes / 4; i += Cfg::kThreads)
      reinterpret_cast<uint32_t*>(smem + Cfg::kOffSfw)[i] = 0x7F7F7F7Fu;
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < AS; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 4); }
    mbar_init(fin, 1);
    mbar_init(never, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc<Cfg::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint64_t tmo = p.timeout_ns;
  long long u_lo, u_hi;
  skinny_range(p.units, blockIdx.x, gridDim.x, &u_lo, &u_hi);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_a);
      int s = 0;
      uint32_t ph = 0, issued_mask = 0, issued_phase = 0;
      for (long long u = u_lo; u < u_hi; ++u) {
        const int nt = static_cast<int>(u / p.KB), kb = static_cast<int>(u - static_cast<long long>(nt) * p.KB);
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutProducer, tmo)) break;
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
        if (Cfg::kBPre)
          tma_load_4d(smem + Cfg::kOffW + s * Cfg::kWBytes, &tm_w, &full[s], 0, nt * 8, kb * 8, 0);
        else
          tma_load_3d(smem + Cfg::kOffW + s * Cfg::kWBytes, &tm_w, &full[s], kb * 128, nt * 128, 0);
        tma_load_3d(smem + Cfg::kOffA + s * Cfg::kABytes, &tm_a, &full[s], kb * 128, 0, 0);
        if (kMode == kModeMX) {
          bulk_load(smem + Cfg::kOffSfw + s * Cfg::kSfBytes, p.sfw + nt * p.sf_rb + kb * 512, 512, &full[s]);
          bulk_load(smem + Cfg::kOffSfa + s * Cfg::kSfBytes, p.sfa + kb * 512, 512, &full[s]);
        }
        issued_mask |= 1u << s;
        issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
        if (++s == ST) { s = 0; ph ^= 1; }
      }
      if (*abort_flag) {
        for (int i = 0; i < ST; ++i)
          if (issued_mask & (1u << i)) {
            volatile int no_abort = 0;
            mbar_wait(&full[i], (issued_phase >> i) & 1u, &no_abort, p.status, kDevTimeoutDrain, 100000000ull);
          }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, as = 0;
      uint32_t ph = 0, aph = 0, sfbuf = 0;
      bool ok = true;
      if (p.debug_stall) ok = mbar_wait(never, 0, abort_flag, p.status, kDevTimeoutMma, tmo);
      long long u = u_lo;
      while (ok && u < u_hi) {
        const int nt = static_cast<int>(u / p.KB);
        const long long seg_end = u_hi < static_cast<long long>(nt + 1) * p.KB ? u_hi : static_cast<long long>(nt + 1) * p.KB;
        if (!mbar_wait(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + as * Cfg::kAccStride;
        for (long long v = u; v < seg_end; ++v) {
          if (!mbar_wait(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_base = smem_u32(smem + Cfg::kOffW + s * Cfg::kWBytes);
          const uint32_t a_base = smem_u32(smem + Cfg::kOffA + s * Cfg::kABytes);
          const uint32_t sf_off = sfbuf * Cfg::kSfCols;
          sfbuf ^= 1;
          if (kMode == kModeMX) {
            tc_cp_32x128b_warpx4(tmem_base + Cfg::kSfCol + sf_off,
                                 desc_sf_atom(smem_u32(smem + Cfg::kOffSfw + s * Cfg::kSfBytes)));
            tc_cp_32x128b_warpx4(tmem_base + Cfg::kSfCol + sf_off + 4,
                                 desc_sf_atom(smem_u32(smem + Cfg::kOffSfa + s * Cfg::kSfBytes)));
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t wdesc = Cfg::kBPre ? desc_kmajor_interleave(w_base + kk * 2 * (128 * 16), 128 * 16)
                                              : desc_kmajor_sw128(w_base + kk * 32);
            const uint64_t adesc = desc_kmajor_sw128(a_base + kk * 32);
            const uint32_t acc = (v > u || kk > 0);
            if (kMode == kModeMX)
              mma_mxf8f6f4(d_tmem, wdesc, adesc, idesc_mxf8f6f4(128, MP, kk, kk), tmem_base + Cfg::kSfCol + sf_off,
                           tmem_base + Cfg::kSfCol + sf_off + 4, acc);
            else
              mma_f8f6f4(d_tmem, wdesc, adesc, idesc_f8f6f4(128, MP), acc);
          }
          tc_commit(&empty[s]);
          if (++s == ST) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit(&acc_full[as]);
        if (++as == AS) { as = 0; aph ^= 1; }
        u = seg_end;
      }
      tc_commit(fin);
      volatile int no_abort = 0;
      mbar_wait(fin, 0, &no_abort, p.status, kDevTimeoutDrain, 1000000000ull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue: 4 warps, one TMEM lane group each
    const int quad = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    int as = 0;
    uint32_t aph = 0;
    long long u = u_lo;
    while (u < u_hi) {
      const int nt = static_cast<int>(u / p.KB);
      const long long seg_end = u_hi < static_cast<long long>(nt + 1) * p.KB ? u_hi : static_cast<long long>(nt + 1) * p.KB;
      if (!mbar_wait(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo)) break;
      tc_fence_after();
      uint32_t v[MP];
      if (MP >= 32) {
#pragma unroll
        for (int c = 0; c < MP / 32; ++c)
          tmem_ld_32x32b_x32(tmem_base + lane_addr + as * Cfg::kAccStride + c * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      } else {
        tmem_ld_32x32b_x16(tmem_base + lane_addr + as * Cfg::kAccStride, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
      }
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[as]);
      if (++as == AS) { as = 0; aph ^= 1; }
      const int n = nt * 128 + quad * 32 + lane;  // this thread's weight row = output column
      if (n < p.N) {
        float* col = p.c + n;
#pragma unroll
        for (int m = 0; m < MP; ++m)
          if (m < p.M) atomicAdd(col + m * p.ldc, __uint_as_float(v[m]) * p.alpha);
      }
      u = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem_base);
  }
}

}  // namespace b2g
