// b2g_gemm_skinny_blk.cuh -- fp32 block-scaled FP8 GEMM for few rows of A (M <= 128).
//
//   C[m, n] = alpha * sum_kb sfa[kb][m] * sfb(n, kb) * sum_{k in kb} A[m, k] * B[n, k]
//
// sfa: one fp32 scale per row of A and 128-K block ([K/128][stride_sfa]); sfb: one
// per 128x128 block of B (GROUP_N = 128, [N/128][stride_sfb]) or per column of C and
// 128-K block (GROUP_N = 1, [K/128][stride_sfb]) -- the opus block_scale_gemm /
// block_scale_1x128x1_gemm semantics (scale_c_tile applied once per 128-K block).
//
// The split of the work is the skinny kernel's (b2g_gemm_skinny.cuh): MMA M = 128
// weight rows, N = MP activation rows, stream-K over (tile, K group) units, split
// tiles completed in-kernel by the right fold of their pieces.  What differs: each
// 128-K block is MMA'd into its own TMEM buffer (four of them, so the MMAs run up to
// three blocks ahead) and the epilogue warps fold it into fp32 registers with that
// block's scales, so a segment's sum lives in registers, not TMEM.  The producer
// thread also fetches every K block's scales (TMA boxes of the fp32 scale arrays)
// into a 16-slot ring with its own full / empty barriers, so the scales are in
// shared memory before the block's accumulator is, and no epilogue thread loads
// them.  Needs 16-byte aligned scale rows (stride_sfa % 4 == 0, and for 128x128
// blocks stride_sfb % 4 == 0); the host routes other layouts to the single-CTA kernel.
#pragma once

#include "b2g_gemm_skinny.cuh"

namespace b2g {

// kNT ("not transposed"): the MMA's M = 128 runs over the rows of A (MP = 128, rows
// past M read as zero) and its N = 128 over the tile's weight rows, so a TMEM lane
// is a row of C and a column a column of C.  With 128 x 128 weight scales the
// promotion then needs one scale product per thread and K block (sfa of its row
// times the tile's block scale) instead of one per column; C rows are written by
// their own thread and the split-tile pieces are row-major.
template <int kMP_, int kKB_, bool kNT_ = false>
struct SkinnyBlkCfg {
  static constexpr bool kNT = kNT_;
  static constexpr int kMP = kMP_;  // padded A rows = MMA N (kNT: MMA M)
  static constexpr int kKB = kKB_;  // 128-K blocks per stage
  // producer, MMA, then 4 epilogue warps (one per TMEM lane group).  Untransposed:
  // 12 warps -- warpgroup 0 (producer, MMA issuer, two idle warps) at 56 registers
  // and 8 epilogue warps, two per lane group, each folding 64 of the tile's 128
  // columns, at 224 (setmaxnreg; 128 * 56 + 256 * 224 = 384 * 168, the launch's total)
  static constexpr int kEpiThreads = kNT_ ? 256 : 128;
  static constexpr int kFirstEpiWarp = kNT_ ? 4 : 2;
  static constexpr int kThreads = 32 * kFirstEpiWarp + kEpiThreads;
  static constexpr int kNAcc = kNT_ ? 64 : kMP_;  // fp32 sums per epilogue thread
  static constexpr int kWBlk = 128 * 128;
  static constexpr int kABlk = kMP * 128;
  static constexpr int kWBytes = kKB * kWBlk;
  static constexpr int kABytes = kKB * kABlk;
  static constexpr int kStageBytes = kWBytes + kABytes;
  // scale ring: per K block, sfa of the MP rows | sfb: the tile's 128 column scales
  // (GROUP_N = 1) or the 8 block scales around this K block (GROUP_N = 128)
  static constexpr int kScaleDepth = 16;  // >= stages * K blocks per stage: never throttles the producer
  static constexpr int kSaFloats = (kMP + 31) / 32 * 32;  // TMA destinations start on 128 bytes
  static constexpr int kScaleSlot = kSaFloats + 128;       // floats
  static constexpr int kScaleBytes = kScaleDepth * kScaleSlot * 4;
  static constexpr int kMaxStages = kKB == 1 ? 8 : 5;
  static constexpr int kFit = (222000 - kScaleBytes) / kStageBytes;
  static constexpr int kStages = kFit < kMaxStages ? kFit : kMaxStages;
  static constexpr int kAccStages = 4;
  static constexpr int kAccStride = kMP < 32 ? 32 : kMP;
  static constexpr int kColsUsed = kAccStages * kAccStride;
  static constexpr int kTmemCols = kColsUsed <= 128 ? 128 : kColsUsed <= 256 ? 256 : 512;

  static constexpr int kOffW = 0;
  static constexpr int kOffA = kOffW + kStages * kWBytes;
  static constexpr int kOffScale = kOffA + kStages * kABytes;
  static constexpr int kOffBar = (kOffScale + kScaleBytes + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2 + 2 * kScaleDepth;
  static constexpr int kOffCtl = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffCtl + 16 + 1024;
  static_assert(kStages >= 3, "ring depth");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kMP == 16 || kMP == 32 || kMP == 64 || kMP == 128, "padded M");
  static_assert(kKB == 1 || kKB == 2, "K blocks per stage");
  static_assert(kColsUsed <= 512, "TMEM columns");
  static_assert(kStages * kKB <= kScaleDepth, "the first ring fill needs no free scale slot");
  static_assert(kOffScale % 128 == 0 && (kScaleSlot * 4) % 128 == 0 && (kSaFloats * 4) % 128 == 0,
                "every scale TMA box lands on a 128-byte boundary");
  static_assert(!kNT || (kMP == 128 && kKB == 1), "the untransposed form takes 128 A rows, one K block per stage");
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    b2g_gemm_skinny_blk_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                               const __grid_constant__ CUtensorMap tm_sa, const __grid_constant__ CUtensorMap tm_sb,
                               const __grid_constant__ SkinnyParams p) {
  constexpr int ST = Cfg::kStages;
  constexpr int AS = Cfg::kAccStages;
  constexpr int MP = Cfg::kMP;
  constexpr int KBS = Cfg::kKB;
  constexpr int SD = Cfg::kScaleDepth;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* acc_full = bars + 2 * ST;
  uint64_t* acc_empty = bars + 2 * ST + AS;
  uint64_t* fin = bars + 2 * ST + 2 * AS;
  uint64_t* never = fin + 1;
  uint64_t* sfull = never + 1;
  uint64_t* sempty = sfull + SD;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffCtl + 4);
  volatile uint32_t* last_flag = reinterpret_cast<volatile uint32_t*>(smem + Cfg::kOffCtl + 8);
  float* sring = reinterpret_cast<float*>(smem + Cfg::kOffScale);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const long long U = p.units;
  const int G = gridDim.x;
  const long long u_lo = U * blockIdx.x / G, u_hi = U * (blockIdx.x + 1) / G;
  const uint64_t tmo = p.timeout_ns;

  // One stage: B tile(s) (read once: evict first) and the A rows of kKB K blocks;
  // then each of those K blocks' scales into its scale slot (K block q of this CTA
  // -> slot q % SD, reused once the epilogue has released it).
  const bool gn1 = p.group_n == 1;
  const uint32_t scale_bytes = MP * 4 + (gn1 ? 512 : 32);
  const uint64_t pol_w = l2_policy_evict_first();
  uint32_t sq_mask = 0, sq_phase = 0;  // scale slots issued, parity of their latest fill
  auto issue = [&](long long u, int s) -> bool {
    const int nt = static_cast<int>(u / p.KG);
    const int kb = static_cast<int>(u - static_cast<long long>(nt) * p.KG) * KBS;
    mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
    tma_load_3d_hint(smem + Cfg::kOffW + s * Cfg::kWBytes, &tm_w, &full[s], 0, nt * 128, kb, pol_w);
    tma_load_3d(smem + Cfg::kOffA + s * Cfg::kABytes, &tm_a, &full[s], 0, 0, kb);
#pragma unroll
    for (int j = 0; j < KBS; ++j) {
      const long long q = (u - u_lo) * KBS + j;
      const int slot = static_cast<int>(q % SD);
      const uint32_t round = static_cast<uint32_t>(q / SD);
      if (round > 0 &&
          !mbar_wait(&sempty[slot], (round - 1) & 1u, abort_flag, p.status, kDevTimeoutProducer, tmo))
        return false;
      float* dst = sring + slot * Cfg::kScaleSlot;
      mbar_arrive_expect_tx(&sfull[slot], scale_bytes);
      tma_load_2d(dst, &tm_sa, &sfull[slot], 0, kb + j);
      if (gn1)
        tma_load_2d(dst + Cfg::kSaFloats, &tm_sb, &sfull[slot], nt * 128, kb + j);
      else
        tma_load_2d(dst + Cfg::kSaFloats, &tm_sb, &sfull[slot], (kb + j) & ~3, nt);
      sq_mask |= 1u << slot;
      sq_phase = (sq_phase & ~(1u << slot)) | ((round & 1u) << slot);
    }
    return true;
  };

  const int pre = static_cast<int>(u_hi - u_lo < ST ? u_hi - u_lo : ST);
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    constexpr int kEpiWarps = Cfg::kEpiThreads / 32;
    for (int s = 0; s < AS; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], kEpiWarps); }
    for (int s = 0; s < SD; ++s) { mbar_init(&sfull[s], 1); mbar_init(&sempty[s], kEpiWarps); }
    mbar_init(fin, 1);
    mbar_init(never, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_sa);
    tma_prefetch_desc(&tm_sb);
    griddep_wait();  // launched as a programmatic dependent: the previous kernel's writes are visible after this
    for (int i = 0; i < pre; ++i) issue(u_lo + i, i);
  }
  if (warp == 1) tmem_alloc<Cfg::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if constexpr (Cfg::kNT) setmaxnreg_dec<56>();
    if (lane == 0) {
      int s = pre % ST;
      uint32_t ph = pre == ST ? 1u : 0u;
      uint32_t issued_mask = pre == ST ? (1u << ST) - 1u : (1u << pre) - 1u, issued_phase = 0;
      for (long long u = u_lo + pre; u < u_hi; ++u) {
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutProducer, tmo)) break;
        issued_mask |= 1u << s;
        issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
        const bool ok = issue(u, s);
        if (++s == ST) { s = 0; ph ^= 1; }
        if (!ok) break;
      }
      if (*abort_flag) {  // every copy in flight lands before the CTA retires
        volatile int no_abort = 0;
        for (int i = 0; i < ST; ++i)
          if (issued_mask & (1u << i))
            mbar_wait(&full[i], (issued_phase >> i) & 1u, &no_abort, p.status, kDevTimeoutDrain, 100000000ull);
        for (int i = 0; i < SD; ++i)
          if (sq_mask & (1u << i))
            mbar_wait(&sfull[i], (sq_phase >> i) & 1u, &no_abort, p.status, kDevTimeoutDrain, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer: one TMEM buffer per K block
    if constexpr (Cfg::kNT) setmaxnreg_dec<56>();
    if (lane == 0) {
      int s = 0, as = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      if (p.debug_stall) ok = mbar_wait(never, 0, abort_flag, p.status, kDevTimeoutMma, tmo);
      for (long long u = u_lo; ok && u < u_hi; ++u) {
        if (!mbar_wait(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < KBS; ++j) {
          if (!mbar_wait(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_base = smem_u32(smem + Cfg::kOffW + s * Cfg::kWBytes + j * Cfg::kWBlk);
          const uint32_t a_base = smem_u32(smem + Cfg::kOffA + s * Cfg::kABytes + j * Cfg::kABlk);
          const uint32_t d_tmem = tmem_base + as * Cfg::kAccStride;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if constexpr (Cfg::kNT)  // rows of A x weight rows
              mma_f8f6f4(d_tmem, desc_kmajor_sw128(a_base + kk * 32), desc_kmajor_sw128(w_base + kk * 32),
                         idesc_f8f6f4(128, 128), kk > 0 ? 1u : 0u);
            else  // weight rows x rows of A
              mma_f8f6f4(d_tmem, desc_kmajor_sw128(w_base + kk * 32), desc_kmajor_sw128(a_base + kk * 32),
                         idesc_f8f6f4(128, MP), kk > 0 ? 1u : 0u);
          }
          tc_commit(&acc_full[as]);
          if (++as == AS) { as = 0; aph ^= 1; }
        }
        if (!ok) break;
        tc_commit(&empty[s]);
        if (++s == ST) { s = 0; ph ^= 1; }
      }
      tc_commit(fin);
      volatile int no_abort = 0;
      mbar_wait(fin, 0, &no_abort, p.status, kDevTimeoutDrain, 1000000000ull);
    }
    __syncwarp();
  } else if (warp < Cfg::kFirstEpiWarp) {
    // ------------------------------------------------------------ idle (kNT: the rest of warpgroup 0)
    if constexpr (Cfg::kNT) setmaxnreg_dec<56>();
  } else {
    // ------------------------------------------------------------ epilogue: 4 warps, one TMEM lane group each
    if constexpr (Cfg::kNT) setmaxnreg_inc<224>();
    constexpr int CH = MP < 32 ? MP : 32;
    const int quad = warp & 3;
    // TMEM lane: a weight row of the tile = a column of C (kNT: a row of A = a row of C)
    const int r = quad * 32 + lane;
    const int ch0 = Cfg::kNT ? ((warp - Cfg::kFirstEpiWarp) >> 2) * Cfg::kNAcc : 0;  // kNT: first column
    const int et = threadIdx.x - 32 * Cfg::kFirstEpiWarp;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const int cta = static_cast<int>(blockIdx.x);
    int as = 0;
    uint32_t aph = 0;
    long long q = 0;  // K blocks folded so far
    bool ok = true;
    long long u = u_lo;
    while (ok && u < u_hi) {
      const int nt = static_cast<int>(u / p.KG);
      const long long t0 = static_cast<long long>(nt) * p.KG;
      const long long seg_end = u_hi < t0 + p.KG ? u_hi : t0 + p.KG;
      const int c0 = skinny_owner(t0, U, G), c1 = skinny_owner(t0 + p.KG - 1, U, G);
      const int nseg = c1 - c0 + 1;
      const int j = cta - c0;
      const bool fin_seg = seg_end == u_hi;
      unsigned long long* cnt = p.cnt + nt;
      const unsigned long long all_others = (p.tag << 16) | static_cast<unsigned long long>(nseg - 1);
      auto slot_base = [&](int jj) {
        return p.part + static_cast<long long>(skinny_slot(c0 + jj, nt, U, G, p.KG)) * MP * 128;
      };
      // this thread's part of piece jj: column r, stride 128 per row of A (kNT: row r of a
      // column-major piece, stride 128 per column, so a warp's 32 rows are one 128-byte run)
      auto piece = [&](int jj) { return slot_base(jj) + (Cfg::kNT ? ch0 * 128 + r : r); };
      if (nseg > 1 && fin_seg && et < nseg && et != j) bulk_prefetch_l2(slot_base(et), MP * 128 * 4);

      // ---- fold the segment's K blocks into registers
      float acc[Cfg::kNAcc];
#pragma unroll
      for (int m = 0; m < Cfg::kNAcc; ++m) acc[m] = 0.f;
      const long long q_end = q + (seg_end - u) * KBS;
      int kb = static_cast<int>(u - t0) * KBS;  // K block within the tile
      for (; q < q_end; ++q, ++kb) {
        const int sslot = static_cast<int>(q % SD);
        const float* slot = sring + sslot * Cfg::kScaleSlot;
        bool got = mbar_wait(&sfull[sslot], static_cast<uint32_t>(q / SD) & 1u, abort_flag, p.status,
                             kDevTimeoutEpilogue, tmo);
        got = got && mbar_wait(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo);
        // each warp decides alone per K block (a wait that gives up raises the CTA's
        // abort flag, so every other warp's next wait returns at once); the warps
        // agree once per segment, before the fix-up's named barriers
        if (!got) { ok = false; break; }
        const float sbc = gn1 ? slot[Cfg::kSaFloats + r] : slot[Cfg::kSaFloats + (kb & 3)];
        tc_fence_after();
        const uint32_t acc_addr = tmem_base + lane_addr + as * Cfg::kAccStride;
        if constexpr (Cfg::kNT) {  // row r of the tile: scale sfa[r] (x the block scale, or the column's)
          const float sar = slot[r];
          const float s_row = sar * slot[Cfg::kSaFloats + (kb & 3)];
#pragma unroll
          for (int mc = 0; mc < Cfg::kNAcc; mc += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(acc_addr + ch0 + mc, v);
            tc_wait_ld();
            if (gn1) {  // (P * sfb[n]) * sfa[m] + acc
#pragma unroll
              for (int i = 0; i < 32; ++i)
                acc[mc + i] = fmaf(__uint_as_float(v[i]) * slot[Cfg::kSaFloats + ch0 + mc + i], sar, acc[mc + i]);
            } else {    // P * (sfa[m] * sfb) + acc
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[mc + i] = fmaf(__uint_as_float(v[i]), s_row, acc[mc + i]);
            }
          }
        } else {
#pragma unroll
        for (int mc = 0; mc < MP; mc += CH) {
          uint32_t v[CH];
          if (CH == 32)
            tmem_ld_32x32b_x32(acc_addr + mc, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          else
            tmem_ld_32x32b_x16(acc_addr + mc, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
          tc_wait_ld();
          if (gn1) {  // (P * sfb[n]) * sfa[m] + acc, as the single-CTA kernel rounds it
#pragma unroll
            for (int i = 0; i < CH; ++i)
              acc[mc + i] = fmaf(__uint_as_float(v[i]) * sbc, slot[mc + i], acc[mc + i]);
          } else {    // P * (sfa[m] * sfb) + acc
#pragma unroll
            for (int i = 0; i < CH; ++i)
              acc[mc + i] = fmaf(__uint_as_float(v[i]), slot[mc + i] * sbc, acc[mc + i]);
          }
        }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acc_empty[as]);
          mbar_arrive(&sempty[sslot]);
        }
        if (++as == AS) { as = 0; aph ^= 1; }
      }
      if (!skinny_epi_all<Cfg::kEpiThreads>(ok)) break;

      // ---- complete the tile: direct store, or the skinny kernel's right fold of the pieces
      const int n = nt * 128 + r;
      const bool col_ok = n < p.N;
      // kNT: columns [mc, mc + 32) of row r of the tile, 16-byte stores (N and the row
      // pitch are whole 16 bytes, so a 4- or 8-column group is all in or all out)
      auto store_row = [&](int mc, const float (&x)[32]) {
        if (r >= p.M) return;
        const int n0 = nt * 128 + ch0 + mc;
        if (p.out_f32) {
          float* row = static_cast<float*>(p.out) + static_cast<long long>(r) * p.ldo + n0;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            if (n0 + i < p.N)
              st_global_v4(row + i, __float_as_uint(x[i] * p.alpha), __float_as_uint(x[i + 1] * p.alpha),
                           __float_as_uint(x[i + 2] * p.alpha), __float_as_uint(x[i + 3] * p.alpha));
        } else {
          __nv_bfloat16* row = static_cast<__nv_bfloat16*>(p.out) + static_cast<long long>(r) * p.ldo + n0;
#pragma unroll
          for (int i = 0; i < 32; i += 8)
            if (n0 + i < p.N)
              st_global_v4(row + i, pack_bf16x2(x[i] * p.alpha, x[i + 1] * p.alpha),
                           pack_bf16x2(x[i + 2] * p.alpha, x[i + 3] * p.alpha),
                           pack_bf16x2(x[i + 4] * p.alpha, x[i + 5] * p.alpha),
                           pack_bf16x2(x[i + 6] * p.alpha, x[i + 7] * p.alpha));
        }
      };
      auto store_out = [&](int mc, const float (&x)[CH]) {
        if (!col_ok) return;
        if (p.out_f32) {
          float* col = static_cast<float*>(p.out) + n;
#pragma unroll
          for (int i = 0; i < CH; ++i)
            if (mc + i < p.M) col[(mc + i) * p.ldo] = x[i] * p.alpha;
        } else {
          __nv_bfloat16* col = static_cast<__nv_bfloat16*>(p.out) + n;
#pragma unroll
          for (int i = 0; i < CH; ++i)
            if (mc + i < p.M) col[(mc + i) * p.ldo] = __float2bfloat16_rn(x[i] * p.alpha);
        }
      };
      if (nseg == 1) {
        if constexpr (Cfg::kNT) {
#pragma unroll
          for (int mc = 0; mc < Cfg::kNAcc; mc += 32) {
            float x[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) x[i] = acc[mc + i];
            store_row(mc, x);
          }
        } else {
#pragma unroll
          for (int mc = 0; mc < MP; mc += CH) {
            float x[CH];
#pragma unroll
            for (int i = 0; i < CH; ++i) x[i] = acc[mc + i];
            store_out(mc, x);
          }
        }
      } else {
        bool last = false;
        if (fin_seg) {  // the tile's other pieces usually finished long ago
          if (et == 0) *last_flag = ld_acquire_gpu_u64(cnt) == all_others ? 1u : 0u;
          skinny_epi_bar<Cfg::kEpiThreads>();
          last = *last_flag != 0;
          skinny_epi_bar<Cfg::kEpiThreads>();  // every thread has read the flag before it is written again
        }
        if (!last) {
          float* mine = piece(j);
          if constexpr (Cfg::kNT) {
#pragma unroll
            for (int i = 0; i < Cfg::kNAcc; ++i)
              if (r < p.M) __stcg(mine + i * 128, acc[i]);  // rows past M hold zeros: never read
          } else {
#pragma unroll
            for (int m = 0; m < MP; ++m) __stcg(mine + m * 128, acc[m]);
          }
          skinny_epi_bar<Cfg::kEpiThreads>();
          if (et == 0) {
            fence_acq_rel_gpu();
            const int arrivals = skinny_arrive(cnt, p.tag, fin_seg ? nseg - 1 : 0, p.status);
            const bool done = arrivals == nseg;
            if (done) fence_acq_rel_gpu();
            *last_flag = done ? 1u : 0u;
          }
          skinny_epi_bar<Cfg::kEpiThreads>();
          last = *last_flag != 0;
          skinny_epi_bar<Cfg::kEpiThreads>();
        }
        if (last) {
          // p_0 + (p_1 + (... + p_{n-1})), this CTA's piece from registers
          if constexpr (Cfg::kNT) {
#pragma unroll
            for (int mc = 0; mc < Cfg::kNAcc; mc += 32) {
              float t[32];
              for (int jj = nseg - 1; jj >= 0; --jj) {
                float y[32];
                if (jj == j) {
#pragma unroll
                  for (int i = 0; i < 32; ++i) y[i] = acc[mc + i];
                } else {
                  const float* pj = piece(jj) + mc * 128;
#pragma unroll
                  for (int i = 0; i < 32; ++i) y[i] = r < p.M ? __ldcg(pj + i * 128) : 0.f;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) t[i] = jj == nseg - 1 ? y[i] : y[i] + t[i];
              }
              store_row(mc, t);
            }
          } else {
#pragma unroll
            for (int mc = 0; mc < MP; mc += CH) {
              float t[CH];
              for (int jj = nseg - 1; jj >= 0; --jj) {
                float y[CH];
                if (jj == j) {
#pragma unroll
                  for (int i = 0; i < CH; ++i) y[i] = acc[mc + i];
                } else {
                  const float* pj = piece(jj) + mc * 128;
#pragma unroll
                  for (int i = 0; i < CH; ++i) y[i] = __ldcg(pj + i * 128);
                }
#pragma unroll
                for (int i = 0; i < CH; ++i) t[i] = jj == nseg - 1 ? y[i] : y[i] + t[i];
              }
              store_out(mc, t);
            }
          }
          if (et == 0) *reinterpret_cast<volatile unsigned long long*>(cnt) = 0ull;
        }
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
