// b2g_gemm_pair.cuh -- CTA-pair (cluster of 2) variant of the persistent FP8 GEMM.
//
// Tile 256 x BN x 128 per pair (BN = 256; 192 also compiles, with two MX
// accumulator stages and seven operand stages, but measured 15 % slower at 8192^3);
// tcgen05.mma.cta_group::2 with M = 256: CTA r of the pair holds A rows
// [r*128, r*128 + 128) and B rows [r*BN/2, (r+1)*BN/2) of the tile in its own
// shared memory and receives the 128 x BN accumulator of its A rows in its own
// TMEM.  At BN = 256 that is 32 KB of operands per SM and 128-K block for
// 128 x 256 x 128 MACs, two thirds of the 48 KB the single-CTA 128 x 256 tile
// needs, which lets the ring hold 6 stages.
//
// Warps: 0 TMA producer, 1 MMA issuer (TMEM allocation), 2-9 epilogue (two
// column halves x four TMEM lane quarters), 10 scale warp (MX kinds only).
//
// Protocol (leader = cluster rank 0):
//   * both CTAs allocate TMEM with cta_group::2 and free it after a cluster sync;
//   * both CTAs' producers wait on their own `empty` ring and issue TMA loads
//     into their own smem whose completion is counted on the LEADER's `full`
//     barrier (cp.async.bulk.tensor ... .cta_group::2); the leader arms it with
//     the bytes of both CTAs;
//   * the leader's single MMA thread issues the MMAs and commits with a
//     multicast arrival on both CTAs' `empty` / `acc_full` barriers;
//   * for the MX kinds the scale warp of each CTA loads its scale atoms for
//     kSfGroup blocks at a time into a two-slot smem ring, and the leader's
//     scale warp copies both CTAs' atoms into TMEM (tcgen05.cp) and commits to
//     `grp_full`; the MMA thread waits on that once per group and commits to
//     `grp_done` after the group's MMAs.  Issuing the copies from the MMA
//     thread stalled it: a blocking barrier wait placed after tcgen05.cp waits
//     for the copies to finish, which holds the issuer to one block ahead of
//     the tensor pipe (measured: 634 instead of 512 clocks per 128-K block);
//   * both CTAs' epilogues drain their own TMEM and arrive on the leader's
//     `acc_empty` (16 arrivals: 8 warps x 2 CTAs).
// Every TMA load targets its own CTA's shared memory (none is broadcast to the
// cluster), and no kernel reads another GPU's memory.
#pragma once

#include "b2g_gemm.cuh"

namespace b2g {

// 128-K blocks whose scale atoms one TMA box brings in (the pair kernel's MX kinds);
// the host encodes the scale tensor maps with boxes of this many blocks.
// Four for both MX kinds (MXFP4 with groups of two and a sixth operand stage ran
// 4280-4497 instead of 5088-5194 TFLOP/s at 8192^3).
__host__ __device__ constexpr int pair_sf_group(int /*mode*/) { return 4; }

template <int kMode_, int kBN_, bool kBPre_, bool kOutF32_, bool kEpi_ = false>
struct PairCfg {
  static constexpr int kMode = kMode_;
  static constexpr bool kEpi = kEpi_;  // beta * C / bias terms compiled in (only the instances that take them)
  static constexpr bool kBPre = kBPre_;
  static constexpr bool kOutF32 = kOutF32_;
  static constexpr int kBN = kBN_;        // pair tile N (MMA N): 256 or 192
  static constexpr int kHalf = 128;       // rows of A per CTA
  static constexpr int kHalfB = kBN / 2;  // rows of B per CTA
  static constexpr int kEpiWarps = 8;
  static constexpr int kSfWarp = 2 + kEpiWarps;                  // MX kinds: the scale-copy warp
  static constexpr int kThreads = 32 * (kSfWarp + (mode_mx(kMode) ? 1 : 0));
  static constexpr int kColsPerThread = kBN / 2;

  static constexpr int kABytes = kHalf * 128;
  static constexpr int kBBytes = kHalfB * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 6;
  // bytes of columns per TMA-store box of C (boxes are that x 32 rows): MXFP4's 32-byte
  // chunks (1 KB of staging per warp) leave room for the sixth operand stage beside its
  // 24 KB of scale slots (measured 3-9 % faster than five stages and 64-byte chunks)
  static constexpr int kStoreChunkBytes = kMode == kModeMX4 ? 32 : 64;
  static constexpr uint32_t kTxPerStage = 2u * kStageBytes;      // both CTAs complete on the leader's barrier

  // Scale atoms travel apart from the operand stages: one TMA box per operand
  // brings the atoms of kSfGroup consecutive 128-K blocks (the atoms of one row
  // block are contiguous along K) into one of two smem slots, well ahead of the
  // operands.  Loading them with every stage cost two small TMA boxes per block,
  // which held the operand ring ~20 % below its plain-FP8 rate.
  // A 192-wide tile starts 0 or 64 rows into a 128-row scale atom, so its B
  // scales span 2 atoms and the MMA's scale address is shifted by 0 or 2 TMEM
  // columns (the even shift CUTLASS's N=192 tiles use).
  static constexpr int kSfbAtoms = 2;
  static constexpr int kKAtoms = mode_atoms(kMode);  // scale K-atoms per 128-byte K block
  static constexpr int kSfGroup = mode_mx(kMode) ? pair_sf_group(kMode) : 1;
  static constexpr int kSfaSlotBytes = 512 * kKAtoms * kSfGroup;  // [K-atom][512 B]
  static constexpr int kSfbSlotBytes = 512 * kSfbAtoms * kKAtoms * kSfGroup;  // [row block][K-atom][512 B]
  static constexpr int kSfSlotBytes = kSfaSlotBytes + kSfbSlotBytes;
  static constexpr int kSfSlots = mode_mx(kMode) ? 2 : 0;
  static constexpr uint32_t kSfTxPerSlot = 2u * kSfSlotBytes;

  // Scale factors live in TMEM in kSfSets column sets, two groups' worth (block
  // i of group g uses set (g % 2) * kSfGroup + i): A K-atom q at + 4q, then B
  // K-atom q of row block j at + 4 * kKAtoms + 4 * (q * kSfbAtoms + j).
  static constexpr int kSfCols = 4 * kKAtoms * (1 + kSfbAtoms);
  static constexpr int kSfSets = mode_mx(kMode) ? 2 * kSfGroup : 0;
  static constexpr int kAccStages = (2 * kBN + kSfSets * kSfCols <= 512) ? 2 : 1;
  static constexpr int kSfCol0 = kAccStages * kBN;  // + set * kSfCols
  static constexpr int kTmemCols = 512;
  static_assert(kSfCol0 + kSfSets * kSfCols <= kTmemCols, "TMEM columns: accumulators + scale sets");
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffSf = kOffB + kStages * kBBytes;  // + slot * kSfSlotBytes: SFA atoms, then SFB atoms
  static constexpr int kOffStageC = (kOffSf + kSfSlots * kSfSlotBytes + 1023) / 1024 * 1024;  // TMA-store staging
  static constexpr int kStageCBytes = kEpiWarps * 32 * kStoreChunkBytes;                      // one box per warp
  static constexpr int kOffBar = (kOffStageC + kStageCBytes + 7) / 8 * 8;
  // full, empty, acc_full, acc_empty, fin, never, then sf_full, sf_empty, grp_full,
  // grp_done (two each) and sf_fin
  static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2 + 8 + 1;
  static constexpr int kOffCtl = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffCtl + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kBBytes % 1024 == 0, "B stage must keep 1024-byte swizzle atoms aligned");
  // every TMEM column address the kernel forms is a multiple of 32 (loads,
  // accumulator stages) and scale shifts stay even
  static_assert(kBN % 64 == 0 && kColsPerThread % 32 == 0, "tile N");
};

struct PairParams {
  GemmParams g;      // shapes, output, scales, diagnostics (MT counts 256-row pair tiles)
  int num_pairs;     // gridDim.x / 2
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    b2g_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                         const __grid_constant__ CUtensorMap tm_sfa, const __grid_constant__ CUtensorMap tm_sfb,
                         const __grid_constant__ PairParams pp) {
  constexpr int kMode = Cfg::kMode;
  constexpr int ST = Cfg::kStages;
  constexpr int AS = Cfg::kAccStages;
  constexpr int kBN = Cfg::kBN;
  const GemmParams& p = pp.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* acc_full = bars + 2 * ST;
  uint64_t* acc_empty = bars + 2 * ST + AS;
  uint64_t* fin = bars + 2 * ST + 2 * AS;
  uint64_t* never = fin + 1;
  uint64_t* sf_full = never + 1;      // [2] scale slot landed (both CTAs' boxes, on the leader)
  uint64_t* sf_empty = sf_full + 2;   // [2] scale slot copied out (multicast to both CTAs)
  uint64_t* grp_full = sf_empty + 2;  // [2] a group's scales are in TMEM (leader)
  uint64_t* grp_done = grp_full + 2;  // [2] a group's MMAs retired: its TMEM sets are free (leader)
  uint64_t* sf_fin = grp_done + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffCtl + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < AS; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 2 * Cfg::kEpiWarps); }
    mbar_init(fin, 1);
    mbar_init(never, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sf_full[i], 1);
      mbar_init(&sf_empty[i], 1);
      mbar_init(&grp_full[i], 1);
      mbar_init(&grp_done[i], 1);
    }
    mbar_init(sf_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair<Cfg::kTmemCols>(tmem_holder);
  tc_fence_before();
  cluster_sync_all();  // barriers initialised in both CTAs before any remote access
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint64_t tmo = p.timeout_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      if (mode_mx(kMode)) { tma_prefetch_desc(&tm_sfa); tma_prefetch_desc(&tm_sfb); }
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int u = pair; u < p.num_units && ok; u += pp.num_pairs) {
        const Unit w = decode_unit(u, p);
        const int arow = w.mt * 256 + static_cast<int>(rank) * 128;  // this CTA's A rows
        const int brow = w.nt * kBN + static_cast<int>(rank) * Cfg::kHalfB;  // this CTA's B rows
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutProducer, tmo)) { ok = false; break; }
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], Cfg::kTxPerStage);
          tma_load_3d_pair(smem + Cfg::kOffA + s * Cfg::kABytes, &tm_a, bar, kb * 128, arow, w.b);
          if (Cfg::kBPre)
            tma_load_4d_pair(smem + Cfg::kOffB + s * Cfg::kBBytes, &tm_b, bar, 0, brow / 16, kb * 8, w.b);
          else
            tma_load_3d_pair(smem + Cfg::kOffB + s * Cfg::kBBytes, &tm_b, bar, kb * 128, brow, w.b);
          issued_mask |= 1u << s;
          issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
          if (++s == ST) { s = 0; ph ^= 1; }
        }
      }
      if (*abort_flag) {
        if (leader) {  // the leader's barriers count both CTAs' copies
          for (int i = 0; i < ST; ++i)
            if (issued_mask & (1u << i)) {
              volatile int no_abort = 0;
              mbar_wait(&full[i], (issued_phase >> i) & 1u, &no_abort, p.status, kDevTimeoutDrain, 100000000ull);
            }
        } else {  // copies signal the leader; give any in flight time to land
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) sleep_ns(10000);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      int s = 0, as = 0;
      uint32_t ph = 0, aph = 0, g = 0;  // g: scale groups issued by this pair
      bool ok = true;
      constexpr uint16_t kBoth = 0x3;
      constexpr int G = Cfg::kSfGroup;
      if (p.debug_stall) ok = mbar_wait(never, 0, abort_flag, p.status, kDevTimeoutMma, tmo);
      for (int u = pair; u < p.num_units && ok; u += pp.num_pairs) {
        const Unit w = decode_unit(u, p);
        if (!mbar_wait(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + as * kBN;
        // B scales of tile row 0 sit ((nt * BN) % 128) / 32 TMEM columns into the first atom
        const uint32_t sfb_shift = ((w.nt * kBN) & 127) >> 5;
        for (int kb = w.kb0; kb < w.kb1; kb += G, ++g) {
          const int gs = G == 1 ? 1 : min(G, w.kb1 - kb);
          const uint32_t slot = g & 1u;
          if (mode_mx(kMode) && !mbar_wait(&grp_full[slot], (g >> 1) & 1u, abort_flag, p.status, kDevTimeoutMma, tmo)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int i = 0; i < G; ++i) {
            if (i >= gs) break;
            if (!mbar_wait(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smem + Cfg::kOffA + s * Cfg::kABytes);
            const uint32_t b_base = smem_u32(smem + Cfg::kOffB + s * Cfg::kBBytes);
            const uint32_t sfa_tmem = tmem_base + Cfg::kSfCol0 + (slot * G + i) * Cfg::kSfCols;
            const uint32_t sfb_tmem = sfa_tmem + 4 * Cfg::kKAtoms + sfb_shift;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t adesc = desc_kmajor_sw128(a_base + kk * 32);
              const uint64_t bdesc = Cfg::kBPre ? desc_kmajor_interleave(b_base + kk * 2 * (Cfg::kHalfB * 16), Cfg::kHalfB * 16)
                                                : desc_kmajor_sw128(b_base + kk * 32);
              const uint32_t acc = (kb + i > w.kb0 || kk > 0);
              if (kMode == kModeMX)
                mma_mxf8f6f4_pair(d_tmem, adesc, bdesc, idesc_mxf8f6f4(256, kBN, kk, kk), sfa_tmem, sfb_tmem, acc);
              else if (kMode == kModeMX4)  // K-atom kk / 2, byte pair 2 * (kk % 2)
                mma_mxf4_pair(d_tmem, adesc, bdesc, idesc_mxf4(256, kBN, (kk & 1) * 2, (kk & 1) * 2),
                              sfa_tmem + 4 * (kk >> 1), sfb_tmem + 4 * Cfg::kSfbAtoms * (kk >> 1), acc);
              else
                mma_f8f6f4_pair(d_tmem, adesc, bdesc, idesc_f8f6f4(256, kBN), acc);
            }
            tc_commit_pair_mc(&empty[s], kBoth);
            if (++s == ST) { s = 0; ph ^= 1; }
          }
          if (!ok) break;
          if (mode_mx(kMode)) tc_commit_pair(&grp_done[slot]);  // the group's TMEM scale sets are free again
        }
        if (!ok) break;
        tc_commit_pair_mc(&acc_full[as], kBoth);
        if (++as == AS) { as = 0; aph ^= 1; }
      }
      tc_commit_pair(fin);
      volatile int no_abort = 0;
      mbar_wait(fin, 0, &no_abort, p.status, kDevTimeoutDrain, 1000000000ull);
    }
    __syncwarp();
  } else if (mode_mx(kMode) && warp == Cfg::kSfWarp) {
    // ------------------------------------------------------------ scale atoms (MX kinds)
    // Loader (both CTAs): group g of this pair's blocks (kSfGroup consecutive
    // 128-K blocks of one unit) comes in as one SFA and one SFB box into slot
    // g % 2, counted on the leader's sf_full; the slot is refilled once the
    // leader's copies of group g - 2 retired (sf_empty, multicast to both CTAs).
    // Copier (leader): once group g has landed and the MMAs of group g - 2 (the
    // previous readers of its TMEM sets) retired, tcgen05.cp of both CTAs' atoms
    // into sets (g % 2) * kSfGroup + i, then commits to grp_full and sf_empty.
    // The loader stays one group ahead of the copier.  Barrier phases cannot
    // run two ahead of a waiter: each refill waits on the use it replaces.
    // Waits poll (mbar_wait_spin) in the thread that issues tcgen05.cp.
    if (lane == 0) {
      constexpr int G = Cfg::kSfGroup;
      constexpr uint16_t kBoth = 0x3;
      int lu = pair, lkb = 0;
      Unit lw{};
      bool lvalid = lu < p.num_units;
      if (lvalid) { lw = decode_unit(lu, p); lkb = lw.kb0; }
      uint32_t gl = 0, gc = 0;  // groups loaded / copied
      bool ok = true;
      auto load_next = [&]() -> bool {
        if (!lvalid) return true;
        const uint32_t slot = gl & 1u;
        if (gl >= 2 && !mbar_wait_spin(&sf_empty[slot], ((gl - 2) >> 1) & 1u, abort_flag, p.status, kDevTimeoutProducer, tmo))
          return false;
        const uint32_t bar = mapa_shared(smem_u32(&sf_full[slot]), 0);
        if (leader) mbar_arrive_expect_tx(&sf_full[slot], Cfg::kSfTxPerSlot);
        uint8_t* dst = smem + Cfg::kOffSf + slot * Cfg::kSfSlotBytes;
        const int ka = lkb * Cfg::kKAtoms;
        // (128 words, K-atoms, row blocks) boxes of the atom-layout buffers,
        // landing as [K-atom][512 B] and [row block][K-atom][512 B]
        tma_load_4d_pair(dst, &tm_sfa, bar, 0, ka, lw.mt * 2 + static_cast<int>(rank), lw.b);
        tma_load_4d_pair(dst + Cfg::kSfaSlotBytes, &tm_sfb, bar, 0, ka, (lw.nt * kBN) >> 7, lw.b);
        ++gl;
        lkb += G;
        if (lkb >= lw.kb1) {
          lu += pp.num_pairs;
          lvalid = lu < p.num_units;
          if (lvalid) { lw = decode_unit(lu, p); lkb = lw.kb0; }
        }
        return true;
      };
      if (leader) {
        tma_prefetch_desc(&tm_sfa);
        tma_prefetch_desc(&tm_sfb);
        ok = load_next();
        for (int u = pair; u < p.num_units && ok; u += pp.num_pairs) {
          const Unit w = decode_unit(u, p);
          for (int kb = w.kb0; kb < w.kb1; kb += G, ++gc) {
            if (!load_next()) { ok = false; break; }
            const int gs = min(G, w.kb1 - kb);
            const uint32_t slot = gc & 1u;
            if (!mbar_wait_spin(&sf_full[slot], (gc >> 1) & 1u, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
            if (gc >= 2 && !mbar_wait_spin(&grp_done[slot], ((gc - 2) >> 1) & 1u, abort_flag, p.status, kDevTimeoutMma, tmo)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint8_t* src = smem + Cfg::kOffSf + slot * Cfg::kSfSlotBytes;
#pragma unroll
            for (int i = 0; i < G; ++i) {
              if (i >= gs) break;
              const uint32_t set_col = tmem_base + Cfg::kSfCol0 + (slot * G + i) * Cfg::kSfCols;
#pragma unroll
              for (int q = 0; q < Cfg::kKAtoms; ++q) {
                tc_cp_32x128b_warpx4_pair(set_col + 4 * q, desc_sf_atom(smem_u32(src + (i * Cfg::kKAtoms + q) * 512)));
#pragma unroll
                for (int j = 0; j < Cfg::kSfbAtoms; ++j)
                  tc_cp_32x128b_warpx4_pair(
                      set_col + 4 * Cfg::kKAtoms + 4 * (q * Cfg::kSfbAtoms + j),
                      desc_sf_atom(smem_u32(src + Cfg::kSfaSlotBytes + ((j * G + i) * Cfg::kKAtoms + q) * 512)));
              }
            }
            tc_commit_pair(&grp_full[slot]);
            tc_commit_pair_mc(&sf_empty[slot], kBoth);
          }
        }
        tc_commit_pair(sf_fin);  // every copy retired before TMEM is freed
        volatile int no_abort = 0;
        mbar_wait(sf_fin, 0, &no_abort, p.status, kDevTimeoutDrain, 1000000000ull);
        if (*abort_flag)  // boxes still in flight land before the CTA exits
          for (uint32_t g2 = gc; g2 < gl; ++g2)
            mbar_wait(&sf_full[g2 & 1u], (g2 >> 1) & 1u, &no_abort, p.status, kDevTimeoutDrain, 100000000ull);
      } else {
        while (ok && lvalid) ok = load_next();
        if (*abort_flag) {  // boxes signal the leader; give any in flight time to land
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) sleep_ns(10000);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = static_cast<int>(rank) * 128 + quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int NC = Cfg::kColsPerThread;
    uint8_t* stage_c = smem + Cfg::kOffStageC + ew * 32 * Cfg::kStoreChunkBytes;
    int as = 0;
    uint32_t aph = 0;
    for (int u = pair; u < p.num_units; u += pp.num_pairs) {
      const Unit w = decode_unit(u, p);
      const int m = w.mt * 256 + row_in_tile;
      const int col0 = w.nt * kBN + half * NC;
      if (!mbar_wait(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo)) break;
      tc_fence_after();
      constexpr int C32 = NC / 32;
      uint32_t v[NC];
#pragma unroll
      for (int c = 0; c < C32; ++c)
        tmem_ld_32x32b_x32(tmem_base + lane_addr + as * kBN + half * NC + c * 32,
                           *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[as]), 0));
      if (++as == AS) { as = 0; aph ^= 1; }
      float acc[NC];
#pragma unroll
      for (int j = 0; j < NC; ++j) acc[j] = __uint_as_float(v[j]) * p.alpha;
      if constexpr (Cfg::kEpi) {
        if (p.out_mode == kOutStore && m < p.M) {
#pragma unroll
          for (int j = 0; j < NC; j += 4)
            if (col0 + j < p.N)
              epi_apply4<Cfg::kOutF32>(p.epi, w.b, m, col0 + j, acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
      }
      if (p.tma_store && p.out_mode == kOutStore) {
        tma_store_rows<NC, Cfg::kOutF32, Cfg::kStoreChunkBytes>(&p.tm_c, acc, col0,
                                                                 w.mt * 256 + static_cast<int>(rank) * 128 + quad * 32,
                                                                 w.b, stage_c, lane);
      } else if (Cfg::kStoreChunkBytes == 64 && p.out_mode == kOutPeers) {  // MXFP8 only: 2 KB of staging per warp
        peer_store_warp<NC, Cfg::kOutF32>(p, acc, w.mt * 256 + static_cast<int>(rank) * 128 + quad * 32, col0,
                                          w.mt * p.NT + w.nt, stage_c, lane);
      } else if (m < p.M) {
        if (p.out_mode == kOutWorkspace) {
          float* dst = p.ws + ((static_cast<long long>(w.ks) * p.batch + w.b) * p.M + m) * static_cast<long long>(p.N);
#pragma unroll
          for (int j = 0; j < NC; j += 4)
            if (col0 + j < p.N)
              st_global_v4(dst + col0 + j, __float_as_uint(acc[j]), __float_as_uint(acc[j + 1]),
                           __float_as_uint(acc[j + 2]), __float_as_uint(acc[j + 3]));
        } else if (Cfg::kOutF32) {
          float* dst = reinterpret_cast<float*>(p.c) + w.b * p.c_bstride + m * p.ldc;
          if (p.out_mode == kOutAtomic) {
#pragma unroll
            for (int j = 0; j < NC; j += 4)
              if (col0 + j < p.N) red_add_v4_f32(dst + col0 + j, acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < NC; j += 4)
              if (col0 + j < p.N)
                st_global_v4(dst + col0 + j, __float_as_uint(acc[j]), __float_as_uint(acc[j + 1]),
                             __float_as_uint(acc[j + 2]), __float_as_uint(acc[j + 3]));
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.c) + w.b * p.c_bstride + m * p.ldc;
#pragma unroll
          for (int j = 0; j < NC; j += 8)
            if (col0 + j < p.N)
              st_global_v4(dst + col0 + j, pack_bf16x2(acc[j], acc[j + 1]), pack_bf16x2(acc[j + 2], acc[j + 3]),
                           pack_bf16x2(acc[j + 4], acc[j + 5]), pack_bf16x2(acc[j + 6], acc[j + 7]));
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's TMA stores of C are complete
    if (p.out_mode == kOutPeers) __threadfence_system();  // peer stores visible to every GPU
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  cluster_sync_all();  // the leader's MMAs have retired and both epilogues are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair<Cfg::kTmemCols>(tmem_base);
  }
}

}  // namespace b2g
