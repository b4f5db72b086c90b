// b2g_gemm_skinny.cuh -- GEMM for few rows of A (M <= 128: decode / small batch).
//
//   C[m, n] = alpha * sum_k A[m, k] * B[n, k]          m < M <= 128, B = weights
//
// The product is computed transposed: the MMA's M = 128 runs over 128 rows of
// B (weights) and its N = MP (M rounded up to 16/32/64/128) over the rows of A,
// so no tensor-core rows are spent on padding.  Work units are (128-row B tile,
// group of kKB 128-K blocks).  With NT tiles over G persistent CTAs, every CTA
// owns W = NT / G whole tiles (one less when the remainder would be spread too
// thin) and the units of the other NT - W*G tiles are split evenly over the
// CTAs (stream-K): CTA c takes stream-K units [c*U/G, (c+1)*U/G), which may
// begin or end inside a tile, and works through them before its whole tiles.
// Each contiguous run of one tile's units ("segment") accumulates in TMEM.  A
// tile covered by a single segment is written straight to C.  Otherwise every
// segment stores its fp32 partial to scratch and counts itself in the tile's
// arrival counter; the last to arrive adds the partials in segment order (a
// fixed order, so results do not depend on timing), applies alpha and writes C
// in the output type.  Because the split tiles come first, their fix-ups run
// while the whole tiles stream, and every CTA ends on a plain TMEM -> C store.
// One launch per call: no zeroing pass, no atomics on C, no separate cast.
//
// Decode GEMMs are bound by streaming B from HBM: every SM streams an equal
// share of B through a deep ring (128-256 KB of B in flight per SM), and a
// stage carries up to two K blocks so one TMA request moves 32 KB of B.
// Modes: kModePlain (alpha only), kModeMX and kModeMX4 (E4M3 or packed E2M1 with
// UE8M0 1x32 scales; the weights' scale atoms are the MMA's A scales, the
// activations' its B scales).
#pragma once

#include "b2g_gemm.cuh"

namespace b2g {

template <int kMode_, int kMP_, bool kBPre_, int kKB_>
struct SkinnyCfg {
  static constexpr int kMode = kMode_;
  static constexpr int kMP = kMP_;  // padded A rows = MMA N
  static constexpr bool kBPre = kBPre_;
  static constexpr int kKB = kKB_;  // 128-K blocks per stage
  static constexpr int kThreads = 192;  // producer, MMA, 4 epilogue warps
  static constexpr int kWBlk = 128 * 128;  // one 128 x 128 B (weight) tile
  static constexpr int kABlk = kMP * 128;  // the A rows of one 128-K block
  static constexpr int kWBytes = kKB * kWBlk;
  static constexpr int kABytes = kKB * kABlk;
  static constexpr int kKAtoms = mode_atoms(kMode);        // scale K-atoms per 128-byte K block
  static constexpr int kSfBytes = 512 * kKB * kKAtoms;      // per operand per stage
  static constexpr int kStageBytes = kWBytes + kABytes + 2 * kSfBytes;
  static constexpr int kMaxStages = kKB == 1 ? 8 : 5;
  // MP = 16: room for the cluster fold buffer (three other pieces of a tile, fp32)
  static constexpr int kFoldBytes = kMP == 16 ? 3 * kMP * 128 * 4 : 0;
  static constexpr int kStages = (225000 - kFoldBytes) / kStageBytes < kMaxStages ? (225000 - kFoldBytes) / kStageBytes
                                                                                  : kMaxStages;
  static constexpr int kAccStages = 2;
  static constexpr int kAccStride = kMP < 32 ? 32 : kMP;  // accumulator stages start 32-column aligned
  static constexpr int kSfCols = 8 * kKAtoms;  // weight K-atoms (4 columns each), then activation K-atoms
  static constexpr int kSfCol = kAccStages * kAccStride;     // two alternating scale sets follow
  static constexpr int kColsUsed = kSfCol + 2 * kSfCols;
  static constexpr int kTmemCols = kColsUsed <= 32 ? 32 : kColsUsed <= 64 ? 64 : kColsUsed <= 128 ? 128
                                   : kColsUsed <= 256 ? 256 : 512;

  static constexpr int kOffW = 0;
  static constexpr int kOffA = kOffW + kStages * kWBytes;
  static constexpr int kOffSfw = kOffA + kStages * kABytes;
  static constexpr int kOffSfa = kOffSfw + kStages * kSfBytes;
  static constexpr int kOffFold = (kOffSfa + kStages * kSfBytes + 15) / 16 * 16;
  static constexpr int kOffBar = (kOffFold + kFoldBytes + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 3;
  static constexpr int kOffCtl = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffCtl + 16 + 1024;
  static_assert(kStages >= 3, "ring depth");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kMP == 16 || kMP == 32 || kMP == 64 || kMP == 128, "padded M");
  static_assert(kKB == 1 || kKB == 2, "K blocks per stage");
  static_assert(kABlk % 1024 == 0 || kMP == 16, "A stage alignment");
};

struct SkinnyParams {
  int M, N, K;
  void* out;           // C [M][ldo]: fp32 or bf16 (out_f32)
  long long ldo;
  int out_f32;
  float alpha;
  const uint8_t* sfw;  // weight (B) scales, tensor-core atom layout, atoms [n_block][k_block]
  const uint8_t* sfa;  // activation (A) scales, same layout (one row block)
  long long sf_rb;     // bytes between row blocks of either scale buffer
  // fp32 block scales (b2g_gemm_skinny_blk_kernel): bsa [K/128][stride_sfa] per row of A;
  // bsb [N/128][stride_sfb] per 128x128 block (group_n 128) or [K/128][stride_sfb] per column (1)
  const float* bsa;
  const float* bsb;
  long long stride_sfa, stride_sfb;
  int group_n;
  int NT, KG;          // 128-row weight tiles; K groups (kKB blocks each) per tile
  int sk_tiles;        // tiles [0, sk_tiles) are split stream-K; the rest are whole tiles
  int dp_w;            // whole tiles per CTA: CTA c owns tiles sk_tiles + c*dp_w + [0, dp_w)
  int kview;           // 1: operand maps are (128, rows, K/128) views, coordinates (0, row, k_block);
                       // 0: (K, rows, 1) maps, coordinates (k_block * 128, row, 0)
  long long units;     // stream-K units: sk_tiles * KG
  float* part;         // partial slots [2 * gridDim.x][kMP][128] fp32
  unsigned long long* cnt;  // per-tile arrival counters, (tag << 16) | arrivals
  unsigned long long tag;   // this launch's counter tag (nonzero, < 2^48)
  int* status;
  unsigned long long timeout_ns;
  int debug_stall;
  int w_early;  // read B and its scales before the preceding kernel completes (static weights)
  EpiTerms epi;  // beta * C and bias (C and the bias in the output type)
  // k > 1: launched in clusters of k CTAs whose k pieces make one tile each
  // (CTA rank j = piece j); the pieces meet in the rank-0 CTA's shared memory
  // instead of L2 slots and counters (MP = 16, k <= 4)
  int cluster_fold;
};

// CTA owning unit u when U units are split evenly over G CTAs (the largest c
// with U*c/G <= u).
__device__ __forceinline__ int skinny_owner(long long u, long long U, int G) {
  return static_cast<int>(((u + 1) * G - 1) / U);
}

// Partial slot of CTA c's segment on tile nt: 2c for the CTA's first segment
// (its range starts inside or at the start of tile nt), 2c + 1 for its last.
__device__ __forceinline__ int skinny_slot(int c, int nt, long long U, int G, int KG) {
  const long long lo = U * c / G;
  return 2 * c + (lo / KG == nt ? 0 : 1);
}

// The epilogue warps (kEpiThreads threads: 128, or 256 in the untransposed
// blockwise kernel) synchronise on named barrier 1.
template <int kEpiThreads = 128>
__device__ __forceinline__ void skinny_epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

// True on every epilogue thread iff `ok` holds on all of them, so the warps
// leave their loop together and never strand one another at a barrier.
template <int kEpiThreads = 128>
__device__ __forceinline__ bool skinny_epi_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(ok)), "n"(kEpiThreads)
      : "memory");
  return r != 0;
}

// Count one arrival at a tile counter and return the arrivals so far this
// launch.  A counter carrying another tag is stale (an earlier launch that
// stopped early) and counts as zero.  `expect` is the caller's guess of the
// arrivals before it, so the usual case costs one compare-and-swap round trip.
// -1 if the CAS loop does not settle.
__device__ __forceinline__ int skinny_arrive(unsigned long long* cnt, unsigned long long tag, int expect,
                                             int* status) {
  unsigned long long cur = expect > 0 ? (tag << 16) | static_cast<unsigned long long>(expect) : 0ull;
  for (int it = 0; it < (1 << 20); ++it) {
    const unsigned long long nxt = (cur >> 16) == tag ? cur + 1 : (tag << 16) | 1ull;
    const unsigned long long prev = atomicCAS(cnt, cur, nxt);
    if (prev == cur) return static_cast<int>(nxt & 0xFFFFull);
    cur = prev;
  }
  atomicCAS(status, 0, static_cast<int>(kDevTimeoutEpilogue));
  return -1;
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    b2g_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                           const __grid_constant__ SkinnyParams p) {
  constexpr int kMode = Cfg::kMode;
  constexpr int ST = Cfg::kStages;
  constexpr int AS = Cfg::kAccStages;
  constexpr int MP = Cfg::kMP;
  constexpr int KBS = Cfg::kKB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* acc_full = bars + 2 * ST;
  uint64_t* acc_empty = bars + 2 * ST + AS;
  uint64_t* fin = bars + 2 * ST + 2 * AS;
  uint64_t* never = fin + 1;
  uint64_t* fold_bar = never + 1;  // cluster fold: the other pieces are in (rank-0 CTA)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffCtl + 4);
  volatile uint32_t* last_flag = reinterpret_cast<volatile uint32_t*>(smem + Cfg::kOffCtl + 8);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const long long U = p.units;
  const int G = gridDim.x;
  // This CTA's work, walked by position q in [0, nq): stream-K units [u_lo, u_hi),
  // then the units [dp_lo, dp_lo + dp_w * KG) of its whole tiles.
  const long long u_lo = U * blockIdx.x / G, u_hi = U * (blockIdx.x + 1) / G;
  const long long dp_lo = (static_cast<long long>(p.sk_tiles) + static_cast<long long>(blockIdx.x) * p.dp_w) * p.KG;
  const long long nsk = u_hi - u_lo, nq = nsk + static_cast<long long>(p.dp_w) * p.KG;
  auto unit_at = [&](long long q) { return q < nsk ? u_lo + q : dp_lo + (q - nsk); };
  // units from position q to the end of its segment (a tile's run of units)
  auto seg_len = [&](long long q) -> long long {
    if (q < nsk) {
      const long long tile_end = (u_lo + q) / p.KG * p.KG + p.KG;
      return (u_hi < tile_end ? u_hi : tile_end) - (u_lo + q);
    }
    return p.KG - (q - nsk) % p.KG;
  };
  const uint64_t tmo = p.timeout_ns;

  // One stage of loads: B tile(s), A rows and, for MX, both scale atoms (which
  // fill the stage's scale buffers completely).  B is read once: evict first,
  // so it does not push A, the scales and the partial slots out of L2.
  const uint64_t pol_w = l2_policy_evict_first();
  // the weights' part of a stage: arms the stage barrier with the whole stage's bytes
  auto issue_w = [&](long long u, int s) {
    const int nt = static_cast<int>(u / p.KG);
    const int kb = static_cast<int>(u - static_cast<long long>(nt) * p.KG) * KBS;
    mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
    uint8_t* w_dst = smem + Cfg::kOffW + s * Cfg::kWBytes;
    if (Cfg::kBPre)
      tma_load_4d_hint(w_dst, &tm_w, &full[s], 0, nt * 8, kb * 8, 0, pol_w);
    else if (p.kview)
      tma_load_3d_hint(w_dst, &tm_w, &full[s], 0, nt * 128, kb, pol_w);
    else
      tma_load_3d_hint(w_dst, &tm_w, &full[s], kb * 128, nt * 128, 0, pol_w);
    if (mode_mx(kMode))
      bulk_load(smem + Cfg::kOffSfw + s * Cfg::kSfBytes, p.sfw + nt * p.sf_rb + kb * 512 * Cfg::kKAtoms, Cfg::kSfBytes,
                &full[s]);
  };
  // the activations' part
  auto issue_a = [&](long long u, int s) {
    const int nt = static_cast<int>(u / p.KG);
    const int kb = static_cast<int>(u - static_cast<long long>(nt) * p.KG) * KBS;
    uint8_t* a_dst = smem + Cfg::kOffA + s * Cfg::kABytes;
    if (p.kview)
      tma_load_3d(a_dst, &tm_a, &full[s], 0, 0, kb);
    else
      tma_load_3d(a_dst, &tm_a, &full[s], kb * 128, 0, 0);
    if (mode_mx(kMode))
      bulk_load(smem + Cfg::kOffSfa + s * Cfg::kSfBytes, p.sfa + kb * 512 * Cfg::kKAtoms, Cfg::kSfBytes, &full[s]);
  };
  auto issue = [&](long long u, int s) {
    issue_w(u, s);
    issue_a(u, s);
  };

  // The producer thread initialises the barriers and fills the whole ring
  // before the block-wide sync, so HBM traffic starts while TMEM is allocated.
  const int pre = static_cast<int>(nq < ST ? nq : ST);
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < AS; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 4); }
    mbar_init(fin, 1);
    mbar_init(never, 1);
    mbar_init(fold_bar, 1);
    // cluster fold: the other k - 1 pieces arrive as bulk copies into this CTA's fold buffer
    if (p.cluster_fold > 1) mbar_arrive_expect_tx(fold_bar, (p.cluster_fold - 1) * MP * 128 * 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
    // Static weights (caller's promise: no kernel before this one on the stream
    // writes B or its scales): their first ring fill streams while the preceding
    // kernel finishes.
    if (p.w_early)
      for (int i = 0; i < pre; ++i) issue_w(unit_at(i), i);
    griddep_wait();  // launched as a programmatic dependent: the previous kernel's writes are visible after this
    for (int i = 0; i < pre; ++i) {
      if (!p.w_early) issue_w(unit_at(i), i);
      issue_a(unit_at(i), i);
    }
  }
  if (warp == 1) tmem_alloc<Cfg::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  if (p.cluster_fold > 1) cluster_sync_all();  // every CTA's fold barrier is initialised before a remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  griddep_wait();
  griddep_launch_dependents();  // the next kernel may start its prologue as SMs free up

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = pre % ST;
      uint32_t ph = pre == ST ? 1u : 0u;
      uint32_t issued_mask = pre == ST ? (1u << ST) - 1u : (1u << pre) - 1u, issued_phase = 0;
      for (long long q = pre; q < nq; ++q) {
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutProducer, tmo)) break;
        issue(unit_at(q), s);
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
      long long q = 0;
      while (ok && q < nq) {
        const long long len = seg_len(q);
        // the MX kinds issue scale copies from this thread: poll (mbar_wait_spin)
        if (!(mode_mx(kMode) ? mbar_wait_spin(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo)
                             : mbar_wait(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + as * Cfg::kAccStride;
        for (long long v = 0; v < len; ++v) {
          if (!(mode_mx(kMode) ? mbar_wait_spin(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo)
                               : mbar_wait(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < KBS; ++j) {
            const uint32_t w_base = smem_u32(smem + Cfg::kOffW + s * Cfg::kWBytes + j * Cfg::kWBlk);
            const uint32_t a_base = smem_u32(smem + Cfg::kOffA + s * Cfg::kABytes + j * Cfg::kABlk);
            const uint32_t sf_off = sfbuf * Cfg::kSfCols;
            sfbuf ^= 1;
            if (mode_mx(kMode)) {
#pragma unroll
              for (int q = 0; q < Cfg::kKAtoms; ++q) {
                const int at = (j * Cfg::kKAtoms + q) * 512;
                tc_cp_32x128b_warpx4(tmem_base + Cfg::kSfCol + sf_off + 4 * q,
                                     desc_sf_atom(smem_u32(smem + Cfg::kOffSfw + s * Cfg::kSfBytes + at)));
                tc_cp_32x128b_warpx4(tmem_base + Cfg::kSfCol + sf_off + 4 * Cfg::kKAtoms + 4 * q,
                                     desc_sf_atom(smem_u32(smem + Cfg::kOffSfa + s * Cfg::kSfBytes + at)));
              }
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t wdesc = Cfg::kBPre ? desc_kmajor_interleave(w_base + kk * 2 * (128 * 16), 128 * 16)
                                                : desc_kmajor_sw128(w_base + kk * 32);
              const uint64_t adesc = desc_kmajor_sw128(a_base + kk * 32);
              const uint32_t acc = (v > 0 || j > 0 || kk > 0);
              if (kMode == kModeMX)
                mma_mxf8f6f4(d_tmem, wdesc, adesc, idesc_mxf8f6f4(128, MP, kk, kk), tmem_base + Cfg::kSfCol + sf_off,
                             tmem_base + Cfg::kSfCol + sf_off + 4, acc);
              else if (kMode == kModeMX4)  // K-atom kk / 2, byte pair 2 * (kk % 2)
                mma_mxf4(d_tmem, wdesc, adesc, idesc_mxf4(128, MP, (kk & 1) * 2, (kk & 1) * 2),
                         tmem_base + Cfg::kSfCol + sf_off + 4 * (kk >> 1),
                         tmem_base + Cfg::kSfCol + sf_off + 4 * Cfg::kKAtoms + 4 * (kk >> 1), acc);
              else
                mma_f8f6f4(d_tmem, wdesc, adesc, idesc_f8f6f4(128, MP), acc);
            }
          }
          tc_commit(&empty[s]);
          if (++s == ST) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit(&acc_full[as]);
        if (++as == AS) { as = 0; aph ^= 1; }
        q += len;
      }
      tc_commit(fin);
      volatile int no_abort = 0;
      mbar_wait(fin, 0, &no_abort, p.status, kDevTimeoutDrain, 1000000000ull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue: 4 warps, one TMEM lane group each
    // Columns are handled CH at a time so one CH-wide register array is live.
    //
    // A split tile's pieces p_0 .. p_{n-1} (segment order) are always added as
    // the right fold p_0 + (p_1 + (... + p_{n-1})), whichever CTA finishes the
    // tile, so the result does not depend on timing.  The CTA finishing a piece
    // either finds (acquire load of the tile counter) that all other pieces are
    // in -- then its own piece never leaves TMEM -- or stores its piece to its
    // slot and counts in with a CAS; the arrival that completes the count adds.
    constexpr int CH = MP < 32 ? MP : 32;
    constexpr bool kPreload = MP <= 32;  // others' pieces fit in registers ahead of the accumulator
    // Pieces read from L2 per fold step: their loads are all issued before the
    // first add, so a tile split over n CTAs costs about n / FB L2 round trips
    // instead of n.  Two is the most that compiles without spills (MP = 32 keeps
    // a 32-row preloaded suffix live as well and stays at one).
    constexpr int FB = MP == 32 ? 1 : 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // TMEM lane = weight row in the tile = output column in the tile
    const int et = threadIdx.x - 64;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const int cta = static_cast<int>(blockIdx.x);
    int as = 0;
    uint32_t aph = 0;
    long long q = 0;
    while (q < nq) {
      const long long len = seg_len(q);
      const bool in_sk = q < nsk;
      const int nt = static_cast<int>(unit_at(q) / p.KG);
      const long long t0 = static_cast<long long>(nt) * p.KG;
      // pieces of a stream-K tile are owned by CTAs c0 .. c1; a whole tile is one piece
      const int c0 = in_sk ? skinny_owner(t0, U, G) : cta, c1 = in_sk ? skinny_owner(t0 + p.KG - 1, U, G) : cta;
      const int nseg = c1 - c0 + 1;
      const int j = cta - c0;  // this piece's index in the tile
      const bool fin_seg = in_sk && q + len == nsk;  // this CTA's last stream-K piece
      unsigned long long* cnt = p.cnt + nt;
      const unsigned long long all_others = (p.tag << 16) | static_cast<unsigned long long>(nseg - 1);
      // Piece jj's slot.  Only the first owner's range can start before the tile;
      // every later owner's starts inside it (c0 is the last CTA starting at or
      // before t0), so its slot is 2 * (c0 + jj): no division per piece.
      const int slot0 = nseg > 1 ? skinny_slot(c0, nt, U, G, p.KG) : 0;
      auto piece = [&](int jj) {  // this thread's column of piece jj's slot
        return p.part + static_cast<long long>(jj == 0 ? slot0 : 2 * (c0 + jj)) * MP * 128 + r;
      };

      const uint32_t acc_addr = tmem_base + lane_addr + as * Cfg::kAccStride;
      auto load_chunk = [&](int mc, uint32_t (&x)[CH]) {
        if (CH == 32)
          tmem_ld_32x32b_x32(acc_addr + mc, *reinterpret_cast<uint32_t(*)[32]>(&x[0]));
        else
          tmem_ld_32x32b_x16(acc_addr + mc, *reinterpret_cast<uint32_t(*)[16]>(&x[0]));
        tc_wait_ld();
      };
      // Right fold of the other CTAs' pieces jj = hi .. lo (descending, all != j)
      // into t, rows [mc, mc + CH); t holds the fold above hi if have_t.  FB
      // pieces' loads are in flight together; they are still added one at a time
      // in descending order.
      auto fold_l2 = [&](int mc, int hi, int lo, float (&t)[CH], bool have_t) {
#pragma unroll 1
        for (int jb = hi; jb >= lo; jb -= FB) {
          float y[FB][CH];
#pragma unroll
          for (int b = 0; b < FB; ++b)
            if (jb - b >= lo) {
              const float* pj = piece(jb - b) + mc * 128;
#pragma unroll
              for (int i = 0; i < CH; ++i) y[b][i] = __ldcg(pj + i * 128);
            }
#pragma unroll
          for (int b = 0; b < FB; ++b)
            if (jb - b >= lo) {
#pragma unroll
              for (int i = 0; i < CH; ++i) t[i] = have_t ? y[b][i] + t[i] : y[b][i];
              have_t = true;
            }
        }
        return have_t;
      };
      // the whole right fold p_0 + (p_1 + (... + p_{n-1})) over pieces j .. 0 (this
      // CTA's piece j from TMEM) into t, which holds the fold above j if have_t
      auto fold = [&](int mc, float (&t)[CH], bool have_t) {
        uint32_t v[CH];
        load_chunk(mc, v);
#pragma unroll
        for (int i = 0; i < CH; ++i) t[i] = have_t ? __uint_as_float(v[i]) + t[i] : __uint_as_float(v[i]);
        fold_l2(mc, j - 1, 0, t, true);
      };

      // This CTA's last piece of a split tile usually finishes after the tile's
      // other pieces: bring their slots into L2 while its MMAs run, and if they
      // are all in already, fold the ones after it into registers now.
      const bool cfold = p.cluster_fold > 1 && p.cluster_fold == nseg;
      bool last = false, have_suffix = false;
      float suffix[CH];
      if (nseg > 1 && fin_seg && !cfold) {
        if (et < nseg && et != j) bulk_prefetch_l2(piece(et) - r, MP * 128 * 4);
        if (et == 0) *last_flag = ld_acquire_gpu_u64(cnt) == all_others ? 1u : 0u;
        skinny_epi_bar();
        last = *last_flag != 0;
        if (kPreload && last && j + 1 < nseg) have_suffix = fold_l2(0, nseg - 1, j + 1, suffix, false);
      }

      const bool got = mbar_wait(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo);
      if (!skinny_epi_all(got)) break;
      tc_fence_after();
      const int n = nt * 128 + r;
      const bool col_ok = n < p.N;

      // output columns [mc, mc + CH) of this thread's output column n
      auto store_out = [&](int mc, const float (&x)[CH]) {
        if (!col_ok) return;
        if (epi_any(p.epi)) {
#pragma unroll
          for (int i = 0; i < CH; ++i)
            if (mc + i < p.M) {
              const float y = epi_apply1(p.epi, __fmul_rn(x[i], p.alpha), mc + i, n, p.out_f32 != 0);
              if (p.out_f32) static_cast<float*>(p.out)[(mc + i) * p.ldo + n] = y;
              else static_cast<__nv_bfloat16*>(p.out)[(mc + i) * p.ldo + n] = __float2bfloat16_rn(y);
            }
        } else if (p.out_f32) {
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
#pragma unroll 1
        for (int mc = 0; mc < MP; mc += CH) {
          uint32_t v[CH];
          load_chunk(mc, v);
          float x[CH];
#pragma unroll
          for (int i = 0; i < CH; ++i) x[i] = __uint_as_float(v[i]);
          store_out(mc, x);
        }
      } else if (cfold) {
        // The tile's pieces are the cluster's CTAs (rank j = piece j).  Ranks > 0 stage
        // their piece in their own fold buffer, row r's MP sums contiguous, and each
        // warp bulk-copies its 32 rows into the rank-0 CTA's buffer (piece jj at
        // (jj - 1) * 128 * MP floats), completing as transaction bytes on rank 0's fold
        // barrier; rank 0 adds them as p_0 + (p_1 + (... + p_{k-1})), the order of the
        // L2 path, and stores C.
        float* fbuf = reinterpret_cast<float*>(smem + Cfg::kOffFold);
        if (j > 0) {
          float* mine = fbuf + r * MP;
#pragma unroll 1
          for (int mc = 0; mc < MP; mc += CH) {
            uint32_t v[CH];
            load_chunk(mc, v);
#pragma unroll
            for (int i = 0; i < CH; ++i) mine[mc + i] = __uint_as_float(v[i]);
          }
          fence_proxy_async_smem();  // the generic-proxy writes above, visible to the bulk copy
          __syncwarp();
          if (lane == 0)
            bulk_copy_to_cluster(mapa_shared(smem_u32(fbuf + ((j - 1) * 128 + quad * 32) * MP), 0), fbuf + quad * 32 * MP,
                                 32 * MP * 4, mapa_shared(smem_u32(fold_bar), 0));
        } else {
          const bool in = mbar_wait(fold_bar, 0, abort_flag, p.status, kDevTimeoutEpilogue, tmo);
          if (in) {
#pragma unroll 1
            for (int mc = 0; mc < MP; mc += CH) {
              float t[CH];
#pragma unroll
              for (int i = 0; i < CH; ++i) t[i] = fbuf[((nseg - 2) * 128 + r) * MP + mc + i];
#pragma unroll 1
              for (int jj = nseg - 2; jj >= 1; --jj) {
#pragma unroll
                for (int i = 0; i < CH; ++i) t[i] = fbuf[((jj - 1) * 128 + r) * MP + mc + i] + t[i];
              }
              uint32_t v[CH];
              load_chunk(mc, v);
#pragma unroll
              for (int i = 0; i < CH; ++i) t[i] = __uint_as_float(v[i]) + t[i];
              store_out(mc, t);
            }
          }
        }
      } else {
        if (fin_seg && !last) {  // look again now that this piece is done
          if (et == 0) *last_flag = ld_acquire_gpu_u64(cnt) == all_others ? 1u : 0u;
          skinny_epi_bar();
          last = *last_flag != 0;
          skinny_epi_bar();  // every thread has read the flag before it is written again
        }
        if (!last) {
          // store this piece (all MP rows, unpredicated, so stores and loads pipeline) and count in:
          // the barrier orders the four warps' stores before thread 0's release fence and CAS; its
          // acquire fence and the second barrier order the reads of the other pieces after it
          float* mine = piece(j);
#pragma unroll 1
          for (int mc = 0; mc < MP; mc += CH) {
            uint32_t v[CH];
            load_chunk(mc, v);
#pragma unroll
            for (int i = 0; i < CH; ++i) __stcg(mine + (mc + i) * 128, __uint_as_float(v[i]));
          }
          skinny_epi_bar();
          if (et == 0) {
            fence_acq_rel_gpu();
            // a CTA's last piece usually arrives after the tile's other pieces, its first before them
            const int arrivals = skinny_arrive(cnt, p.tag, fin_seg ? nseg - 1 : 0, p.status);
            const bool done = arrivals == nseg;
            if (done) fence_acq_rel_gpu();
            *last_flag = done ? 1u : 0u;
          }
          skinny_epi_bar();
          last = *last_flag != 0;
          have_suffix = false;  // the fold below reads every other piece
        }
        if (last) {
#pragma unroll 1
          for (int mc = 0; mc < MP; mc += CH) {
            float t[CH];
            if (kPreload && have_suffix) {
#pragma unroll
              for (int i = 0; i < CH; ++i) t[i] = suffix[i];
              fold(mc, t, true);
            } else {
              fold(mc, t, fold_l2(mc, nseg - 1, j + 1, t, false));
            }
            store_out(mc, t);
          }
          // every piece is in: leave the counter at zero for the next launch (or a replay)
          if (et == 0) *reinterpret_cast<volatile unsigned long long*>(cnt) = 0ull;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[as]);
      if (++as == AS) { as = 0; aph ^= 1; }
      q += len;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (p.cluster_fold > 1) cluster_sync_all();  // no CTA leaves while a peer may still write its fold buffer
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem_base);
  }
}

}  // namespace b2g
