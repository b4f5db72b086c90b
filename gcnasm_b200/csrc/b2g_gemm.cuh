// b2g_gemm.cuh -- persistent, warp-specialised FP8 GEMM for sm_100a.
//
//   C[b, m, n] = epilogue( sum_k A[b, m, k] * B[b, n, k] )      (TN: both K-major)
//
// One kernel template covers the reference's opus_gemm FP8 family:
//   kModePlain : fp8_gemm (opus_gemm/fp8_gemm/gemm_a8w8_8wave.cc:261-563) plus a
//                per-tensor alpha in the epilogue;
//   kModeMX    : MXFP8, E4M3 with one UE8M0 scale per 1x32 K-block, applied by
//                the tensor core (tcgen05.mma kind::mxf8f6f4.block_scale);
//   kModeMX4   : MXFP4, packed E2M1 (two per byte, the asm_f4gemm operand format)
//                with one UE8M0 scale per 1x32 K-block (kind::mxf4.block_scale);
//                the host passes K and the row strides in bytes, so the tiles,
//                maps and K loop are those of the FP8 modes;
//   kModeBlk   : fp32 block scales, one per 1x128 of A and per 128x128 (GROUP_N=128,
//                opus_gemm/block_scale_gemm) or 1x128 of B (GROUP_N=1,
//                opus_gemm/block_scale_1x128x1_gemm).  Each 128-K block's MMA
//                result lands in its own TMEM buffer and the epilogue warps fold
//                it into fp32 registers with sfa*sfb -- the scale_c_tile step of
//                block_scale_gemm/gemm_a8w8_blockscale_kernel_template.hpp:23-39,
//                applied to TMEM accumulator tiles.
//
// Structure (one CTA per SM, 320 threads; the 256-wide blockwise tile 640):
//   warp 0      TMA producer: A/B tiles (and MX scale atoms) -> smem ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: tcgen05.ld -> registers -> scale / convert -> global
//               (256-wide blockwise: warps 4..11 or 4..19, see GemmCfg::kWide)
// Tiles are 128 x kBN x 128 (M x N x K).  Work units (batch, m-tile, n-tile,
// k-split) are walked statically: CTA i takes units i, i + grid, ... in a
// grouped raster so that concurrently running tiles share A rows in L2.
// Split-K partial sums are either added with fp32 vector reductions into a
// zeroed C (fp32 output) or written to an fp32 workspace that
// b2g_splitk_reduce sums and casts (the workspace + reduce scheme of
// opus_gemm_dist/opus_gemm_mem_gemm_a2a/include/gfx950/splitk_reduce_gfx950.cuh:68-259).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "b2g_epi.cuh"
#include "b2g_ptx.cuh"

namespace b2g {

enum Mode : int { kModePlain = 0, kModeMX = 1, kModeBlk = 2, kModeMX4 = 3 };

// The MX modes carry UE8M0 scale atoms (128 rows x 4 scales: 128 elements of K).
// Operands are walked in 128-byte K blocks: 128 E4M3 elements (kModeMX, one atom
// per block) or 256 packed E2M1 elements (kModeMX4, two atoms per block).
__host__ __device__ constexpr bool mode_mx(int m) { return m == kModeMX || m == kModeMX4; }
__host__ __device__ constexpr int mode_atoms(int m) { return m == kModeMX4 ? 2 : (m == kModeMX ? 1 : 0); }
// kOutPeers: column-parallel multi-GPU use -- every element (m, n) of this call's C is
// stored into each peer buffer at peer_c[i] + m * peer_ldc + peer_col0 + n (the
// caller's full-width C on every GPU of the job, mapped into this process), so
// no all-gather follows the GEMM.
enum OutMode : int { kOutStore = 0, kOutAtomic = 1, kOutWorkspace = 2, kOutPeers = 3 };
constexpr int kMaxPeers = 8;

struct GemmParams {
  // C as a (N, M, batch) TMA map with (64 bytes of columns) x 32 rows boxes; used
  // when tma_store is set (plain stores, 16-byte row pitch), else C is written
  // with vector stores
  CUtensorMap tm_c;
  int tma_store;
  int M, N, K, batch;
  // output: C[b][m][n] at c + b*c_bstride + m*ldc + n (elements of the output type)
  void* c;
  long long ldc, c_bstride;
  int out_mode;
  float* ws;  // split-K workspace [S][batch][M][N] fp32 (out_mode == kOutWorkspace)
  void* peer_c[kMaxPeers];  // out_mode == kOutPeers
  int n_peers, peer_first;  // peer_first: this GPU's index, where a tile's round of peer stores starts
  long long peer_ldc, peer_col0;
  // all-to-all (peer_shard > 0): column shard q = n / peer_shard goes to peer q only, row
  // peer_row0 + m of its [rows][peer_shard] window; else every peer gets every column
  long long peer_shard, peer_row0;
  float alpha;
  EpiTerms epi;  // beta * C and bias, applied where C is written (kOutStore) or in the split-K reduce
  // MX: UE8M0 scales in the tensor-core atom layout (128 rows x 4 K-blocks per
  // 512-byte atom, atoms [row_block][k_block]); *_rb = bytes between row blocks
  const uint8_t* sfa;
  long long sfa_rb, sfa_bstride;
  const uint8_t* sfb;
  long long sfb_rb, sfb_bstride;
  int sfb_blocks;  // ceil(N / 128): number of valid B row blocks
  // kModeBlk: fp32 scales (opus_gemm_kargs semantics)
  const float* bsa;
  long long stride_sfa, bsa_bstride;  // SFA[kg * stride_sfa + m]
  const float* bsb;
  long long stride_sfb, bsb_bstride;  // GROUP_N=128: SFB[(n/128)*stride_sfb + kg]; GROUP_N=1: SFB[kg*stride_sfb + n]
  int group_n;
  // static schedule
  int MT, NT, S, KB, kb_per_split, group_m, num_units;
  // diagnostics
  int* status;
  unsigned long long timeout_ns;
  int debug_stall;  // test hook: the MMA issuer waits on a barrier nothing arrives on
};

struct Unit {
  int b, mt, nt, ks, kb0, kb1;
};

// Epilogue write to every peer: this warp's 32 rows (row0 + lane) x NC columns
// (col0 + j, values acc[j] of the lane's row) of this call's C into each peer
// buffer.  A lane holds one row, so its own stores would scatter 16-byte pieces
// over 32 rows -- one small NVLink transaction each.  Instead 16 rows x 128 bytes
// of columns at a time are staged in the warp's 2 KB of shared memory and read
// back so that every warp-wide store writes four rows as whole 128-byte runs.
// The peers are taken in a different order per tile and GPU so the GPUs' store
// streams spread over the destinations.
// (not inlined: its working set stays off the kernels' main epilogue path)
template <int NC, bool kF32>
__device__ __noinline__ void peer_store_warp(const GemmParams& p, const float (&acc)[NC], int row0, int col0,
                                             int tile, uint8_t* stage, int lane) {
  constexpr int CW = kF32 ? 32 : 64;  // columns in 128 bytes
  constexpr int EP = kF32 ? 4 : 8;    // elements in 16 bytes
  const int first = (p.peer_first + tile) % p.n_peers;
  const int es = kF32 ? 4 : 2;
#pragma unroll
  for (int h = 0; h < 2; ++h) {         // rows row0 + 16h .. + 15
#pragma unroll
    for (int c = 0; c < NC / CW; ++c) {  // columns col0 + c*CW .. + CW - 1
      __syncwarp();
      if ((lane >> 4) == h) {
        uint4* dst = reinterpret_cast<uint4*>(stage + (lane & 15) * 128);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (kF32)
            dst[q] = make_uint4(__float_as_uint(acc[c * CW + 4 * q]), __float_as_uint(acc[c * CW + 4 * q + 1]),
                                __float_as_uint(acc[c * CW + 4 * q + 2]), __float_as_uint(acc[c * CW + 4 * q + 3]));
          else
            dst[q] = make_uint4(pack_bf16x2(acc[c * CW + 8 * q], acc[c * CW + 8 * q + 1]),
                                pack_bf16x2(acc[c * CW + 8 * q + 2], acc[c * CW + 8 * q + 3]),
                                pack_bf16x2(acc[c * CW + 8 * q + 4], acc[c * CW + 8 * q + 5]),
                                pack_bf16x2(acc[c * CW + 8 * q + 6], acc[c * CW + 8 * q + 7]));
        }
      }
      __syncwarp();
      // piece i*32 + lane of the staged 16 x 128 bytes: row (..)/8, 16-byte piece (..)%8;
      // re-read from shared memory per peer so that only one piece is live at a time
      if (p.peer_shard > 0) {  // all-to-all: these CW columns belong to one peer's shard
        const int n0 = col0 + c * CW;
        const int q = static_cast<int>(n0 / p.peer_shard);
        uint8_t* base = static_cast<uint8_t*>(p.peer_c[q]);
        const long long c_off = n0 - static_cast<long long>(q) * p.peer_shard;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int idx = i * 32 + lane;
          const int r = idx >> 3, pc = idx & 7;
          const int m = row0 + 16 * h + r;
          if (m < p.M && n0 + pc * EP < p.N) {
            const uint4 v = reinterpret_cast<const uint4*>(stage + r * 128)[pc];
            st_global_v4(base + ((p.peer_row0 + m) * p.peer_shard + c_off + pc * EP) * es, v.x, v.y, v.z, v.w);
          }
        }
        continue;
      }
      for (int t = 0; t < p.n_peers; ++t) {
        int q = first + t;
        if (q >= p.n_peers) q -= p.n_peers;
        uint8_t* base = static_cast<uint8_t*>(p.peer_c[q]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int idx = i * 32 + lane;
          const int r = idx >> 3, pc = idx & 7;
          const int m = row0 + 16 * h + r;
          const int n = col0 + c * CW + pc * EP;
          if (m < p.M && n < p.N) {
            const uint4 v = reinterpret_cast<const uint4*>(stage + r * 128)[pc];
            st_global_v4(base + (static_cast<long long>(m) * p.peer_ldc + p.peer_col0 + n) * es, v.x, v.y, v.z,
                         v.w);
          }
        }
      }
    }
  }
  __syncwarp();
}

// Epilogue write through TMA: this warp's 32 rows (row0 + lane) x NC columns
// (col0 + j, values acc[j] of the lane's row) of C, converted to the output type
// and staged 64 bytes of columns at a time in the warp's 2 KB of shared memory,
// each chunk a (64 B x 32 rows) box stored by lane 0.  Rows past M and columns
// past N are clipped by the store itself, so every lane takes part.
template <int NC, bool kF32, int kChunkBytes = 64>
__device__ __forceinline__ void tma_store_rows(const CUtensorMap* tm, const float (&acc)[NC], int col0, int row0,
                                               int b, uint8_t* stage, int lane) {
  constexpr int CH = kChunkBytes / (kF32 ? 4 : 2);  // columns per row chunk
  constexpr int Q = kChunkBytes / 16;               // 16-byte pieces per row chunk
  uint4* mine = reinterpret_cast<uint4*>(stage + lane * kChunkBytes);
#pragma unroll
  for (int c = 0; c < NC / CH; ++c) {
    if (c > 0) {  // the previous chunk's store has read the stage
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
    }
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      if (kF32)
        mine[q] = make_uint4(__float_as_uint(acc[c * CH + 4 * q]), __float_as_uint(acc[c * CH + 4 * q + 1]),
                             __float_as_uint(acc[c * CH + 4 * q + 2]), __float_as_uint(acc[c * CH + 4 * q + 3]));
      else
        mine[q] = make_uint4(pack_bf16x2(acc[c * CH + 8 * q], acc[c * CH + 8 * q + 1]),
                             pack_bf16x2(acc[c * CH + 8 * q + 2], acc[c * CH + 8 * q + 3]),
                             pack_bf16x2(acc[c * CH + 8 * q + 4], acc[c * CH + 8 * q + 5]),
                             pack_bf16x2(acc[c * CH + 8 * q + 6], acc[c * CH + 8 * q + 7]));
    }
    fence_proxy_async_smem();  // the generic-proxy writes above, visible to the TMA
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tm, stage, col0 + c * CH, row0, b);
      bulk_commit_group();
    }
  }
  if (lane == 0) bulk_wait_read_all();  // the stage is free for the next tile
  __syncwarp();
}

__host__ __device__ __forceinline__ Unit decode_unit(int u, const GemmParams& p) {
  Unit w;
  w.ks = u % p.S;
  const int t = u / p.S;
  const int tiles = p.MT * p.NT;
  w.b = t / tiles;
  const int r = t - w.b * tiles;
  const int gsz = p.group_m * p.NT;
  const int g = r / gsz;
  const int first_m = g * p.group_m;
  const int gm = (p.MT - first_m) < p.group_m ? (p.MT - first_m) : p.group_m;
  const int q = r - g * gsz;
  w.mt = first_m + q % gm;
  w.nt = q / gm;
  w.kb0 = w.ks * p.kb_per_split;
  w.kb1 = (w.kb0 + p.kb_per_split) < p.KB ? (w.kb0 + p.kb_per_split) : p.KB;
  return w;
}

// compile-time configuration -------------------------------------------------
template <int kMode_, int kBN_, bool kBPre_, bool kOutF32_, bool kEpi_ = false, bool kGn1_ = false>
struct GemmCfg {
  static constexpr int kMode = kMode_;
  // blockwise: B's fp32 scales per column (GROUP_N = 1) instead of per 128 x 128 block
  static constexpr bool kGn1 = kGn1_;
  static constexpr bool kEpi = kEpi_;  // beta * C / bias terms compiled in (only the instances that take them)
  static constexpr int kBN = kBN_;
  static constexpr bool kBPre = kBPre_;     // B given 16x16-preshuffled ([N/16][K/16][16][16] bytes)
  static constexpr bool kOutF32 = kOutF32_;
  static constexpr int kBM = 128, kBK = 128, kUmmaK = 32;
  // The 256-wide blockwise tile promotes every 128-K block's 128 x 256 partial in
  // registers and re-splits the registers between warpgroups (setmaxnreg); the
  // two weight-scale layouts are separate instances (kGn1), so each epilogue
  // carries only its own promotion code:
  //   - 128 x 128 weight scales (kQuad): 20 warps, warpgroup 0 (producer, MMA
  //     issuer, two idle warps) and 16 epilogue warps, four per TMEM lane group,
  //     each holding 64 fp32 sums of one row, so a partial buffer drains in half
  //     the time of 8 warps.  The launch holds 640 * 96 registers; warpgroup 0
  //     drops to 32, the epilogue rises to 112: 128 * 32 + 512 * 112 = 640 * 96,
  //     per sub-partition 32 + 4 * 112 <= 512.
  //   - per-column weight scales: 12 warps, 8 epilogue warps of 128 sums each in
  //     the .16x256b fragment form (measured 20 % faster than 16 warps of 64);
  //     warpgroup 0 at 56, the epilogue at 224: 128 * 56 + 256 * 224 = 384 * 168.
  // Every other tile: 10 warps, epilogue warps 2..9, each half a tile's columns.
  static constexpr bool kWide = kMode == kModeBlk && kBN_ == 256;
  static constexpr bool kQuad = kWide && !kGn1;
  static constexpr int kThreads = kQuad ? 640 : (kWide ? 384 : 320);
  static constexpr int kFirstEpiWarp = kWide ? 4 : 2;
  static constexpr int kEpiWarps = kQuad ? 16 : 8;
  static constexpr int kRegsLow = kQuad ? 32 : 56, kRegsHigh = kQuad ? 112 : 224;  // kWide re-split
  static constexpr int kColsPerThread = kBN / (kEpiWarps / 4);  // each epilogue thread: one row, a column slice
  static constexpr int kChunks = kColsPerThread / 32;
  // bytes of columns per TMA-store box of C (boxes are that x 32 rows)
  static constexpr int kStoreChunkBytes = kQuad ? 32 : 64;

  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = kBN * kBK;
  static constexpr int kKAtoms = mode_atoms(kMode);  // scale atoms per 128-row block per stage
  static constexpr int kSfaBytes = 512 * kKAtoms;
  static constexpr int kSfbAtoms = (kBN + 127) / 128;
  static constexpr int kSfbBytes = 512 * kSfbAtoms * kKAtoms;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr int kStages = (kBN == 256) ? 4 : 6;

  // TMEM: accumulator (or per-K-block partial) buffers, then the MX scales in two
  // alternating column sets (the copies for block k+1 never overwrite columns the
  // MMAs of block k still read)
  static constexpr int kSfCols = 4 * kKAtoms * (1 + kSfbAtoms);
  static constexpr int kSfBufs = 2;
  // blockwise: as many per-K-block partial buffers as TMEM holds, so the MMAs run
  // up to three K blocks ahead of the promotion
  static constexpr int kAccStages = (kMode == kModeBlk) ? 512 / kBN : ((2 * kBN + kSfBufs * kSfCols <= 512) ? 2 : 1);
  // per column set: A atoms (4 columns each, K-atom q at + 4q), then B atoms
  // (K-atom q of row block j at + 4 * (q * kSfbAtoms + j): one K-atom's B scales
  // are contiguous over the tile's rows, as the MMA reads them)
  static constexpr int kSfaCol = kAccStages * kBN;  // + buffer * kSfCols
  static constexpr int kSfbCol = kSfaCol + 4 * kKAtoms;
  static constexpr int kTmemCols = 512;

  // shared memory carve-up (offsets from a 1024-byte aligned base)
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffSfa = kOffB + kStages * kBBytes;
  static constexpr int kOffSfb = kOffSfa + kStages * kSfaBytes;
  static constexpr int kOffSbStage = kOffSfb + kStages * kSfbBytes;  // GROUP_N=1 column scales
  static constexpr int kSbStageBytes = kMode == kModeBlk ? kEpiWarps * kColsPerThread * 4 : 0;
  static constexpr int kOffStageC = (kOffSbStage + kSbStageBytes + 1023) / 1024 * 1024;  // TMA-store staging
  static constexpr int kStageCBytes = kEpiWarps * 32 * kStoreChunkBytes;                  // one box per warp
  static constexpr int kOffBar = (kOffStageC + kStageCBytes + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2;
  static constexpr int kOffCtl = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffCtl + 16 + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kBN == 128 || kBN == 256, "tile N");
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    b2g_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ GemmParams p) {
  constexpr int kMode = Cfg::kMode;
  constexpr int kBN = Cfg::kBN;
  constexpr int ST = Cfg::kStages;
  constexpr int AS = Cfg::kAccStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* acc_full = bars + 2 * ST;
  uint64_t* acc_empty = bars + 2 * ST + AS;
  uint64_t* fin = bars + 2 * ST + 2 * AS;      // end-of-kernel MMA drain
  uint64_t* never = fin + 1;                    // test hook: nothing ever arrives here
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kOffCtl);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffCtl + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (mode_mx(kMode)) {  // scale atoms never fetched (tile edge) must hold a finite scale
    for (int i = threadIdx.x; i < ST * (Cfg::kSfaBytes + Cfg::kSfbBytes) / 4; i += Cfg::kThreads)
      reinterpret_cast<uint32_t*>(smem + Cfg::kOffSfa)[i] = 0x7F7F7F7Fu;
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < AS; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], Cfg::kEpiWarps); }
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

  // kWide: each role's branch opens with its warpgroup's register re-split, so the
  // compiler allocates the epilogue's code with 224 registers
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if constexpr (Cfg::kWide) setmaxnreg_dec<Cfg::kRegsLow>();
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        const Unit w = decode_unit(u, p);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutProducer, tmo)) { ok = false; break; }
          uint32_t tx = Cfg::kABytes + Cfg::kBBytes;
          int nsfb = 0;
          if (mode_mx(kMode)) {
            nsfb = p.sfb_blocks - w.nt * Cfg::kSfbAtoms;
            nsfb = nsfb < Cfg::kSfbAtoms ? nsfb : Cfg::kSfbAtoms;
            tx += 512u * Cfg::kKAtoms * (1 + nsfb);
          }
          mbar_arrive_expect_tx(&full[s], tx);
          tma_load_3d(smem + Cfg::kOffA + s * Cfg::kABytes, &tm_a, &full[s], kb * 128, w.mt * 128, w.b);
          if (Cfg::kBPre)
            tma_load_4d(smem + Cfg::kOffB + s * Cfg::kBBytes, &tm_b, &full[s], 0, w.nt * (kBN / 16), kb * 8, w.b);
          else
            tma_load_3d(smem + Cfg::kOffB + s * Cfg::kBBytes, &tm_b, &full[s], kb * 128, w.nt * kBN, w.b);
          if (mode_mx(kMode)) {  // the block's K-atoms of each 128-row block are contiguous
            constexpr uint32_t kAB = 512u * Cfg::kKAtoms;
            bulk_load(smem + Cfg::kOffSfa + s * Cfg::kSfaBytes,
                      p.sfa + w.b * p.sfa_bstride + w.mt * p.sfa_rb + kb * kAB, kAB, &full[s]);
            for (int j = 0; j < nsfb; ++j)
              bulk_load(smem + Cfg::kOffSfb + s * Cfg::kSfbBytes + j * kAB,
                        p.sfb + w.b * p.sfb_bstride + (w.nt * Cfg::kSfbAtoms + j) * p.sfb_rb + kb * kAB, kAB,
                        &full[s]);
          }
          issued_mask |= 1u << s;
          issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
          if (++s == ST) { s = 0; ph ^= 1; }
        }
      }
      if (*abort_flag) {  // let copies already in flight land before the CTA retires
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
    if constexpr (Cfg::kWide) setmaxnreg_dec<Cfg::kRegsLow>();
    if (lane == 0) {
      int s = 0, as = 0;
      uint32_t ph = 0, aph = 0, sfbuf = 0;
      bool ok = true;
      if (p.debug_stall) ok = mbar_wait(never, 0, abort_flag, p.status, kDevTimeoutMma, tmo);
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        const Unit w = decode_unit(u, p);
        // the MX kinds issue scale copies from this thread: poll (mbar_wait_spin)
        if (kMode != kModeBlk) {
          if (!(mode_mx(kMode) ? mbar_wait_spin(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo)
                               : mbar_wait(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!(mode_mx(kMode) ? mbar_wait_spin(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo)
                               : mbar_wait(&full[s], ph, abort_flag, p.status, kDevTimeoutMma, tmo))) {
            ok = false;
            break;
          }
          if (kMode == kModeBlk) {
            // a partial buffer frees every K block: poll, the wait is short and a suspended
            // thread wakes late (same-box A/B: 0-10 % faster over the C3 shapes)
            if (!mbar_wait_spin(&acc_empty[as], aph ^ 1, abort_flag, p.status, kDevTimeoutMma, tmo)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + Cfg::kOffA + s * Cfg::kABytes);
          const uint32_t b_base = smem_u32(smem + Cfg::kOffB + s * Cfg::kBBytes);
          const uint32_t d_tmem = tmem_base + as * kBN;
          const uint32_t sf_off = sfbuf * Cfg::kSfCols;
          sfbuf ^= 1;
          if (mode_mx(kMode)) {
#pragma unroll
            for (int q = 0; q < Cfg::kKAtoms; ++q) {
              tc_cp_32x128b_warpx4(tmem_base + Cfg::kSfaCol + sf_off + 4 * q,
                                   desc_sf_atom(smem_u32(smem + Cfg::kOffSfa + s * Cfg::kSfaBytes + q * 512)));
#pragma unroll
              for (int j = 0; j < Cfg::kSfbAtoms; ++j)
                tc_cp_32x128b_warpx4(tmem_base + Cfg::kSfbCol + sf_off + 4 * (q * Cfg::kSfbAtoms + j),
                                     desc_sf_atom(smem_u32(smem + Cfg::kOffSfb + s * Cfg::kSfbBytes +
                                                           (j * Cfg::kKAtoms + q) * 512)));
            }
          }
#pragma unroll
          for (int kk = 0; kk < Cfg::kBK / Cfg::kUmmaK; ++kk) {
            const uint64_t adesc = desc_kmajor_sw128(a_base + kk * 32);
            const uint64_t bdesc = Cfg::kBPre ? desc_kmajor_interleave(b_base + kk * 2 * (kBN * 16), kBN * 16)
                                              : desc_kmajor_sw128(b_base + kk * 32);
            const uint32_t acc = (kMode == kModeBlk) ? (kk > 0) : (kb > w.kb0 || kk > 0);
            if (kMode == kModeMX)
              mma_mxf8f6f4(d_tmem, adesc, bdesc, idesc_mxf8f6f4(128, kBN, kk, kk), tmem_base + Cfg::kSfaCol + sf_off,
                           tmem_base + Cfg::kSfbCol + sf_off, acc);
            else if (kMode == kModeMX4)  // K-atom kk / 2, byte pair 2 * (kk % 2)
              mma_mxf4(d_tmem, adesc, bdesc, idesc_mxf4(128, kBN, (kk & 1) * 2, (kk & 1) * 2),
                       tmem_base + Cfg::kSfaCol + sf_off + 4 * (kk >> 1),
                       tmem_base + Cfg::kSfbCol + sf_off + 4 * Cfg::kSfbAtoms * (kk >> 1), acc);
            else
              mma_f8f6f4(d_tmem, adesc, bdesc, idesc_f8f6f4(128, kBN), acc);
          }
          tc_commit(&empty[s]);  // smem stage free once these MMAs have read it
          if (++s == ST) { s = 0; ph ^= 1; }
          if (kMode == kModeBlk) {
            tc_commit(&acc_full[as]);
            if (++as == AS) { as = 0; aph ^= 1; }
          }
        }
        if (!ok) break;
        if (kMode != kModeBlk) {
          tc_commit(&acc_full[as]);
          if (++as == AS) { as = 0; aph ^= 1; }
        }
      }
      // all MMAs retired before TMEM is released
      tc_commit(fin);
      volatile int no_abort = 0;
      mbar_wait(fin, 0, &no_abort, p.status, kDevTimeoutDrain, 1000000000ull);
    }
    __syncwarp();
  } else if (warp < Cfg::kFirstEpiWarp) {
    // ------------------------------------------------------------ idle (kWide: the rest of warpgroup 0)
    if constexpr (Cfg::kWide) setmaxnreg_dec<Cfg::kRegsLow>();
  } else {
    // ------------------------------------------------------------ epilogue
    if constexpr (Cfg::kWide) setmaxnreg_inc<Cfg::kRegsHigh>();
    const int ew = warp - Cfg::kFirstEpiWarp;
    const int quad = warp & 3;                 // TMEM lane group this warp may access
    const int half = ew >> 2;                  // which column slice of the tile (half, or quarter when kQuad)
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int NC = Cfg::kColsPerThread;
    int as = 0;
    uint32_t aph = 0;
    float* sb_stage = reinterpret_cast<float*>(smem + Cfg::kOffSbStage) + ew * NC;
    uint8_t* stage_c = smem + Cfg::kOffStageC + ew * (32 * Cfg::kStoreChunkBytes);

    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
      const Unit w = decode_unit(u, p);
      const int m = w.mt * 128 + row_in_tile;
      const int col0 = w.nt * kBN + half * NC;
      float acc[NC];
      bool ok = true;

      if constexpr (Cfg::kWide && Cfg::kGn1) {
        // Per-column weight scales on the 256-wide tile, fragment form: each K block's
        // partial is read with tcgen05.ld .16x256b, so a thread holds 4 rows x NC/4
        // columns of its warp's 32 x NC slice -- rows quad*32 + t/4 + 8i (i = 0..3),
        // columns col0 + 8j + 2(t%4) + {0, 1} (j < NC/8) -- and needs NC/4 column scales
        // per K block (8-byte shared-memory reads, one wavefront each) instead of all NC.
        // Same rounding as the row form: (P * sfb[n]) * sfa[m] + acc.
        const int t4 = lane & 3, r8 = lane >> 2;
        constexpr int NG = NC / 8;  // 8-column groups of this warp's slice
        float2 f[4][NG];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < NG; ++j) f[i][j] = make_float2(0.f, 0.f);
        const bool row_ok = m < p.M;  // this lane's own row: its sfa is shared with the fragment's rows
        const float* sa_ptr = p.bsa + w.b * p.bsa_bstride + m;
        const float* sb_ptr = p.bsb + w.b * p.bsb_bstride + col0 + 4 * lane;
        const bool sb_lane_ok = 4 * lane < NC && col0 + 4 * lane < p.N;
        auto load_sa = [&](int kb) -> float { return (row_ok && kb < w.kb1) ? __ldg(sa_ptr + kb * p.stride_sfa) : 0.f; };
        auto load_sb = [&](int kb) -> float4 {
          return (kb < w.kb1 && sb_lane_ok) ? __ldg(reinterpret_cast<const float4*>(sb_ptr + kb * p.stride_sfb))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        float sa0 = load_sa(w.kb0), sa1 = load_sa(w.kb0 + 1);
        float4 sb0 = load_sb(w.kb0), sb1 = load_sb(w.kb0 + 1);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const float sa = sa0;
          const float4 sb = sb0;
          sa0 = sa1; sb0 = sb1;
          sa1 = load_sa(kb + 2); sb1 = load_sb(kb + 2);
          if (4 * lane < NC) *reinterpret_cast<float4*>(sb_stage + 4 * lane) = sb;
          __syncwarp();
          float2 sa2[4];  // the fragment rows' A scales, from the lanes that own those rows
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float x = __shfl_sync(0xffffffffu, sa, r8 + 8 * i);
            sa2[i] = make_float2(x, x);
          }
          if (!mbar_wait_spin(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < NC / 32; ++c) {  // 32 columns: groups j = 4c .. 4c + 3
            uint32_t lo[16], hi[16];
            const uint32_t col_addr = tmem_base + as * kBN + half * NC + c * 32;
            tmem_ld_16x256b_x4(col_addr + lane_addr, lo);                                  // rows t/4, t/4 + 8
            tmem_ld_16x256b_x4(col_addr + lane_addr + (static_cast<uint32_t>(16) << 16), hi);  // + 16
            tc_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int j = 4 * c + jj;
              const float2 b2 = *reinterpret_cast<const float2*>(sb_stage + 8 * j + 2 * t4);
              f[0][j] = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(lo[4 * jj]), __uint_as_float(lo[4 * jj + 1])), b2),
                                   sa2[0], f[0][j]);
              f[1][j] = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(lo[4 * jj + 2]), __uint_as_float(lo[4 * jj + 3])), b2),
                                   sa2[1], f[1][j]);
              f[2][j] = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(hi[4 * jj]), __uint_as_float(hi[4 * jj + 1])), b2),
                                   sa2[2], f[2][j]);
              f[3][j] = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(hi[4 * jj + 2]), __uint_as_float(hi[4 * jj + 3])), b2),
                                   sa2[3], f[3][j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[as]);
          if (++as == AS) { as = 0; aph ^= 1; }
        }
        if (!ok) break;
        // ---- write the fragment: rows w.mt*128 + quad*32 + r8 + 8i, columns col0 + 8j + 2*t4 + {0, 1}
        const int row_base = w.mt * 128 + quad * 32;
        if (p.tma_store && p.out_mode == kOutStore) {
          // column chunks of kStoreChunkBytes x 32 rows staged row-major in the warp's
          // staging slot, then one TMA box store each (rows past M, columns past N clipped)
          constexpr int ES = Cfg::kOutF32 ? 4 : 2;
          constexpr int CB = Cfg::kStoreChunkBytes;
          constexpr int GPC = CB / (8 * ES);  // 8-column groups per chunk
#pragma unroll
          for (int ch = 0; ch < NG / GPC; ++ch) {
            if (ch > 0) {
              if (lane == 0) bulk_wait_read_all();
              __syncwarp();
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int g = 0; g < GPC; ++g) {
                const float2 x = f[i][ch * GPC + g];
                uint8_t* dst = stage_c + (r8 + 8 * i) * CB + (8 * g + 2 * t4) * ES;
                if (Cfg::kOutF32)
                  *reinterpret_cast<float2*>(dst) = x;
                else
                  *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(x.x, x.y);
              }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&p.tm_c, stage_c, col0 + ch * GPC * 8, row_base, w.b);
              bulk_commit_group();
            }
          }
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int mr = row_base + r8 + 8 * i;
            if (mr >= p.M) continue;
#pragma unroll
            for (int j = 0; j < NG; ++j) {
              const int n = col0 + 8 * j + 2 * t4;
              if (n >= p.N) continue;
              const float2 x = f[i][j];
              if (p.out_mode == kOutWorkspace) {
                float* dst = p.ws + ((static_cast<long long>(w.ks) * p.batch + w.b) * p.M + mr) * static_cast<long long>(p.N);
                st_global_v2(dst + n, __float_as_uint(x.x), __float_as_uint(x.y));
              } else if (Cfg::kOutF32) {
                float* dst = reinterpret_cast<float*>(p.c) + w.b * p.c_bstride + static_cast<long long>(mr) * p.ldc;
                if (p.out_mode == kOutAtomic) red_add_v2_f32(dst + n, x.x, x.y);
                else st_global_v2(dst + n, __float_as_uint(x.x), __float_as_uint(x.y));
              } else {
                __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.c) + w.b * p.c_bstride +
                                     static_cast<long long>(mr) * p.ldc;
                *reinterpret_cast<uint32_t*>(dst + n) = pack_bf16x2(x.x, x.y);
              }
            }
          }
        }
        continue;
      }

      if (kMode != kModeBlk) {
        if (!mbar_wait(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo)) break;
        tc_fence_after();
        uint32_t v[Cfg::kChunks][32];
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c)
          tmem_ld_32x32b_x32(tmem_base + lane_addr + as * kBN + half * NC + c * 32, v[c]);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[as]);
        if (++as == AS) { as = 0; aph ^= 1; }
        const float alpha = p.alpha;
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c * 32 + j] = __uint_as_float(v[c][j]) * alpha;
      } else {
        // fp32 block-scale promotion, one 128-K block at a time
#pragma unroll
        for (int j = 0; j < NC; ++j) acc[j] = 0.f;
        // the promotion keeps its sums as register pairs for the packed two-wide fp32
        // FMA (one instruction per two columns, each rounded as the scalar fmaf)
        float2 acc2[NC / 2];
#pragma unroll
        for (int j = 0; j < NC / 2; ++j) acc2[j] = make_float2(0.f, 0.f);
        const bool row_ok = m < p.M;
        const float* sa_ptr = p.bsa + w.b * p.bsa_bstride + m;
        constexpr bool gn1 = Cfg::kGn1;
        const int nblk = col0 / 128;
        const float* sb_ptr = gn1 ? (p.bsb + w.b * p.bsb_bstride + col0 + 4 * lane)
                                  : (p.bsb + w.b * p.bsb_bstride + nblk * p.stride_sfb);
        const bool sb_lane_ok = gn1 ? (4 * lane < NC && col0 + 4 * lane < p.N) : (col0 < p.N);
        auto load_sa = [&](int kb) -> float { return (row_ok && kb < w.kb1) ? __ldg(sa_ptr + kb * p.stride_sfa) : 0.f; };
        auto load_sb = [&](int kb) -> float4 {
          float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
          if (kb < w.kb1 && sb_lane_ok) {
            if (gn1) r = __ldg(reinterpret_cast<const float4*>(sb_ptr + kb * p.stride_sfb));
            else r.x = __ldg(sb_ptr + kb);
          }
          return r;
        };
        float sa0 = load_sa(w.kb0), sa1 = load_sa(w.kb0 + 1);
        float4 sb0 = load_sb(w.kb0), sb1 = load_sb(w.kb0 + 1);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const float sa = sa0;
          const float4 sb = sb0;
          sa0 = sa1; sb0 = sb1;
          sa1 = load_sa(kb + 2); sb1 = load_sb(kb + 2);
          if (gn1) {
            if (4 * lane < NC) *reinterpret_cast<float4*>(sb_stage + 4 * lane) = sb;
            __syncwarp();
          }
          if (!mbar_wait_spin(&acc_full[as], aph, abort_flag, p.status, kDevTimeoutEpilogue, tmo)) { ok = false; break; }
          tc_fence_after();
          const float s_const = sa * __shfl_sync(0xffffffffu, sb.x, 0);
          // the K block's partial in 32-column groups, one wait per group (64 columns
          // at once would exceed the 168-register budget of a 10-warp CTA)
          constexpr int KBLK = 32;
#pragma unroll
          for (int c = 0; c < NC / KBLK; ++c) {
            uint32_t v[KBLK];
#pragma unroll
            for (int q = 0; q < KBLK / 16; ++q)
              tmem_ld_32x32b_x16(tmem_base + lane_addr + as * kBN + half * NC + c * KBLK + q * 16,
                                 *reinterpret_cast<uint32_t(*)[16]>(&v[q * 16]));
            tc_wait_ld();
            if (gn1) {  // (P * sfb[n]) * sfa[m] + acc
              const float2 sa2 = make_float2(sa, sa);
#pragma unroll
              for (int j = 0; j < KBLK; j += 4) {
                const float4 b4 = *reinterpret_cast<const float4*>(sb_stage + c * KBLK + j);
                float2& a0 = acc2[(c * KBLK + j) / 2];
                float2& a1 = acc2[(c * KBLK + j) / 2 + 1];
                a0 = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])),
                                           make_float2(b4.x, b4.y)), sa2, a0);
                a1 = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])),
                                           make_float2(b4.z, b4.w)), sa2, a1);
              }
            } else {    // P * (sfa[m] * sfb) + acc
              const float2 s2 = make_float2(s_const, s_const);
#pragma unroll
              for (int j = 0; j < KBLK; j += 2) {
                float2& a = acc2[(c * KBLK + j) / 2];
                a = __ffma2_rn(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), s2, a);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[as]);
          if (++as == AS) { as = 0; aph ^= 1; }
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < NC / 2; ++j) { acc[2 * j] = acc2[j].x; acc[2 * j + 1] = acc2[j].y; }
      }

      if constexpr (Cfg::kEpi) {
        if (p.out_mode == kOutStore && m < p.M) {
#pragma unroll
          for (int j = 0; j < NC; j += 4)
            if (col0 + j < p.N)
              epi_apply4<Cfg::kOutF32>(p.epi, w.b, m, col0 + j, acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
      }
      // ---- write the row segment [col0, col0 + NC) of row m
      if (p.tma_store && p.out_mode == kOutStore) {
        tma_store_rows<NC, Cfg::kOutF32, Cfg::kStoreChunkBytes>(&p.tm_c, acc, col0, w.mt * 128 + quad * 32, w.b,
                                                                 stage_c, lane);
      } else if (kMode != kModeBlk && p.out_mode == kOutPeers) {  // the peer entry point is MX only
        peer_store_warp<NC, Cfg::kOutF32>(p, acc, w.mt * 128 + quad * 32, col0, w.mt * p.NT + w.nt, stage_c, lane);
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
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem_base);
  }
}

}  // namespace b2g
