// b2g_api.cu -- C ABI of the B200 FP8 GEMM library (declared in include/b2g/gemm.h).
//
// Host responsibilities: argument validation (status codes, never exit), tile
// selection (the reference's select_kernel algorithm over this library's own
// tile manifest), TMA tensor-map encoding, split-K bookkeeping, per-device
// scratch (split-K workspace, per-call scale re-layout) and the device status
// word the kernels' bounded waits report into.
#include "b2g/gemm.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "b2g_aux.cuh"
#include "b2g_gemm.cuh"
#include "b2g_gemm_pair.cuh"
#include "b2g_gemm_skinny.cuh"
#include "b2g_gemm_skinny_blk.cuh"

using namespace b2g;

// Arrival counters of the skinny (decode) kernel's split tiles: one per
// 128-row weight tile, zero at load, left at zero by every launch that
// completes.  Shared by all calls on a device (they are stream-ordered).
static constexpr int kSkinnyMaxTiles = 8192;  // N <= 1M
static __device__ unsigned long long g_skinny_tile_cnt[kSkinnyMaxTiles];

// Status word of the allocating entry points' kernels: zero at load, set (once,
// by compare-and-swap) by a bounded wait that gives up, read and cleared by
// b2g_device_status.  A file-scope word, so that reading it allocates nothing.
static __device__ int g_status_word;

namespace {

constexpr int kVersion = 100;  // 0.1.0

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

#define B2G_CUDA(call)                                                                  \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(B2G_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                  __FILE__, __LINE__);                                                  \
  } while (0)

std::atomic<unsigned long long> g_timeout_ns{4000ull * 1000000ull};
std::atomic<int> g_static_weights{0};
std::atomic<int> g_force_stall{0};

// ------------------------------------------------------------------ driver entry
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// ------------------------------------------------------------------ per-device state
// Kernels whose dynamic shared-memory attribute has been raised (fixed capacity,
// no heap growth).
struct FnCache {
  const void* fn[64] = {};
  int n = 0;
};

struct DevState {
  bool init = false;
  int sms = 0;
  int* status = nullptr;  // device status word written by bounded waits
  void* ws = nullptr;     // scratch: split-K workspace and per-call scale re-layout
  size_t ws_bytes = 0;
  unsigned long long* tile_cnt = nullptr;  // device address of g_skinny_tile_cnt
  FnCache fns;
};

// Where one GEMM launch gets its SM count, status word and scratch.  The
// allocating entry points draw scratch from DevState (grown with cudaMalloc);
// a fixed environment hands out a caller-independent buffer of fixed size.
struct Env {
  DevState* dev = nullptr;  // allocating path
  int sms = 0;
  int* status = nullptr;
  FnCache* fns = nullptr;
  unsigned long long* tile_cnt = nullptr;
  uint8_t* fixed_ws = nullptr;  // non-null: scratch of fixed capacity, never allocated
  size_t fixed_ws_bytes = 0;
};

// device address of the skinny kernel's tile counters on the current device
int skinny_counters(unsigned long long** out) {
  void* ptr = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&ptr, g_skinny_tile_cnt);
  if (err != cudaSuccess || !ptr)
    return fail(B2G_ERR_CUDA, "cudaGetSymbolAddress(tile counters) failed: %s", cudaGetErrorString(err));
  *out = static_cast<unsigned long long*>(ptr);
  return B2G_OK;
}

std::mutex g_mu;
DevState g_dev[64];

int device_state(DevState** out, int* dev_out = nullptr) {
  int dev = 0;
  B2G_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_NO_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DevState& d = g_dev[dev];
  if (!d.init) {
    int major = 0;
    B2G_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return fail(B2G_ERR_NO_DEVICE, "device %d is sm_%d0; this library targets sm_100a", dev, major);
    B2G_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    void* sw = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&sw, g_status_word);
    if (err != cudaSuccess || !sw)
      return fail(B2G_ERR_CUDA, "cudaGetSymbolAddress(status word) failed: %s", cudaGetErrorString(err));
    d.status = static_cast<int*>(sw);
    int rc = skinny_counters(&d.tile_cnt);
    if (rc) return rc;
    d.init = true;
  }
  *out = &d;
  if (dev_out) *dev_out = dev;
  return B2G_OK;
}

// Grow-only per-device scratch.  Growing frees the old block with cudaFree,
// which waits for outstanding device work, so no kernel still reads it.
int workspace(DevState* d, size_t bytes, void** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (d->ws_bytes < bytes) {
    if (d->ws) B2G_CUDA(cudaFree(d->ws));
    d->ws = nullptr;
    d->ws_bytes = 0;
    size_t want = std::max(bytes, size_t(1) << 20);
    if (cudaMalloc(&d->ws, want) != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(B2G_ERR_WORKSPACE, "could not allocate %zu bytes of scratch", want);
    }
    d->ws_bytes = want;
  }
  *out = d->ws;
  return B2G_OK;
}

int ensure_smem_attr(FnCache* c, const void* fn, int bytes) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < c->n; ++i)
      if (c->fn[i] == fn) return B2G_OK;
  }
  B2G_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  std::lock_guard<std::mutex> lk(g_mu);
  if (c->n < 64) c->fn[c->n++] = fn;
  return B2G_OK;
}

Env env_of(DevState* d) {
  Env e;
  e.dev = d;
  e.sms = d->sms;
  e.status = d->status;
  e.fns = &d->fns;
  e.tile_cnt = d->tile_cnt;
  return e;
}

// Scratch of `bytes` for one call: the fixed buffer when the environment has
// one (too small -> B2G_ERR_WORKSPACE), else the per-device grow-only block.
int env_workspace(const Env& e, size_t bytes, void** out) {
  if (e.fixed_ws) {
    if (bytes > e.fixed_ws_bytes)
      return fail(B2G_ERR_WORKSPACE, "this call needs %zu bytes of scratch; the fixed scratch array holds %zu",
                  bytes, e.fixed_ws_bytes);
    *out = e.fixed_ws;
    return B2G_OK;
  }
  return workspace(e.dev, bytes, out);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int cdiv(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }
inline int grid_for(long long work, int per_block, int sms) {
  long long g = (work + per_block - 1) / per_block;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(g, 8LL * sms)));
}

// ------------------------------------------------------------------ tile manifest
struct TileCfg {
  int tile_m, tile_n, splitk, bpre;
  const char* name;
};
// Same columns as the reference manifest f4gemm_bf16_per1x32Fp4.csv
// (tile_M, tile_N, splitK, bpreshuffle, knl_name), one row per kernel variant.
// tile_M = 256 rows are the CTA-pair kernel (two SMs per tile).
const TileCfg kManifest[] = {
    {128, 256, 1, 0, "b2g_sm100a_fp8_128x256"},
    {128, 128, 1, 0, "b2g_sm100a_fp8_128x128"},
    {128, 256, 1, 1, "b2g_sm100a_fp8_128x256_bpreshuffle"},
    {128, 128, 1, 1, "b2g_sm100a_fp8_128x128_bpreshuffle"},
    {256, 256, 1, 0, "b2g_sm100a_fp8_pair_256x256"},
    {256, 256, 1, 1, "b2g_sm100a_fp8_pair_256x256_bpreshuffle"},
};
constexpr int kManifestN = sizeof(kManifest) / sizeof(kManifest[0]);

// The reference heuristic (asm_f4gemm/f4gemm.hpp:210-267): fewest waves of
// ceil(tiles * splitK / num_sm); ties go to fewer idle SMs, then to the larger
// tile_m*tile_n/(tile_m+tile_n); manifest order breaks remaining ties.
void select_tile(int M, int N, int num_sm, int log2_k_split, int bpreshuffle, int* idx, int* log2_out,
                 int max_tile_n = 1 << 30, int max_tile_m = 1 << 30, int only = -1) {
  uint32_t empty_cu = static_cast<uint32_t>(num_sm);
  uint32_t round = 0xffffffffu;
  float effi = 1.0f;
  const int split_en = log2_k_split > 0 ? 1 : 0;
  const int bpre_en = bpreshuffle ? 1 : 0;
  int sel = -1, sel_split = 1;
  for (int i = 0; i < kManifestN; ++i) {
    const TileCfg& c = kManifest[i];
    if (only >= 0 && i != only) continue;
    if (c.bpre != bpre_en || c.splitk < split_en || c.tile_n > max_tile_n || c.tile_m > max_tile_m) continue;
    if (c.tile_m == 128 && c.tile_n == 512 && (N % c.tile_n) != 0) continue;
    int cand[4], nc = 0;
    if (log2_k_split >= 0 && c.splitk) cand[nc++] = 1 << log2_k_split;
    else if (c.splitk) { cand[0] = 2; cand[1] = 4; cand[2] = 8; cand[3] = 16; nc = 4; }
    else cand[nc++] = 1;
    for (int j = 0; j < nc; ++j) {
      const int sk = cand[j];
      const uint32_t tg = static_cast<uint32_t>(((M + c.tile_m - 1) / c.tile_m) * ((N + c.tile_n - 1) / c.tile_n) * sk);
      const uint32_t lr = (tg + num_sm - 1) / num_sm;
      const float le = static_cast<float>(c.tile_m) * c.tile_n / (c.tile_m + c.tile_n);
      const bool earlier = lr < round, same = lr == round;
      const bool more_busy = empty_cu > (lr * static_cast<uint32_t>(num_sm) - tg);
      const bool better = le > effi;
      if (earlier || (same && (more_busy || better))) {
        round = lr;
        empty_cu = lr * static_cast<uint32_t>(num_sm) - tg;
        effi = le;
        sel = i;
        sel_split = sk;
      }
    }
  }
  int l = 0;
  while (sel_split >>= 1) ++l;
  *idx = sel;
  *log2_out = l;
}

// ------------------------------------------------------------------ tensor maps
int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B2G_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled rejected a %d-D map (error %d)", rank, (int)r);
  return B2G_OK;
}

// ------------------------------------------------------------------ generic launch
struct Req {
  int mode = kModePlain;
  int bn = 0;  // 0: heuristic
  bool bpre = false;
  bool out_f32 = false;
  int M = 0, N = 0, K = 0, batch = 1;
  const void* a = nullptr;
  long long lda = 0, a_bstride = 0;  // bytes
  const void* b = nullptr;
  long long ldb = 0, b_bstride = 0;  // bytes
  void* c = nullptr;
  long long ldc = 0, c_bstride = 0;  // elements
  float alpha = 1.f;
  const uint8_t* sfa = nullptr;
  const uint8_t* sfb = nullptr;
  long long sfa_bstride = 0, sfb_bstride = 0;
  const float* bsa = nullptr;
  const float* bsb = nullptr;
  long long stride_sfa = 0, stride_sfb = 0, bsa_bstride = 0, bsb_bstride = 0;
  int group_n = 128;
  int log2_k_split = 0;
  size_t ws_offset = 0;  // scratch bytes already claimed by the caller of run_gemm
  cudaStream_t stream = nullptr;
  // column-parallel output into every GPU's full C (b2g_gemm_mxfp8_peer_out)
  void* const* peer_c = nullptr;
  int n_peers = 0, peer_self = 0;
  long long peer_ldc = 0, peer_col0 = 0;
  long long peer_shard = 0;  // all-to-all output (b2g_gemm_mxfp8_a2a_out): columns per peer
  // beta * C and a per-column bias (b2g_epilogue), in the output's element type
  EpiTerms epi = {};
};

template <class Cfg>
int launch_cfg(const Env& d, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
               cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&b2g_gemm_kernel<Cfg>);
  int rc = ensure_smem_attr(d.fns, fn, Cfg::kSmemBytes);
  if (rc) return rc;
  b2g_gemm_kernel<Cfg><<<grid, Cfg::kThreads, Cfg::kSmemBytes, st>>>(ta, tb, p);
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

template <int kMode, int kBN>
int dispatch_pre_out(const Env& d, bool pre, bool f32, const CUtensorMap& ta, const CUtensorMap& tb,
                     const GemmParams& p, int grid, cudaStream_t st) {
  // beta * C / bias in the epilogue: separate instances (MX modes, 256-wide tiles),
  // so the kernels without the terms compile exactly as before
  if constexpr (mode_mx(kMode) && kBN == 256) {
    if (epi_any(p.epi) && p.out_mode == kOutStore) {
      if (pre)
        return f32 ? launch_cfg<GemmCfg<kMode, 256, true, true, true>>(d, ta, tb, p, grid, st)
                   : launch_cfg<GemmCfg<kMode, 256, true, false, true>>(d, ta, tb, p, grid, st);
      return f32 ? launch_cfg<GemmCfg<kMode, 256, false, true, true>>(d, ta, tb, p, grid, st)
                 : launch_cfg<GemmCfg<kMode, 256, false, false, true>>(d, ta, tb, p, grid, st);
    }
  }
  if (epi_any(p.epi) && p.out_mode == kOutStore)
    return fail(B2G_ERR_UNSUPPORTED, "beta * C / bias epilogue: MX modes with 256-wide tiles only");
  if (kMode == kModeBlk) {  // blockwise path: row-major B only; instances per weight-scale layout
    if (p.group_n == 1)
      return f32 ? launch_cfg<GemmCfg<kMode, kBN, false, true, false, true>>(d, ta, tb, p, grid, st)
                 : launch_cfg<GemmCfg<kMode, kBN, false, false, false, true>>(d, ta, tb, p, grid, st);
    return f32 ? launch_cfg<GemmCfg<kMode, kBN, false, true>>(d, ta, tb, p, grid, st)
               : launch_cfg<GemmCfg<kMode, kBN, false, false>>(d, ta, tb, p, grid, st);
  } else {
    if (pre)
      return f32 ? launch_cfg<GemmCfg<kMode, kBN, true, true>>(d, ta, tb, p, grid, st)
                 : launch_cfg<GemmCfg<kMode, kBN, true, false>>(d, ta, tb, p, grid, st);
    return f32 ? launch_cfg<GemmCfg<kMode, kBN, false, true>>(d, ta, tb, p, grid, st)
               : launch_cfg<GemmCfg<kMode, kBN, false, false>>(d, ta, tb, p, grid, st);
  }
}

template <int kMode>
int dispatch_bn(const Env& d, int bn, bool pre, bool f32, const CUtensorMap& ta, const CUtensorMap& tb,
                const GemmParams& p, int grid, cudaStream_t st) {
  // (the 256-wide blockwise tile runs its 12-warp register split, GemmCfg::kWide)
  if (bn == 256) return dispatch_pre_out<kMode, 256>(d, pre, f32, ta, tb, p, grid, st);
  if (bn != 128) return fail(B2G_ERR_UNSUPPORTED, "no single-CTA kernel of width %d", bn);
  return dispatch_pre_out<kMode, 128>(d, pre, f32, ta, tb, p, grid, st);
}

template <class Cfg>
int launch_pair(const Env& d, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                const CUtensorMap& tsb, const PairParams& pp, cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&b2g_gemm_pair_kernel<Cfg>);
  int rc = ensure_smem_attr(d.fns, fn, Cfg::kSmemBytes);
  if (rc) return rc;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * pp.num_pairs, 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2G_CUDA(cudaLaunchKernelEx(&cfg, b2g_gemm_pair_kernel<Cfg>, ta, tb, tsa, tsb, pp));
  return B2G_OK;
}

int dispatch_pair(const Env& d, int mode, int bn, bool pre, bool f32, const CUtensorMap& ta, const CUtensorMap& tb,
                  const CUtensorMap& tsa, const CUtensorMap& tsb, const PairParams& pp, cudaStream_t st) {
  if (bn != 256) return fail(B2G_ERR_UNSUPPORTED, "no pair kernel of width %d", bn);
  if (epi_any(pp.g.epi) && pp.g.out_mode == kOutStore) {  // instances with the beta * C / bias terms
    if (mode == kModeMX4) {
      if (pre) return f32 ? launch_pair<PairCfg<kModeMX4, 256, true, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                          : launch_pair<PairCfg<kModeMX4, 256, true, false, true>>(d, ta, tb, tsa, tsb, pp, st);
      return f32 ? launch_pair<PairCfg<kModeMX4, 256, false, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                 : launch_pair<PairCfg<kModeMX4, 256, false, false, true>>(d, ta, tb, tsa, tsb, pp, st);
    }
    if (mode == kModeMX) {
      if (pre) return f32 ? launch_pair<PairCfg<kModeMX, 256, true, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                          : launch_pair<PairCfg<kModeMX, 256, true, false, true>>(d, ta, tb, tsa, tsb, pp, st);
      return f32 ? launch_pair<PairCfg<kModeMX, 256, false, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                 : launch_pair<PairCfg<kModeMX, 256, false, false, true>>(d, ta, tb, tsa, tsb, pp, st);
    }
    return fail(B2G_ERR_UNSUPPORTED, "beta * C / bias epilogue: MX modes only");
  }
  if (mode == kModeMX4) {
    if (pre) return f32 ? launch_pair<PairCfg<kModeMX4, 256, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                        : launch_pair<PairCfg<kModeMX4, 256, true, false>>(d, ta, tb, tsa, tsb, pp, st);
    return f32 ? launch_pair<PairCfg<kModeMX4, 256, false, true>>(d, ta, tb, tsa, tsb, pp, st)
               : launch_pair<PairCfg<kModeMX4, 256, false, false>>(d, ta, tb, tsa, tsb, pp, st);
  }
  if (mode == kModeMX) {
    if (pre) return f32 ? launch_pair<PairCfg<kModeMX, 256, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                        : launch_pair<PairCfg<kModeMX, 256, true, false>>(d, ta, tb, tsa, tsb, pp, st);
    return f32 ? launch_pair<PairCfg<kModeMX, 256, false, true>>(d, ta, tb, tsa, tsb, pp, st)
               : launch_pair<PairCfg<kModeMX, 256, false, false>>(d, ta, tb, tsa, tsb, pp, st);
  }
  if (pre) return f32 ? launch_pair<PairCfg<kModePlain, 256, true, true>>(d, ta, tb, tsa, tsb, pp, st)
                      : launch_pair<PairCfg<kModePlain, 256, true, false>>(d, ta, tb, tsa, tsb, pp, st);
  return f32 ? launch_pair<PairCfg<kModePlain, 256, false, true>>(d, ta, tb, tsa, tsb, pp, st)
             : launch_pair<PairCfg<kModePlain, 256, false, false>>(d, ta, tb, tsa, tsb, pp, st);
}

// B2G_SYNC_CHECK=1: wait for the call's kernels and report (and clear) the
// status word of the environment they ran in -- the allocating path's word or
// the no-alloc array's.  A nonzero word also zeroes the decode kernel's tile
// counters, which a launch that stopped early can leave mid-count.  Allocates
// nothing.
int maybe_sync_check(const Env& e) {
  static const bool on = [] {
    const char* v = getenv("B2G_SYNC_CHECK");
    return v && v[0] == '1';
  }();
  if (!on) return B2G_OK;
  int st = 0;
  B2G_CUDA(cudaDeviceSynchronize());
  B2G_CUDA(cudaMemcpy(&st, e.status, sizeof(int), cudaMemcpyDeviceToHost));
  if (!st) return B2G_OK;
  B2G_CUDA(cudaMemset(e.status, 0, sizeof(int)));
  B2G_CUDA(cudaMemset(e.tile_cnt, 0, sizeof(unsigned long long) * kSkinnyMaxTiles));
  return fail(B2G_ERR_DEVICE_TIMEOUT, "kernel reported device status %d", st);
}

// Tile width, split count and K-blocks per split for a request.
// Widest single-CTA tile of the blockwise mode.  For more than 128 rows the
// 12-warp 256-wide tile runs 30-43 % faster than the 128-wide one at C3's shapes
// with 128x128 weight scales (M = 1024..16384) and 23-40 % faster with per-column
// weight scales (GROUP_N = 1); at M = 128 (split-K, HBM-bound) the 128-wide tile's
// four TMEM partial buffers win on two of C3's three shapes.  B2G_BLK_BN=128 or
// 256 sets the width for every blockwise GEMM.
int blk_max_bn(const Req& r) {
  static const int force = [] {
    const char* v = getenv("B2G_BLK_BN");
    const int w = v ? atoi(v) : 0;
    return (w == 128 || w == 256) ? w : 0;
  }();
  if (force) return force;
  return r.M <= 128 ? 128 : 256;
}

// B2G_FORCE_TILE=<manifest knl_name>: run that manifest entry (and only its
// split choices) for every request it can serve -- the analogue of the reference
// host's `--kernel <co>` (asm_f4gemm/main.cpp), used by the regression sweep.
// Read at every call.  Returns the entry, -1 when unset, -2 for an unknown name.
int forced_tile() {
  const char* v = getenv("B2G_FORCE_TILE");
  if (!v || !*v) return -1;
  for (int i = 0; i < kManifestN; ++i)
    if (!strcmp(kManifest[i].name, v)) return i;
  return -2;
}

int plan_tiles(const Req& r, int sms, int* bn_out, int* S_out, int* kb_per_out, int* bm_out = nullptr) {
  int bn = r.bn, l2 = r.log2_k_split, bm = 128;
  if (r.mode == kModeBlk && bn > blk_max_bn(r)) bn = blk_max_bn(r);
  if (bn == 0) {
    // The pair tile wastes half its rows at M <= 128 and the blockwise mode has no
    // pair kernel: those select among the single-CTA entries only.
    static const bool pair_off = [] {
      const char* v = getenv("B2G_DISABLE_PAIR");
      return v && v[0] == '1';
    }();
    const bool pair_ok = r.M > 128 && r.mode != kModeBlk && !pair_off;
    const int only = forced_tile();
    if (only == -2) return fail(B2G_ERR_INVALID_ARG, "B2G_FORCE_TILE names no manifest entry");
    int idx = -1, lsel = 0;
    select_tile(r.M, r.N, sms, r.log2_k_split, r.bpre ? 1 : 0, &idx, &lsel, r.mode == kModeBlk ? blk_max_bn(r) : 1 << 30,
                pair_ok ? 1 << 30 : 128, only);
    if (idx < 0 && only >= 0)
      return fail(B2G_ERR_UNSUPPORTED, "B2G_FORCE_TILE=%s cannot serve this request (B layout, mode or M)",
                  kManifest[only].name);
    if (idx < 0) return fail(B2G_ERR_UNSUPPORTED, "no tile in the manifest fits");
    bn = kManifest[idx].tile_n;
    bm = kManifest[idx].tile_m;
    l2 = lsel;
  }
  // the widths the kernels are compiled for: pair 256, single CTA 256 / 128
  if (bm == 256) bn = 256;
  else bn = (bn == 256 && (r.mode != kModeBlk || blk_max_bn(r) == 256)) ? 256 : 128;
  if (r.mode == kModeBlk && bm == 128 && getenv("B2G_BLK_BN")) bn = blk_max_bn(r);  // a forced width
  if (bm_out) *bm_out = bm;
  if (l2 < 0) l2 = 0;
  if (l2 > 8) return fail(B2G_ERR_INVALID_ARG, "log2_k_split %d too large", l2);
  const int KB = cdiv(r.K, 128);
  int S = std::min(1 << l2, KB);
  const int kb_per = cdiv(KB, S);
  S = cdiv(KB, kb_per);
  *bn_out = bn;
  *S_out = S;
  *kb_per_out = kb_per;
  return B2G_OK;
}

// Bytes between 128-row blocks of a tensor-core scale-atom buffer: one 512-byte
// atom per 128 elements of K (an MXFP4 request's K counts bytes, two elements each).
long long sf_row_block_bytes(const Req& r) {
  return static_cast<long long>(cdiv(r.K, 128)) * 512 * (r.mode == kModeMX4 ? 2 : 1);
}

// Blockwise GEMMs with 32 < M <= 128 and a long K run the blockwise decode kernel
// untransposed (rows of A on the MMA's M): every SM streams an equal share of B
// (stream-K) instead of the single-CTA kernel's one CTA per 128-column tile.  Its
// per-call cost (about 3 us of prologue and the split-tile fix-up) only pays back
// over enough K blocks.  Measured on B200 (graph replay, L2 flushed; M = 64 / 100 /
// 128, N = 4096..28672): with 128 x 128 weight scales it wins from K/128 = 56 on
// (K = 7168: 25.7 against 26.8 us; K = 18432: 45.9 against 64.0 us) and loses at
// K <= 4096 (K = 2048: 19.6 against 11.2 us); with per-column scales it wins from
// K/128 = 32 (K = 18432: 54.9 against 128.7 us, 128 x 28672 x 4096: 48 against
// 64 us).  B2G_BLK_NT=0 / 1 forces either route (read at every call).
bool skinny_blk_nt(const Req& r) {
  if (r.mode != kModeBlk || r.M > 128 || r.batch != 1) return false;
  const char* v = getenv("B2G_BLK_NT");
  if (v && v[0] == '0') return false;
  if (v && v[0] == '1') return r.M > 16;
  const int kb = r.K / 128;
  return r.M > 32 && (kb >= 48 || (r.group_n == 1 && kb >= 32));
}

// Few rows of A (decode): the transposed stream-K kernel.
bool use_skinny(const Req& r, int sms) {
  static const bool off = [] {
    const char* v = getenv("B2G_DISABLE_SKINNY");
    return v && v[0] == '1';
  }();
  if (off || r.M > 128 || r.batch != 1 || r.n_peers || cdiv(r.N, 128) > kSkinnyMaxTiles) return false;
  // The blockwise decode kernel folds every K block's partial into registers, one
  // 32-column TMEM load at a time.  Measured against the single-CTA kernel it wins
  // only for at most 32 rows of A and more 128-row tiles than SMs (the single-CTA
  // kernel then needs a second, partial wave).  It TMA-loads the scale rows, which
  // must start on 16 bytes.
  if (r.mode == kModeBlk) {
    const bool scales_ok = r.stride_sfa % 4 == 0 && aligned16(r.bsa) &&
                           (r.group_n == 1 || (r.stride_sfb % 4 == 0 && aligned16(r.bsb)));
    return scales_ok && ((r.M <= 32 && cdiv(r.N, 128) > sms) || skinny_blk_nt(r));
  }
  return true;
}

// B2G_DISABLE_PDL=1 launches without programmatic stream serialization.
bool use_pdl() {
  static const bool off = [] {
    const char* v = getenv("B2G_DISABLE_PDL");
    return v && v[0] == '1';
  }();
  return !off;
}

int skinny_mp(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }
// rows of A per stage of a decode launch: M rounded up, or all 128 MMA rows untransposed
int skinny_rows(const Req& r) { return skinny_blk_nt(r) ? 128 : skinny_mp(r.M); }


// 128-K blocks per ring stage: two (one 32 KB request of B) when K splits into
// whole pairs of blocks and the stage still leaves room for a deep ring.
int skinny_kkb(const Req& r) { return (r.K % 256 == 0 && skinny_rows(r) <= 64) ? 2 : 1; }

long long skinny_units(const Req& r) {
  return static_cast<long long>(cdiv(r.N, 128)) * (cdiv(r.K, 128) / skinny_kkb(r));
}

// Whole tiles per CTA of a decode launch on G CTAs: NT / G, one less when the
// leftover tiles would give each CTA under half a tile of stream-K work (many
// pieces per tile).  The blockwise kernel splits every tile stream-K.
int skinny_dp_w(const Req& r, int NT, int G) {
  int dp_w = r.mode == kModeBlk ? 0 : NT / G;
  if (dp_w > 0 && 2 * (NT - dp_w * G) < G) --dp_w;
  return dp_w;
}

// CTAs of a decode launch.  Measured on B200 with two 128-K blocks per stage
// (M <= 64) and at least 8 stages per tile (the C4 decode shapes, 16 x 57344 x
// 8192, 16 x 16384 x 3584): a grid whose stream-K units split evenly (every CTA
// the same number of units, tiles cut into fewer pieces) beats one CTA per SM with
// uneven shares by 2-17 %, down to about 0.85 x the SM count.  Where a CTA's
// work is dominated by per-tile costs instead (M = 128: one K block per stage and
// a 64 KB output tile; K = 1024: four stages per tile) the extra tiles per CTA
// cost 3-15 %, and the blockwise kernel was not measured: those keep one CTA per
// SM.  So: the largest even-split grid in [0.85 * sms, sms] when it applies, else
// sms.  B2G_SKINNY_GRID=<n> forces n CTAs (tuning).
int skinny_grid(const Req& r, int sms, int NT, int KG) {
  static const int forced = [] {
    const char* v = getenv("B2G_SKINNY_GRID");
    return v ? atoi(v) : 0;
  }();
  const long long units = static_cast<long long>(NT) * KG;
  if (units <= sms) return static_cast<int>(units);
  if (forced > 0) return std::min(forced, sms);
  if (r.mode == kModeBlk || skinny_kkb(r) != 2 || KG < 8) return sms;
  for (int G = sms; 20 * G >= 17 * sms; --G)
    if ((static_cast<long long>(NT - skinny_dp_w(r, NT, G) * G) * KG) % G == 0) return G;
  return sms;
}

// Scratch bytes run_gemm will ask for beyond r.ws_offset.
size_t split_ws_bytes(const Req& r, int S, int sms) {
  if (use_skinny(r, sms)) {  // fp32 partial slots, two per CTA
    const long long grid = std::min<long long>(skinny_units(r), sms);
    return static_cast<size_t>(2 * grid) * skinny_rows(r) * 128 * 4;
  }
  // fp32 output adds its split-K partials into C in place, unless the epilogue has
  // beta * C or bias terms: those go through the workspace and the reduce
  return (S > 1 && (!r.out_f32 || epi_any(r.epi))) ? static_cast<size_t>(S) * r.batch * r.M * r.N * 4 : 0;
}

template <class Cfg>
int launch_skinny(const Env& d, const CUtensorMap& tw, const CUtensorMap& ta, const SkinnyParams& sp, int grid,
                  cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&b2g_gemm_skinny_kernel<Cfg>);
  int rc = ensure_smem_attr(d.fns, fn, Cfg::kSmemBytes);
  if (rc) return rc;
  // programmatic dependent launch: this kernel's prologue overlaps the tail of
  // the previous kernel on the stream (the kernel waits before touching memory)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = use_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SkinnyParams spl = sp;
  if (spl.cluster_fold > 1) {
    // clusters of k CTAs, only if the whole grid fits on the GPU at once (the pieces of
    // a tile wait for one another); otherwise the L2 fold
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = spl.cluster_fold;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    static std::atomic<int> fit_k[5] = {-1, -1, -1, -1, -1};  // clusters that fit at once, per k (queried once)
    int fit = fit_k[spl.cluster_fold].load();
    if (fit < 0) {
      if (cudaOccupancyMaxActiveClusters(&fit, b2g_gemm_skinny_kernel<Cfg>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        fit = 0;
      }
      fit_k[spl.cluster_fold].store(fit);
    }
    if (fit * spl.cluster_fold < grid) {
      spl.cluster_fold = 0;
      cfg.numAttrs = 1;
    }
  }
  B2G_CUDA(cudaLaunchKernelEx(&cfg, b2g_gemm_skinny_kernel<Cfg>, tw, ta, spl));
  return B2G_OK;
}

template <class Cfg>
int launch_skinny_blk(const Env& d, const CUtensorMap& tw, const CUtensorMap& ta, const CUtensorMap& tsa,
                      const CUtensorMap& tsb, const SkinnyParams& sp, int grid, cudaStream_t st) {
  const void* fn = reinterpret_cast<const void*>(&b2g_gemm_skinny_blk_kernel<Cfg>);
  int rc = ensure_smem_attr(d.fns, fn, Cfg::kSmemBytes);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = use_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2G_CUDA(cudaLaunchKernelEx(&cfg, b2g_gemm_skinny_blk_kernel<Cfg>, tw, ta, tsa, tsb, sp));
  return B2G_OK;
}

int dispatch_skinny_blk(const Env& d, int mp, int kkb, bool nt, const CUtensorMap& tw, const CUtensorMap& ta,
                        const CUtensorMap& tsa, const CUtensorMap& tsb, const SkinnyParams& sp, int grid,
                        cudaStream_t st) {
  if (nt) return launch_skinny_blk<SkinnyBlkCfg<128, 1, true>>(d, tw, ta, tsa, tsb, sp, grid, st);
  if (kkb == 2) {
    switch (mp) {
      case 16: return launch_skinny_blk<SkinnyBlkCfg<16, 2>>(d, tw, ta, tsa, tsb, sp, grid, st);
      case 32: return launch_skinny_blk<SkinnyBlkCfg<32, 2>>(d, tw, ta, tsa, tsb, sp, grid, st);
      default: return launch_skinny_blk<SkinnyBlkCfg<64, 2>>(d, tw, ta, tsa, tsb, sp, grid, st);
    }
  }
  switch (mp) {
    case 16: return launch_skinny_blk<SkinnyBlkCfg<16, 1>>(d, tw, ta, tsa, tsb, sp, grid, st);
    case 32: return launch_skinny_blk<SkinnyBlkCfg<32, 1>>(d, tw, ta, tsa, tsb, sp, grid, st);
    case 64: return launch_skinny_blk<SkinnyBlkCfg<64, 1>>(d, tw, ta, tsa, tsb, sp, grid, st);
    default: return launch_skinny_blk<SkinnyBlkCfg<128, 1>>(d, tw, ta, tsa, tsb, sp, grid, st);
  }
}

template <int kMode, bool kPre>
int dispatch_skinny_mp(const Env& d, int mp, int kkb, const CUtensorMap& tw, const CUtensorMap& ta,
                       const SkinnyParams& sp, int grid, cudaStream_t st) {
  if (kkb == 2) {
    switch (mp) {
      case 16: return launch_skinny<SkinnyCfg<kMode, 16, kPre, 2>>(d, tw, ta, sp, grid, st);
      case 32: return launch_skinny<SkinnyCfg<kMode, 32, kPre, 2>>(d, tw, ta, sp, grid, st);
      default: return launch_skinny<SkinnyCfg<kMode, 64, kPre, 2>>(d, tw, ta, sp, grid, st);
    }
  }
  switch (mp) {
    case 16: return launch_skinny<SkinnyCfg<kMode, 16, kPre, 1>>(d, tw, ta, sp, grid, st);
    case 32: return launch_skinny<SkinnyCfg<kMode, 32, kPre, 1>>(d, tw, ta, sp, grid, st);
    case 64: return launch_skinny<SkinnyCfg<kMode, 64, kPre, 1>>(d, tw, ta, sp, grid, st);
    default: return launch_skinny<SkinnyCfg<kMode, 128, kPre, 1>>(d, tw, ta, sp, grid, st);
  }
}

std::atomic<unsigned long long> g_skinny_tag{0};

int run_skinny(const Req& r, const Env& d) {
  int rc = B2G_OK;
  const int mp = skinny_rows(r);
  const int kkb = skinny_kkb(r);
  SkinnyParams sp;
  memset(&sp, 0, sizeof(sp));
  sp.M = r.M; sp.N = r.N; sp.K = r.K;
  sp.out = r.c;
  sp.ldo = r.ldc;
  sp.out_f32 = r.out_f32 ? 1 : 0;
  sp.alpha = r.alpha;
  sp.epi = r.epi;
  sp.sfw = r.sfb;
  sp.sfa = r.sfa;
  sp.sf_rb = sf_row_block_bytes(r);
  sp.NT = cdiv(r.N, 128);
  sp.KG = cdiv(r.K, 128) / kkb;
  sp.kview = r.K % 128 == 0 ? 1 : 0;
  const int grid = skinny_grid(r, d.sms, sp.NT, sp.KG);
  // Whole tiles per CTA, worked after the stream-K units so that every split
  // tile's fix-up overlaps streaming.
  const int dp_w = skinny_dp_w(r, sp.NT, grid);
  sp.dp_w = dp_w;
  sp.sk_tiles = sp.NT - dp_w * grid;
  sp.units = static_cast<long long>(sp.sk_tiles) * sp.KG;
  sp.cnt = d.tile_cnt;
  // tags are nonzero and below 2^48 (the counter keeps 16 bits of arrivals)
  sp.tag = (g_skinny_tag.fetch_add(1) % ((1ull << 48) - 1)) + 1;
  sp.status = d.status;
  sp.timeout_ns = g_timeout_ns.load();
  sp.debug_stall = g_force_stall.load();
  sp.w_early = (g_static_weights.load() && use_pdl() && r.mode != kModeBlk) ? 1 : 0;
  // Every tile split into k equal pieces, one per CTA, k CTAs per tile (the C4 long-K
  // shapes: 32 tiles x 4 pieces on 128 CTAs): launch in clusters of k and let the
  // pieces meet in the rank-0 CTA's shared memory (B2G_CLUSTER_FOLD=0 turns it off).
  {
    static const bool off = [] {
      const char* v = getenv("B2G_CLUSTER_FOLD");
      return v && v[0] == '0';
    }();
    sp.cluster_fold = 0;
    if (!off && r.mode != kModeBlk && mp == 16 && dp_w == 0 && sp.sk_tiles == sp.NT && grid % sp.NT == 0) {
      const int k = grid / sp.NT;
      if ((k == 2 || k == 4) && sp.KG % k == 0) sp.cluster_fold = k;
    }
  }
  sp.bsa = r.bsa;
  sp.bsb = r.bsb;
  sp.stride_sfa = r.stride_sfa;
  sp.stride_sfb = r.stride_sfb;
  sp.group_n = r.group_n;

  // Operand maps.  With K % 128 == 0 they view a row-major [rows][K] operand as
  // (128 bytes, rows, K/128 blocks) so one box brings kkb whole K blocks, each
  // landing as its own [rows][128 B] swizzled tile; otherwise (kkb == 1) plain
  // (K, rows) maps whose out-of-range tail reads as zero.
  CUtensorMap tw, ta;
  const long long kb_total = cdiv(r.K, 128);
  if (!r.bpre) {
    if (sp.kview) {
      cuuint64_t dims[3] = {128, (cuuint64_t)r.N, (cuuint64_t)kb_total};
      cuuint64_t str[2] = {(cuuint64_t)r.ldb, 128};
      cuuint32_t box[3] = {128, 128, (cuuint32_t)kkb};
      rc = encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, r.b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
      cuuint64_t dims[3] = {(cuuint64_t)r.K, (cuuint64_t)r.N, 1};
      cuuint64_t str[2] = {(cuuint64_t)r.ldb, (cuuint64_t)(r.ldb * r.N)};
      cuuint32_t box[3] = {128, 128, 1};
      rc = encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, r.b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
  } else {
    cuuint64_t dims[4] = {256, (cuuint64_t)(r.N / 16), (cuuint64_t)(r.K / 16), 1};
    cuuint64_t str[3] = {(cuuint64_t)16 * r.K, 256, (cuuint64_t)((long long)r.N * r.K)};
    cuuint32_t box[4] = {256, 8, (cuuint32_t)(8 * kkb), 1};
    rc = encode(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, r.b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (rc) return rc;
  if (sp.kview) {
    cuuint64_t dims[3] = {128, (cuuint64_t)r.M, (cuuint64_t)kb_total};
    cuuint64_t str[2] = {(cuuint64_t)r.lda, 128};
    cuuint32_t box[3] = {128, (cuuint32_t)mp, (cuuint32_t)kkb};
    rc = encode(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, r.a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    cuuint64_t dims[3] = {(cuuint64_t)r.K, (cuuint64_t)r.M, 1};
    cuuint64_t str[2] = {(cuuint64_t)r.lda, (cuuint64_t)(r.lda * r.M)};
    cuuint32_t box[3] = {128, (cuuint32_t)mp, 1};
    rc = encode(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, r.a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;

  void* ws = nullptr;
  rc = env_workspace(d, r.ws_offset + split_ws_bytes(r, 1, d.sms), &ws);
  if (rc) return rc;
  sp.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + r.ws_offset);
  if (r.mode == kModeBlk) {
    // fp32 scale rows as 2-D TMA boxes: sfa (MP rows of one K block); sfb the tile's
    // 128 column scales (GROUP_N = 1) or 8 block scales around the K block (GROUP_N = 128)
    CUtensorMap tsa, tsb;
    const long long kbt = r.K / 128;
    {
      cuuint64_t dims[2] = {(cuuint64_t)r.M, (cuuint64_t)kbt};
      cuuint64_t str[1] = {(cuuint64_t)(r.stride_sfa * 4)};
      cuuint32_t box[2] = {(cuuint32_t)mp, 1};
      rc = encode(&tsa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, r.bsa, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    }
    if (r.group_n == 1) {
      cuuint64_t dims[2] = {(cuuint64_t)r.N, (cuuint64_t)kbt};
      cuuint64_t str[1] = {(cuuint64_t)(r.stride_sfb * 4)};
      cuuint32_t box[2] = {128, 1};
      rc = encode(&tsb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, r.bsb, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
      cuuint64_t dims[2] = {(cuuint64_t)kbt, (cuuint64_t)(r.N / 128)};
      cuuint64_t str[1] = {(cuuint64_t)(r.stride_sfb * 4)};
      cuuint32_t box[2] = {8, 1};
      rc = encode(&tsb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, r.bsb, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (rc) return rc;
    rc = dispatch_skinny_blk(d, mp, kkb, skinny_blk_nt(r), tw, ta, tsa, tsb, sp, grid, r.stream);
  }
  else if (r.mode == kModeMX)
    rc = r.bpre ? dispatch_skinny_mp<kModeMX, true>(d, mp, kkb, tw, ta, sp, grid, r.stream)
                : dispatch_skinny_mp<kModeMX, false>(d, mp, kkb, tw, ta, sp, grid, r.stream);
  else if (r.mode == kModeMX4)
    rc = r.bpre ? dispatch_skinny_mp<kModeMX4, true>(d, mp, kkb, tw, ta, sp, grid, r.stream)
                : dispatch_skinny_mp<kModeMX4, false>(d, mp, kkb, tw, ta, sp, grid, r.stream);
  else
    rc = r.bpre ? dispatch_skinny_mp<kModePlain, true>(d, mp, kkb, tw, ta, sp, grid, r.stream)
                : dispatch_skinny_mp<kModePlain, false>(d, mp, kkb, tw, ta, sp, grid, r.stream);
  if (rc) return rc;
  return maybe_sync_check(d);
}

int run_gemm(const Req& r, const Env* fixed_env = nullptr) {
  int rc = B2G_OK;
  if (r.M <= 0 || r.N <= 0 || r.K <= 0 || r.batch <= 0) return fail(B2G_ERR_INVALID_ARG, "non-positive problem size");
  if (!r.a || !r.b || !r.c) return fail(B2G_ERR_INVALID_ARG, "null A/B/C pointer");
  if (r.N % 16) return fail(B2G_ERR_UNSUPPORTED, "N (%d) must be a multiple of 16", r.N);
  if (r.K % 16) return fail(B2G_ERR_UNSUPPORTED, "K (%d) must be a multiple of 16", r.K);
  if (r.mode == kModeMX && r.K % 32) return fail(B2G_ERR_UNSUPPORTED, "MXFP8 needs K %% 32 == 0 (K=%d)", r.K);
  // MXFP4 requests carry K and the strides in bytes (two E2M1 elements per byte)
  if (r.mode == kModeMX4 && r.K % 128)
    return fail(B2G_ERR_UNSUPPORTED, "MXFP4 needs K %% 256 == 0 (K=%d elements)", 2 * r.K);
  if (r.mode == kModeBlk && r.K % 128) return fail(B2G_ERR_UNSUPPORTED, "block-scale GEMM needs K %% 128 == 0 (K=%d)", r.K);
  if (!aligned16(r.a) || !aligned16(r.b) || !aligned16(r.c)) return fail(B2G_ERR_ALIGNMENT, "A/B/C must be 16-byte aligned");
  if (r.lda < r.K || r.lda % 16) return fail(B2G_ERR_ALIGNMENT, "A row stride %lld must be >= K and a multiple of 16", r.lda);
  if (!r.bpre && (r.ldb < r.K || r.ldb % 16)) return fail(B2G_ERR_ALIGNMENT, "B row stride %lld must be >= K and a multiple of 16", r.ldb);
  if (r.bpre && r.K % 32) return fail(B2G_ERR_UNSUPPORTED, "preshuffled B needs K %% 32 == 0");
  const int esz = r.out_f32 ? 4 : 2;
  if (r.ldc < r.N || (r.ldc * esz) % 16) return fail(B2G_ERR_ALIGNMENT, "C row stride %lld must be >= N and 16-byte aligned", r.ldc);
  if (r.batch > 1 && (r.a_bstride % 16 || r.b_bstride % 16 || (r.c_bstride * esz) % 16))
    return fail(B2G_ERR_ALIGNMENT, "batch strides must be 16-byte multiples");
  if (epi_any(r.epi)) {
    if (!mode_mx(r.mode)) return fail(B2G_ERR_UNSUPPORTED, "beta * C / bias terms: MX modes only");
    if (r.n_peers) return fail(B2G_ERR_UNSUPPORTED, "the peer-store output takes no beta or bias term");
    if (r.epi.cin && (!aligned16(r.epi.cin) || r.epi.ldcin < r.N || (r.epi.ldcin * esz) % 16 ||
                      (r.batch > 1 && (r.epi.cin_bstride * esz) % 16)))
      return fail(B2G_ERR_ALIGNMENT, "C input needs a 16-byte aligned base, row pitch >= N and whole 16-byte pitches");
    if (r.epi.bias && (!aligned16(r.epi.bias) || (r.epi.bias_bstride * esz) % 16))
      return fail(B2G_ERR_ALIGNMENT, "bias needs a 16-byte aligned base and batch stride");
  }
  if (mode_mx(r.mode)) {
    if (!r.sfa || !r.sfb) return fail(B2G_ERR_INVALID_ARG, "null scale pointer");
    if (!aligned16(r.sfa) || !aligned16(r.sfb) || r.sfa_bstride % 16 || r.sfb_bstride % 16)
      return fail(B2G_ERR_ALIGNMENT, "scale buffers must be 16-byte aligned");
  }
  if (r.mode == kModeBlk) {
    if (!r.bsa || !r.bsb) return fail(B2G_ERR_INVALID_ARG, "null scale pointer");
    if (r.group_n != 1 && r.group_n != 128) return fail(B2G_ERR_INVALID_ARG, "group_n must be 1 or 128");
    if (r.N % r.group_n) return fail(B2G_ERR_UNSUPPORTED, "N %% GROUP_N != 0");
    if (r.stride_sfa < r.M) return fail(B2G_ERR_INVALID_ARG, "stride_sfa < M");
    if (r.group_n == 1 && (r.stride_sfb < r.N || r.stride_sfb % 4 || !aligned16(r.bsb) || r.bsb_bstride % 4))
      return fail(B2G_ERR_ALIGNMENT, "GROUP_N=1 SFB needs stride_sfb >= N, a multiple of 4, and a 16-byte aligned base");
    if (r.group_n == 128 && r.stride_sfb < r.K / 128) return fail(B2G_ERR_INVALID_ARG, "stride_sfb < K/128");
  }

  Env env;
  if (fixed_env) {
    env = *fixed_env;
  } else {
    DevState* dst = nullptr;
    rc = device_state(&dst);
    if (rc) return rc;
    env = env_of(dst);
  }
  const Env& d = env;
  if (use_skinny(r, d.sms)) return run_skinny(r, d);

  // ---- tile + split
  int bn = 0, S = 1, kb_per = 1, bm = 128;
  rc = plan_tiles(r, d.sms, &bn, &S, &kb_per, &bm);
  if (rc) return rc;
  // the epilogue-term kernels are compiled for 256-wide tiles (unsplit calls)
  if (epi_any(r.epi) && S == 1 && bm != 256) bn = 256;
  const bool pair = bm == 256;
  const int KB = cdiv(r.K, 128);

  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = r.M; p.N = r.N; p.K = r.K; p.batch = r.batch;
  p.c = r.c; p.ldc = r.ldc; p.c_bstride = r.c_bstride;
  p.alpha = r.alpha;
  p.epi = r.epi;
  p.sfa = r.sfa; p.sfb = r.sfb;
  p.sfa_rb = sf_row_block_bytes(r);
  p.sfb_rb = p.sfa_rb;
  p.sfa_bstride = r.sfa_bstride; p.sfb_bstride = r.sfb_bstride;
  p.sfb_blocks = cdiv(r.N, 128);
  p.bsa = r.bsa; p.bsb = r.bsb;
  p.stride_sfa = r.stride_sfa; p.stride_sfb = r.stride_sfb;
  p.bsa_bstride = r.bsa_bstride; p.bsb_bstride = r.bsb_bstride;
  p.group_n = r.group_n;
  p.MT = cdiv(r.M, bm); p.NT = cdiv(r.N, bn);
  p.S = S; p.KB = KB; p.kb_per_split = kb_per;
  // grouped raster: group_m row tiles walked together down every column tile
  // (B2G_GROUP_M=<n> overrides, for tuning)
  static const int group_m_env = [] {
    const char* v = getenv("B2G_GROUP_M");
    return v ? atoi(v) : 0;
  }();
  p.group_m = group_m_env > 0 ? group_m_env : 8;
  const long long units = static_cast<long long>(r.batch) * p.MT * p.NT * S;
  if (units > 0x7fffffffLL) return fail(B2G_ERR_UNSUPPORTED, "problem too large");
  p.num_units = static_cast<int>(units);
  p.status = d.status;
  p.timeout_ns = g_timeout_ns.load();
  p.debug_stall = g_force_stall.load();

  if (r.n_peers) {
    if (S != 1) return fail(B2G_ERR_UNSUPPORTED, "the peer-store output takes no K split");
    p.out_mode = kOutPeers;
    for (int i = 0; i < r.n_peers; ++i) p.peer_c[i] = r.peer_c[i];
    p.n_peers = r.n_peers;
    p.peer_first = r.peer_self;
    p.peer_ldc = r.peer_ldc;
    p.peer_col0 = r.peer_col0;
    p.peer_shard = r.peer_shard;
    p.peer_row0 = static_cast<long long>(r.peer_self) * r.M;
  } else if (S == 1) {
    p.out_mode = kOutStore;
  } else if (r.out_f32 && !epi_any(r.epi)) {
    p.out_mode = kOutAtomic;
  } else {
    p.out_mode = kOutWorkspace;
  }

  // C through TMA stores when its row pitch (and batch stride) are whole 16 bytes
  {
    const long long es = r.out_f32 ? 4 : 2;
    const long long bstride = r.batch > 1 ? r.c_bstride : r.ldc * r.M;
    if (p.out_mode == kOutStore && (r.ldc * es) % 16 == 0 && (bstride * es) % 16 == 0) {
      cuuint64_t dims[3] = {(cuuint64_t)r.N, (cuuint64_t)r.M, (cuuint64_t)r.batch};
      cuuint64_t str[2] = {(cuuint64_t)(r.ldc * es), (cuuint64_t)(bstride * es)};
      // boxes of the epilogue's store chunk (GemmCfg / PairCfg::kStoreChunkBytes): 32 bytes
      // of columns for the 20-warp blockwise tile (256 wide, 128 x 128 weight scales) and
      // the MXFP4 pair kernel, 64 for every other kernel
      const long long chunk =
          ((r.mode == kModeBlk && r.group_n != 1 && !pair && bn == 256) || (pair && r.mode == kModeMX4)) ? 32 : 64;
      cuuint32_t box[3] = {(cuuint32_t)(chunk / es), 32, 1};
      rc = encode(&p.tm_c, r.out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, r.c,
                  dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      p.tma_store = 1;
    }
  }

  // ---- tensor maps
  CUtensorMap ta, tb;
  {
    cuuint64_t dims[3] = {(cuuint64_t)r.K, (cuuint64_t)r.M, (cuuint64_t)r.batch};
    cuuint64_t str[2] = {(cuuint64_t)r.lda, (cuuint64_t)(r.batch > 1 ? r.a_bstride : r.lda * r.M)};
    cuuint32_t box[3] = {128, 128, 1};
    rc = encode(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, r.a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (!r.bpre) {
    cuuint64_t dims[3] = {(cuuint64_t)r.K, (cuuint64_t)r.N, (cuuint64_t)r.batch};
    cuuint64_t str[2] = {(cuuint64_t)r.ldb, (cuuint64_t)(r.batch > 1 ? r.b_bstride : r.ldb * r.N)};
    cuuint32_t box[3] = {128, (cuuint32_t)(pair ? bn / 2 : bn), 1};  // a pair CTA loads half the B rows
    rc = encode(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, r.b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    // [N/16][K/16][16 rows x 16 bytes] viewed as (256-byte tile, n_grp, k_grp, batch):
    // a box of (256, BN/16, 8, 1) lands in smem as [k_grp][n][16 B], the interleaved
    // K-major operand layout of tcgen05.mma, with 256 contiguous bytes per request.
    cuuint64_t dims[4] = {256, (cuuint64_t)(r.N / 16), (cuuint64_t)(r.K / 16), (cuuint64_t)r.batch};
    cuuint64_t str[3] = {(cuuint64_t)16 * r.K, 256, (cuuint64_t)(r.batch > 1 ? r.b_bstride : (long long)r.N * r.K)};
    cuuint32_t box[4] = {256, (cuuint32_t)((pair ? bn / 2 : bn) / 16), 8, 1};
    rc = encode(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, r.b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }

  // ---- split-K output preparation
  if (p.out_mode == kOutAtomic) {
    for (int bi = 0; bi < r.batch; ++bi)
      B2G_CUDA(cudaMemset2DAsync(reinterpret_cast<float*>(r.c) + bi * r.c_bstride, r.ldc * 4, 0,
                                 static_cast<size_t>(r.N) * 4, r.M, r.stream));
  } else if (p.out_mode == kOutWorkspace) {
    void* ws = nullptr;
    const size_t need = r.ws_offset + split_ws_bytes(r, S, d.sms);
    rc = env_workspace(d, need, &ws);
    if (rc) return rc;
    p.ws = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + r.ws_offset);
  }

  if (pair) {
    // scale atoms as (128 words, K-atom, row block, batch) boxes of
    // pair_sf_group(mode) 128-K blocks (one box per operand brings a group's atoms)
    CUtensorMap tsa, tsb;
    memset(&tsa, 0, sizeof(tsa));
    memset(&tsb, 0, sizeof(tsb));
    if (mode_mx(r.mode)) {
      const int ka = mode_atoms(r.mode);  // K-atoms per 128-byte K block
      const long long kb4 = cdiv(r.K, 128) * ka;
      for (int which = 0; which < 2; ++which) {
        const int rows = which ? r.N : r.M;
        const long long rb = cdiv(rows, 128);
        const long long bstr = which ? r.sfb_bstride : r.sfa_bstride;
        cuuint64_t dims[4] = {128, (cuuint64_t)kb4, (cuuint64_t)rb, (cuuint64_t)r.batch};
        cuuint64_t str[3] = {512, (cuuint64_t)(kb4 * 512), (cuuint64_t)(r.batch > 1 ? bstr : rb * kb4 * 512)};
        cuuint32_t box[4] = {128, (cuuint32_t)(ka * pair_sf_group(r.mode)), (cuuint32_t)(which ? 2 : 1), 1};
        rc = encode(which ? &tsb : &tsa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, which ? (const void*)r.sfb : (const void*)r.sfa,
                    dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
      }
    }
    PairParams pp;
    pp.g = p;
    pp.num_pairs = static_cast<int>(std::min<long long>(units, d.sms / 2));
    rc = dispatch_pair(d, r.mode, bn, r.bpre, r.out_f32, ta, tb, tsa, tsb, pp, r.stream);
    if (rc) return rc;
  } else {
  const int grid = static_cast<int>(std::min<long long>(units, d.sms));
  switch (r.mode) {
    case kModePlain: rc = dispatch_bn<kModePlain>(d, bn, r.bpre, r.out_f32, ta, tb, p, grid, r.stream); break;
    case kModeMX: rc = dispatch_bn<kModeMX>(d, bn, r.bpre, r.out_f32, ta, tb, p, grid, r.stream); break;
    case kModeMX4: rc = dispatch_bn<kModeMX4>(d, bn, r.bpre, r.out_f32, ta, tb, p, grid, r.stream); break;
    default: rc = dispatch_bn<kModeBlk>(d, bn, r.bpre, r.out_f32, ta, tb, p, grid, r.stream); break;
  }
  if (rc) return rc;
  }

  if (p.out_mode == kOutWorkspace) {
    const long long work = static_cast<long long>(r.batch) * r.M * (r.N / 4);
    const int g = grid_for(work, 256, d.sms);
    if (r.out_f32)
      b2g_splitk_reduce_kernel<true><<<g, 256, 0, r.stream>>>(p.ws, r.c, S, r.batch, r.M, r.N, r.ldc, r.c_bstride,
                                                               r.epi);
    else
      b2g_splitk_reduce_kernel<false><<<g, 256, 0, r.stream>>>(p.ws, r.c, S, r.batch, r.M, r.N, r.ldc, r.c_bstride,
                                                                r.epi);
    B2G_CUDA(cudaGetLastError());
  }
  return maybe_sync_check(d);
}

}  // namespace

// =================================================================== fixed scratch
// Device scratch for b2g_gemm_mxfp8_noalloc: a file-scope array every GPU that
// loads this library holds until the process exits.  Bytes [0, 256) hold the
// kernel status word (zero at load, sticky until b2g_device_status clears it);
// the rest holds either the split-K fp32 partials (M > 128, bf16 output or a
// split with fp32 output and epilogue terms) or the decode kernel's fp32 piece
// slots (M <= 128: 2 * grid * MP * 128 * 4 bytes, 18.5 MiB at M = 128 on 148
// SMs).  32 MiB holds every decode shape on a 148-SM B200.
static constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
static constexpr size_t kNoAllocStatusBytes = 256;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

struct NoAllocDev {
  bool ready = false;
  int sms = 0;
  uint8_t* base = nullptr;  // device address of g_noalloc_scratch on this device
  unsigned long long* tile_cnt = nullptr;
  FnCache fns;
};
NoAllocDev g_noalloc[64];

// Once per device, with that device current: look up the array's device
// address (host code may not use the symbol itself; it is a host-side stand-in).
int noalloc_env(Env* e) {
  int dev = 0;
  B2G_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_NO_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  NoAllocDev& d = g_noalloc[dev];
  if (!d.ready) {
    int major = 0;
    B2G_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return fail(B2G_ERR_NO_DEVICE, "device %d is sm_%d0; this library targets sm_100a", dev, major);
    B2G_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess || !ptr)
      return fail(B2G_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed: %s", cudaGetErrorString(err));
    d.base = static_cast<uint8_t*>(ptr);
    int rc = skinny_counters(&d.tile_cnt);
    if (rc) return rc;
    d.ready = true;
  }
  e->dev = nullptr;
  e->sms = d.sms;
  e->status = reinterpret_cast<int*>(d.base);
  e->fns = &d.fns;
  e->tile_cnt = d.tile_cnt;
  e->fixed_ws = d.base + kNoAllocStatusBytes;
  e->fixed_ws_bytes = kNoAllocScratchBytes - kNoAllocStatusBytes;
  return B2G_OK;
}

}  // namespace

// =================================================================== C ABI
extern "C" {

int b2g_version(void) { return kVersion; }
const char* b2g_last_error(void) { return g_last_error; }

const char* b2g_status_string(int s) {
  switch (s) {
    case B2G_OK: return "ok";
    case B2G_ERR_INVALID_ARG: return "invalid argument";
    case B2G_ERR_UNSUPPORTED: return "unsupported shape or layout";
    case B2G_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case B2G_ERR_CUDA: return "CUDA error";
    case B2G_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case B2G_ERR_NO_DEVICE: return "no sm_100 device";
    case B2G_ERR_WORKSPACE: return "scratch allocation failed";
    default: return "unknown status";
  }
}

int b2g_set_wait_timeout_ms(int ms) {
  if (ms <= 0) return fail(B2G_ERR_INVALID_ARG, "timeout must be positive");
  g_timeout_ns.store(static_cast<unsigned long long>(ms) * 1000000ull);
  return B2G_OK;
}

int b2g_set_static_weights(int on) {
  g_static_weights.store(on ? 1 : 0);
  return B2G_OK;
}

int b2g_debug_force_stall(int on) {
  g_force_stall.store(on ? 1 : 0);
  return B2G_OK;
}

// Reads the allocating entry points' status word and, once b2g_gemm_mxfp8_noalloc
// has run on this device, the no-alloc array's: the first nonzero one is reported.
// Allocates nothing, so a caller of the no-alloc entry point may use it too.
int b2g_device_status(int* status, int clear) {
  if (!status) return fail(B2G_ERR_INVALID_ARG, "null status pointer");
  DevState* d = nullptr;
  int dev = 0;
  int rc = device_state(&d, &dev);
  if (rc) return rc;
  int* na_status = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_noalloc[dev].ready) na_status = reinterpret_cast<int*>(g_noalloc[dev].base);
  }
  B2G_CUDA(cudaDeviceSynchronize());
  int st = 0, na = 0;
  B2G_CUDA(cudaMemcpy(&st, d->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (na_status) B2G_CUDA(cudaMemcpy(&na, na_status, sizeof(int), cudaMemcpyDeviceToHost));
  *status = st ? st : na;
  if (clear) {
    if (st) B2G_CUDA(cudaMemset(d->status, 0, sizeof(int)));
    if (na) B2G_CUDA(cudaMemset(na_status, 0, sizeof(int)));
    // a launch that stopped early can leave tile counters mid-count
    if (*status) B2G_CUDA(cudaMemset(d->tile_cnt, 0, sizeof(unsigned long long) * kSkinnyMaxTiles));
  }
  return *status ? B2G_ERR_DEVICE_TIMEOUT : B2G_OK;
}

int b2g_manifest_size(void) { return kManifestN; }

int b2g_manifest_entry(int i, int* tile_m, int* tile_n, int* splitk, int* bpreshuffle, const char** name) {
  if (i < 0 || i >= kManifestN) return fail(B2G_ERR_INVALID_ARG, "manifest index %d out of range", i);
  if (tile_m) *tile_m = kManifest[i].tile_m;
  if (tile_n) *tile_n = kManifest[i].tile_n;
  if (splitk) *splitk = kManifest[i].splitk;
  if (bpreshuffle) *bpreshuffle = kManifest[i].bpre;
  if (name) *name = kManifest[i].name;
  return B2G_OK;
}

int b2g_select(int m, int n, int k, int num_sm, int log2_k_split, int bpreshuffle, int* index, int* tile_m,
               int* tile_n, int* log2_split) {
  (void)k;
  if (m <= 0 || n <= 0 || num_sm <= 0) return fail(B2G_ERR_INVALID_ARG, "bad select arguments");
  int idx = -1, l2 = 0;
  select_tile(m, n, num_sm, log2_k_split, bpreshuffle, &idx, &l2);
  if (index) *index = idx;
  if (idx < 0) return fail(B2G_ERR_UNSUPPORTED, "no manifest entry fits");
  if (tile_m) *tile_m = kManifest[idx].tile_m;
  if (tile_n) *tile_n = kManifest[idx].tile_n;
  if (log2_split) *log2_split = l2;
  return B2G_OK;
}

int b2g_gemm_a8w8_blockscale(const opus_gemm_kargs* ka, int group_n, int out_dtype, int log2_k_split,
                             void* stream) {
  if (!ka) return fail(B2G_ERR_INVALID_ARG, "null kargs");
  if (out_dtype != B2G_OUT_BF16 && out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  Req r;
  r.mode = kModeBlk;
  r.out_f32 = out_dtype == B2G_OUT_F32;
  r.M = ka->m; r.N = ka->n; r.K = ka->k; r.batch = ka->batch;
  r.a = ka->ptr_a; r.lda = ka->stride_a; r.a_bstride = ka->stride_a_batch;
  r.b = ka->ptr_b; r.ldb = ka->stride_b; r.b_bstride = ka->stride_b_batch;
  r.c = ka->ptr_c; r.ldc = ka->stride_c; r.c_bstride = ka->stride_c_batch;
  r.bsa = static_cast<const float*>(ka->ptr_sfa);
  r.bsb = static_cast<const float*>(ka->ptr_sfb);
  r.stride_sfa = ka->stride_sfa; r.stride_sfb = ka->stride_sfb;
  r.bsa_bstride = ka->stride_sfa_batch; r.bsb_bstride = ka->stride_sfb_batch;
  r.group_n = group_n;
  r.log2_k_split = log2_k_split;
  r.stream = static_cast<cudaStream_t>(stream);
  return run_gemm(r);
}

static int a8w8_common(const opus_gemm_kargs_a8w8* ka, float alpha, int out_dtype, int log2_k_split, void* stream,
                       bool pre) {
  if (!ka) return fail(B2G_ERR_INVALID_ARG, "null kargs");
  if (out_dtype != B2G_OUT_BF16 && out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  Req r;
  r.mode = kModePlain;
  r.bpre = pre;
  r.out_f32 = out_dtype == B2G_OUT_F32;
  r.M = ka->m; r.N = ka->n; r.K = ka->k; r.batch = ka->batch;
  r.a = ka->ptr_a; r.lda = ka->stride_a; r.a_bstride = ka->stride_a_batch;
  r.b = ka->ptr_b; r.ldb = pre ? ka->k : ka->stride_b; r.b_bstride = ka->stride_b_batch;
  r.c = ka->ptr_c; r.ldc = ka->stride_c; r.c_bstride = ka->stride_c_batch;
  r.alpha = alpha;
  r.log2_k_split = log2_k_split;
  r.stream = static_cast<cudaStream_t>(stream);
  return run_gemm(r);
}

int b2g_gemm_a8w8(const opus_gemm_kargs_a8w8* ka, float alpha, int out_dtype, int log2_k_split, void* stream) {
  return a8w8_common(ka, alpha, out_dtype, log2_k_split, stream, false);
}

int b2g_gemm_a8w8_preshuffled(const opus_gemm_kargs_a8w8* ka, float alpha, int out_dtype, int log2_k_split,
                              void* stream) {
  return a8w8_common(ka, alpha, out_dtype, log2_k_split, stream, true);
}

long long b2g_sf_tc_bytes(int rows, int k) {
  if (rows <= 0 || k <= 0) return 0;
  return static_cast<long long>((rows + 127) / 128) * ((k / 32 + 3) / 4) * 512;
}

// b2g_gemm_mxfp8 / b2g_gemm_mxfp4: K and the A/B strides arrive in elements; an
// MXFP4 request carries them in bytes (two E2M1 elements per byte).
static int run_mx_native(const b2g_mxfp8_args* g, int mode, void* stream, const b2g_epilogue* epi = nullptr) {
  if (!g) return fail(B2G_ERR_INVALID_ARG, "null args");
  if (g->out_dtype != B2G_OUT_BF16 && g->out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  const int per = mode == kModeMX4 ? 2 : 1;
  if (per == 2 && (g->k % 2 || g->lda % 2 || (!g->b_preshuffled && g->ldb % 2)))
    return fail(B2G_ERR_ALIGNMENT, "MXFP4 K and row strides count E2M1 elements and must be even");
  Req r;
  r.mode = mode;
  r.bpre = g->b_preshuffled != 0;
  r.out_f32 = g->out_dtype == B2G_OUT_F32;
  r.M = g->m; r.N = g->n; r.K = g->k / per;
  r.a = g->a; r.lda = g->lda / per;
  r.b = g->b; r.ldb = r.bpre ? g->k / per : g->ldb / per;
  r.c = g->d; r.ldc = g->ldd;
  r.alpha = g->alpha;
  r.sfa = static_cast<const uint8_t*>(g->sfa);
  r.sfb = static_cast<const uint8_t*>(g->sfb);
  r.log2_k_split = g->log2_k_split;
  r.stream = static_cast<cudaStream_t>(stream);
  if (epi) {
    r.epi.cin = epi->c;
    r.epi.ldcin = epi->ldc;
    r.epi.beta = epi->beta;
    r.epi.bias = epi->bias;
  }
  return run_gemm(r);
}

int b2g_gemm_mxfp8(const b2g_mxfp8_args* g, void* stream) { return run_mx_native(g, kModeMX, stream); }

int b2g_gemm_mxfp8_ex(const b2g_mxfp8_args* g, const b2g_epilogue* epi, void* stream) {
  return run_mx_native(g, kModeMX, stream, epi);
}

int b2g_gemm_mxfp4(const b2g_mxfp8_args* g, void* stream) { return run_mx_native(g, kModeMX4, stream); }

int b2g_gemm_mxfp4_ex(const b2g_mxfp8_args* g, const b2g_epilogue* epi, void* stream) {
  return run_mx_native(g, kModeMX4, stream, epi);
}

int b2g_gemm_mxfp8_peer_out(const b2g_mxfp8_args* g, void* const* peer_d, int n_peers, int self,
                            long long ldd_full, long long col_offset, void* stream) {
  if (!g || !peer_d) return fail(B2G_ERR_INVALID_ARG, "null args");
  if (g->out_dtype != B2G_OUT_BF16 && g->out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  if (n_peers < 1 || n_peers > kMaxPeers) return fail(B2G_ERR_INVALID_ARG, "n_peers must be 1..%d", kMaxPeers);
  if (self < 0 || self >= n_peers) return fail(B2G_ERR_INVALID_ARG, "self %d outside 0..%d", self, n_peers - 1);
  const long long es = g->out_dtype == B2G_OUT_F32 ? 4 : 2;
  for (int i = 0; i < n_peers; ++i)
    if (!peer_d[i] || !aligned16(peer_d[i])) return fail(B2G_ERR_ALIGNMENT, "peer buffer %d null or not 16-byte aligned", i);
  if (col_offset < 0 || ldd_full < col_offset + g->n)
    return fail(B2G_ERR_INVALID_ARG, "columns [%lld, %lld) outside the %lld-column peer buffers", col_offset,
                col_offset + g->n, ldd_full);
  if ((ldd_full * es) % 16 || (col_offset * es) % 16)
    return fail(B2G_ERR_ALIGNMENT, "peer row pitch and column offset must be whole 16 bytes");
  Req r;
  r.mode = kModeMX;
  r.bpre = g->b_preshuffled != 0;
  r.out_f32 = g->out_dtype == B2G_OUT_F32;
  r.M = g->m; r.N = g->n; r.K = g->k;
  r.a = g->a; r.lda = g->lda;
  r.b = g->b; r.ldb = r.bpre ? g->k : g->ldb;
  r.c = peer_d[self]; r.ldc = ldd_full;
  r.alpha = g->alpha;
  r.sfa = static_cast<const uint8_t*>(g->sfa);
  r.sfb = static_cast<const uint8_t*>(g->sfb);
  r.log2_k_split = 0;
  r.stream = static_cast<cudaStream_t>(stream);
  r.peer_c = peer_d;
  r.n_peers = n_peers;
  r.peer_self = self;
  r.peer_ldc = ldd_full;
  r.peer_col0 = col_offset;
  return run_gemm(r);
}

int b2g_gemm_mxfp8_a2a_out(const b2g_mxfp8_args* g, void* const* peer_d, int n_peers, int self, void* stream) {
  if (!g || !peer_d) return fail(B2G_ERR_INVALID_ARG, "null args");
  if (g->out_dtype != B2G_OUT_BF16 && g->out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  if (n_peers < 1 || n_peers > kMaxPeers) return fail(B2G_ERR_INVALID_ARG, "n_peers must be 1..%d", kMaxPeers);
  if (self < 0 || self >= n_peers) return fail(B2G_ERR_INVALID_ARG, "self %d outside 0..%d", self, n_peers - 1);
  if (g->n <= 0 || g->n % n_peers) return fail(B2G_ERR_INVALID_ARG, "N (%d) must split evenly over %d peers", g->n, n_peers);
  const long long shard = g->n / n_peers;
  if (shard % 64) return fail(B2G_ERR_UNSUPPORTED, "columns per peer (%lld) must be a multiple of 64", shard);
  for (int i = 0; i < n_peers; ++i)
    if (!peer_d[i] || !aligned16(peer_d[i])) return fail(B2G_ERR_ALIGNMENT, "peer buffer %d null or not 16-byte aligned", i);
  Req r;
  r.mode = kModeMX;
  r.bpre = g->b_preshuffled != 0;
  r.out_f32 = g->out_dtype == B2G_OUT_F32;
  r.M = g->m; r.N = g->n; r.K = g->k;
  r.a = g->a; r.lda = g->lda;
  r.b = g->b; r.ldb = r.bpre ? g->k : g->ldb;
  r.c = peer_d[self]; r.ldc = g->n;  // C is written only through the peer windows
  r.alpha = g->alpha;
  r.sfa = static_cast<const uint8_t*>(g->sfa);
  r.sfb = static_cast<const uint8_t*>(g->sfb);
  r.log2_k_split = 0;
  r.stream = static_cast<cudaStream_t>(stream);
  r.peer_c = peer_d;
  r.n_peers = n_peers;
  r.peer_self = self;
  r.peer_shard = shard;
  return run_gemm(r);
}

// The f4gemm kernarg entries.  Strides count elements (f4gemm.hpp:351-353: an
// MXFP4 row of K elements is K/2 bytes); MXFP4 keeps the reference's K % 256 rule
// (asm_f4gemm/main.cpp:141-150).
static int run_mx_f4gemm(const b2g_f4gemm_kargs* a, int bpreshuffle, int out_dtype, void* stream, int mode) {
  if (!a) return fail(B2G_ERR_INVALID_ARG, "null kargs");
  if (out_dtype != B2G_OUT_BF16 && out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  const int M = static_cast<int>(a->M), N = static_cast<int>(a->N), K = static_cast<int>(a->K);
  const int per = mode == kModeMX4 ? 2 : 1;  // elements per byte
  if (M <= 0 || N <= 0 || K <= 0) return fail(B2G_ERR_INVALID_ARG, "non-positive problem size");
  if (K % 32) return fail(B2G_ERR_UNSUPPORTED, "K %% 32 != 0");
  if (per == 2 && K % 256) return fail(B2G_ERR_UNSUPPORTED, "MXFP4 needs K %% 256 == 0 (K=%d)", K);
  if (per == 2 && (a->stride_A0 % 2 || (!bpreshuffle && a->stride_B0 % 2)))
    return fail(B2G_ERR_ALIGNMENT, "MXFP4 A/B strides count E2M1 elements and must be even");
  if (!a->ptr_ScaleA || !a->ptr_ScaleB || !a->ptr_A || !a->ptr_B || !a->ptr_D)
    return fail(B2G_ERR_INVALID_ARG, "null pointer in kargs");
  if (N % 16) return fail(B2G_ERR_UNSUPPORTED, "N (%d) must be a multiple of 16", N);
  const bool with_c = a->beta != 0.0f && a->ptr_C;
  if (with_c && ((static_cast<long long>(a->stride_C0) * (out_dtype == B2G_OUT_F32 ? 4 : 2)) % 16 ||
                 !aligned16(a->ptr_C) || !aligned16(a->ptr_D)))
    return fail(B2G_ERR_ALIGNMENT, "with beta, C and D need 16-byte aligned bases and row pitch");
  const int cols = K / 32;
  const int snA = static_cast<int>(a->stride_ScaleA0), snB = static_cast<int>(a->stride_ScaleB0);
  if (snA < cols || snA % 8 || snB < cols || snB % 8)
    return fail(B2G_ERR_INVALID_ARG, "scale row strides must be the padded column count (>= K/32, multiple of 8)");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  Req r;
  r.mode = mode;
  r.bpre = bpreshuffle != 0;
  r.out_f32 = out_dtype == B2G_OUT_F32;
  r.M = M; r.N = N; r.K = K / per;
  r.a = a->ptr_A; r.lda = a->stride_A0 / per;
  r.b = a->ptr_B; r.ldb = r.bpre ? K / per : static_cast<long long>(a->stride_B0) / per;
  r.c = a->ptr_D; r.ldc = a->stride_C0;  // the reference kernels use stride_C0 for D
  r.alpha = a->alpha;
  r.log2_k_split = a->log2_k_split;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  r.stream = st;
  // D = alpha * A . B^T + beta * C (f4gemm_ref.hpp reference_gemm): the beta term is
  // added where the GEMM writes D (its epilogue, or the split-K reduce); beta is
  // ignored without a C, as there.  C has D's type and row pitch stride_C0 (the
  // reference kernels read stride_C0 for both) and may be D itself.
  if (with_c) {
    r.epi.cin = a->ptr_C;
    r.epi.ldcin = a->stride_C0;
    r.epi.beta = a->beta;
  }
  // One scratch block for the re-laid-out scales and the split-K workspace,
  // sized before anything is written into it (growing it later would free it).
  int bn = 0, S = 1, kb_per = 1;
  rc = plan_tiles(r, d->sms, &bn, &S, &kb_per);
  if (rc) return rc;
  const long long tcA = b2g_sf_tc_bytes(M, K), tcB = b2g_sf_tc_bytes(N, K);
  const size_t offB = static_cast<size_t>((tcA + 255) / 256 * 256);
  const size_t offW = offB + static_cast<size_t>((tcB + 255) / 256 * 256);
  void* ws = nullptr;
  rc = workspace(d, offW + split_ws_bytes(r, S, d->sms), &ws);
  if (rc) return rc;
  uint8_t* sA = static_cast<uint8_t*>(ws);
  uint8_t* sB = sA + offB;
  b2g_sf_f4gemm_to_tc_kernel<<<grid_for(tcA, 256, d->sms), 256, 0, st>>>(
      static_cast<const uint8_t*>(a->ptr_ScaleA), M, cols, snA, sA);
  b2g_sf_f4gemm_to_tc_kernel<<<grid_for(tcB, 256, d->sms), 256, 0, st>>>(
      static_cast<const uint8_t*>(a->ptr_ScaleB), N, cols, snB, sB);
  B2G_CUDA(cudaGetLastError());
  r.sfa = sA; r.sfb = sB;
  r.ws_offset = offW;
  return run_gemm(r);
}

int b2g_gemm_mxfp8_f4gemm(const b2g_f4gemm_kargs* a, int bpreshuffle, int out_dtype, void* stream) {
  return run_mx_f4gemm(a, bpreshuffle, out_dtype, stream, kModeMX);
}

int b2g_gemm_mxfp4_f4gemm(const b2g_f4gemm_kargs* a, int bpreshuffle, int out_dtype, void* stream) {
  return run_mx_f4gemm(a, bpreshuffle, out_dtype, stream, kModeMX4);
}

int b2g_gemm_mxfp8_noalloc(const b2g_mxfp8_args* g, void* stream) {
  if (!g) return fail(B2G_ERR_INVALID_ARG, "null args");
  if (g->out_dtype != B2G_OUT_BF16 && g->out_dtype != B2G_OUT_F32) return fail(B2G_ERR_INVALID_ARG, "bad out_dtype");
  Req r;
  r.mode = kModeMX;
  r.bpre = g->b_preshuffled != 0;
  r.out_f32 = g->out_dtype == B2G_OUT_F32;
  r.M = g->m; r.N = g->n; r.K = g->k;
  r.a = g->a; r.lda = g->lda;
  r.b = g->b; r.ldb = r.bpre ? g->k : g->ldb;
  r.c = g->d; r.ldc = g->ldd;
  r.alpha = g->alpha;
  r.sfa = static_cast<const uint8_t*>(g->sfa);
  r.sfb = static_cast<const uint8_t*>(g->sfb);
  r.log2_k_split = g->log2_k_split;
  r.stream = static_cast<cudaStream_t>(stream);
  if (r.M <= 0 || r.N <= 0 || r.K <= 0) return fail(B2G_ERR_INVALID_ARG, "non-positive problem size");
  Env e;
  int rc = noalloc_env(&e);
  if (rc) return rc;
  // reject up front, before any device work is queued, if the scratch does not fit
  int bn = 0, S = 1, kb_per = 1;
  rc = plan_tiles(r, e.sms, &bn, &S, &kb_per);
  if (rc) return rc;
  const size_t need = split_ws_bytes(r, S, e.sms);
  if (need > e.fixed_ws_bytes) {
    if (use_skinny(r, e.sms))
      return fail(B2G_ERR_WORKSPACE,
                  "b2g_gemm_mxfp8_noalloc: M=%d takes the decode kernel, whose piece slots need %zu bytes; "
                  "the fixed scratch array holds %zu", r.M, need, e.fixed_ws_bytes);
    return fail(B2G_ERR_WORKSPACE,
                "b2g_gemm_mxfp8_noalloc: %d-way split-K partials (S*M*N*4) need %zu bytes; the fixed scratch "
                "array holds %zu (use a smaller log2_k_split, or b2g_gemm_mxfp8)", S, need, e.fixed_ws_bytes);
  }
  // Every slot and partial the kernels read is written earlier in the same call,
  // so nothing in the array needs zeroing per call.  The status word is sticky
  // (a timeout stays visible to b2g_device_status until cleared there);
  // B2G_SYNC_CHECK=1 checks it inside run_gemm.
  return run_gemm(r, &e);
}

// ------------------------------------------------------------ layout helpers
int b2g_sf_rowmajor_to_tc(const void* src, int rows, int cols, long long ld, void* dst, void* stream) {
  if (!src || !dst || rows <= 0 || cols <= 0 || ld < cols) return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  const long long total = static_cast<long long>((rows + 127) / 128) * ((cols + 3) / 4) * 512;
  b2g_sf_rowmajor_to_tc_kernel<<<grid_for(total, 256, d->sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), rows, cols, ld, static_cast<uint8_t*>(dst));
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

int b2g_sf_f4gemm_to_tc(const void* src, int rows, int cols, int sn, void* dst, void* stream) {
  if (!src || !dst || rows <= 0 || cols <= 0 || sn < cols || sn % 8) return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  const long long total = static_cast<long long>((rows + 127) / 128) * ((cols + 3) / 4) * 512;
  b2g_sf_f4gemm_to_tc_kernel<<<grid_for(total, 256, d->sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), rows, cols, sn, static_cast<uint8_t*>(dst));
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

int b2g_shuffle_scale(const void* src, int rows, int cols, int sm, int sn, void* dst, void* stream) {
  if (!src || !dst || rows <= 0 || cols <= 0 || sm < rows || sn < cols || sm % 32 || sn % 8)
    return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  b2g_shuffle_scale_kernel<<<grid_for((long long)sm * sn, 256, d->sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), rows, cols, sm, sn, static_cast<uint8_t*>(dst));
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

static int shuffle_w(const void* src, void* dst, int n, int kp, void* stream, bool inverse) {
  if (!src || !dst || n <= 0 || kp <= 0 || n % 16 || kp % 32) return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  if (!aligned16(src) || !aligned16(dst)) return fail(B2G_ERR_ALIGNMENT, "buffers must be 16-byte aligned");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  const long long total = static_cast<long long>(n) * (kp / 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (inverse)
    b2g_shuffle_weight_16x16_kernel<true><<<grid_for(total, 256, d->sms), 256, 0, st>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), n, kp / 16);
  else
    b2g_shuffle_weight_16x16_kernel<false><<<grid_for(total, 256, d->sms), 256, 0, st>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), n, kp / 16);
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

int b2g_shuffle_weight_16x16(const void* src, void* dst, int n, int kp, void* stream) {
  return shuffle_w(src, dst, n, kp, stream, false);
}
int b2g_unshuffle_weight_16x16(const void* src, void* dst, int n, int kp, void* stream) {
  return shuffle_w(src, dst, n, kp, stream, true);
}

// ------------------------------------------------------------ quantisers
static int run_quant_mx(const void* x, int x_dtype, bool fp4, int rows, int k, long long ldx, void* q,
                        long long ldq, void* sf_tc, void* sf_rowmajor, void* stream) {
  if (x_dtype != B2G_OUT_F32 && x_dtype != B2G_OUT_BF16) return fail(B2G_ERR_INVALID_ARG, "x_dtype must be fp32 or bf16");
  const long long q_row = fp4 ? k / 2 : k;  // bytes of one quantised row
  if (!x || !q || rows <= 0 || k <= 0 || k % 32 || ldx < k || ldq < q_row) return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  const long long xe = x_dtype == B2G_OUT_F32 ? 4 : 8;  // elements per 16 bytes
  if (!aligned16(x) || ldx % xe || (fp4 ? (ldq % 4 || (reinterpret_cast<uintptr_t>(q) & 3))
                                        : (ldq % 8 || (reinterpret_cast<uintptr_t>(q) & 7))))
    return fail(B2G_ERR_ALIGNMENT, "x must be 16-byte aligned with 16-byte rows; q rows aligned to 4 (MXFP4) or 8 bytes");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (sf_tc) {  // padding of the atom layout holds 1.0
    B2G_CUDA(cudaMemsetAsync(sf_tc, 0x7F, static_cast<size_t>(b2g_sf_tc_bytes(rows, k)), st));
  }
  const long long work = static_cast<long long>(rows) * (k / 8);
  const int grid = grid_for(work, 256, d->sms);
  uint8_t* qb = static_cast<uint8_t*>(q);
  uint8_t* stc = static_cast<uint8_t*>(sf_tc);
  uint8_t* srm = static_cast<uint8_t*>(sf_rowmajor);
  if (x_dtype == B2G_OUT_F32) {
    const float* xf = static_cast<const float*>(x);
    if (fp4) b2g_quant_mx_kernel<true><<<grid, 256, 0, st>>>(xf, rows, k, ldx, qb, ldq, stc, srm);
    else b2g_quant_mx_kernel<false><<<grid, 256, 0, st>>>(xf, rows, k, ldx, qb, ldq, stc, srm);
  } else {
    const __nv_bfloat16* xh = static_cast<const __nv_bfloat16*>(x);
    if (fp4) b2g_quant_mx_kernel<true><<<grid, 256, 0, st>>>(xh, rows, k, ldx, qb, ldq, stc, srm);
    else b2g_quant_mx_kernel<false><<<grid, 256, 0, st>>>(xh, rows, k, ldx, qb, ldq, stc, srm);
  }
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

int b2g_quant_mxfp8(const float* x, int rows, int k, long long ldx, void* q, long long ldq, void* sf_tc,
                    void* sf_rowmajor, void* stream) {
  return run_quant_mx(x, B2G_OUT_F32, false, rows, k, ldx, q, ldq, sf_tc, sf_rowmajor, stream);
}

int b2g_quant_mxfp8_ex(const void* x, int x_dtype, int rows, int k, long long ldx, void* q, long long ldq,
                       void* sf_tc, void* sf_rowmajor, void* stream) {
  return run_quant_mx(x, x_dtype, false, rows, k, ldx, q, ldq, sf_tc, sf_rowmajor, stream);
}

int b2g_quant_mxfp4(const void* x, int x_dtype, int rows, int k, long long ldx, void* q, long long ldq,
                    void* sf_tc, void* sf_rowmajor, void* stream) {
  return run_quant_mx(x, x_dtype, true, rows, k, ldx, q, ldq, sf_tc, sf_rowmajor, stream);
}

static int run_quant_1x128(const void* x, int x_dtype, int rows, int k, void* q, float* sf, void* stream) {
  if (x_dtype != B2G_OUT_F32 && x_dtype != B2G_OUT_BF16) return fail(B2G_ERR_INVALID_ARG, "x_dtype must be fp32 or bf16");
  if (!x || !q || !sf || rows <= 0 || k <= 0 || k % 128) return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  if (!aligned16(x) || !aligned16(q)) return fail(B2G_ERR_ALIGNMENT, "x and q must be 16-byte aligned");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  const long long warps = static_cast<long long>(rows) * (k / 128);
  const int grid = grid_for(warps * 32, 256, d->sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == B2G_OUT_F32)
    b2g_quant_1x128_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(x), rows, k, static_cast<uint8_t*>(q), sf);
  else
    b2g_quant_1x128_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), rows, k,
                                                 static_cast<uint8_t*>(q), sf);
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

int b2g_quant_1x128(const float* x, int rows, int k, void* q, float* sf, void* stream) {
  return run_quant_1x128(x, B2G_OUT_F32, rows, k, q, sf, stream);
}

int b2g_quant_1x128_ex(const void* x, int x_dtype, int rows, int k, void* q, float* sf, void* stream) {
  return run_quant_1x128(x, x_dtype, rows, k, q, sf, stream);
}

int b2g_quant_128x128(const float* x, int n, int k, void* q, float* sf, void* stream) {
  if (!x || !q || !sf || n <= 0 || k <= 0 || n % 128 || k % 128) return fail(B2G_ERR_INVALID_ARG, "bad arguments");
  if (!aligned16(x) || !aligned16(q)) return fail(B2G_ERR_ALIGNMENT, "x and q must be 16-byte aligned");
  DevState* d = nullptr;
  int rc = device_state(&d);
  if (rc) return rc;
  const int tiles = (n / 128) * (k / 128);
  b2g_quant_128x128_kernel<<<std::min(tiles, 8 * d->sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, n, k, static_cast<uint8_t*>(q), sf);
  B2G_CUDA(cudaGetLastError());
  return B2G_OK;
}

}  // extern "C"
