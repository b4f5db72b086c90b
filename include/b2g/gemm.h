/*
 * b2g/gemm.h -- C ABI of the B200 (sm_100a) block-scaled FP8 GEMM library.
 *
 * Drop-in boundary for the reference's opus_gemm FP8 family and its f4gemm MX
 * launch conventions (Fyzyukk/gcnasm).  Plain pointers, sizes and an opaque
 * stream handle (a cudaStream_t passed as void*, NULL = legacy default stream);
 * no torch or CUDA types in the signatures.  Every call is stream-ordered and
 * returns a status code; the library never exits the process.
 *
 * Element types: A/B are OCP E4M3 bytes; MX scales are UE8M0 bytes (value
 * 2^(e-127)); blockwise scales are fp32; C/D is bf16 (B2G_OUT_BF16) or fp32.
 */
#ifndef B2G_GEMM_H
#define B2G_GEMM_H

#include <stdint.h>

#if defined(__GNUC__)
#define B2G_API __attribute__((visibility("default")))
#else
#define B2G_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum {
    B2G_OK = 0,
    B2G_ERR_INVALID_ARG = 1,    /* null pointer, non-positive size, bad enum   */
    B2G_ERR_UNSUPPORTED = 2,    /* shape/stride outside the kernels' contract   */
    B2G_ERR_ALIGNMENT = 3,      /* pointer or stride not 16-byte aligned        */
    B2G_ERR_CUDA = 4,           /* a CUDA runtime/driver call failed            */
    B2G_ERR_DEVICE_TIMEOUT = 5, /* a kernel gave up waiting (see b2g_device_status) */
    B2G_ERR_NO_DEVICE = 6,      /* no sm_100 device current                      */
    B2G_ERR_WORKSPACE = 7       /* split-K / layout scratch could not be obtained */
};

enum { B2G_OUT_BF16 = 0, B2G_OUT_F32 = 1 };

/* --------------------------------------------------------- opus_gemm ABI */
/* Byte-for-byte the reference's kernel argument block
 * (opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_common.h:4-25, identical in
 * opus_gemm/block_scale_1x128x1_gemm/gemm_a8w8_1x128x1_blockscale_common.h:4-25).
 * Strides are in elements.  SFA is fp32 [K/128, M] (stride_sfa between K groups);
 * SFB is fp32 [N/128, K/128] for group_n = 128 (stride_sfb between N groups) or
 * [K/128, N] for group_n = 1 (stride_sfb between K groups). */
typedef struct opus_gemm_kargs {
    const void* ptr_a;
    const void* ptr_b;
    void* ptr_c;
    int m;
    int n;
    int k;
    int batch;
    int stride_a;
    int stride_b;
    int stride_c;
    int stride_a_batch;
    int stride_b_batch;
    int stride_c_batch;
    const void* ptr_sfa;
    const void* ptr_sfb;
    int stride_sfa;
    int stride_sfb;
    int stride_sfa_batch;
    int stride_sfb_batch;
} opus_gemm_kargs;

/* The fp8_gemm kernel's argument block: the first 13 fields above
 * (opus_gemm/fp8_gemm/gemm_a8w8_8wave.cc:99-113). */
typedef struct opus_gemm_kargs_a8w8 {
    const void* ptr_a;
    const void* ptr_b;
    void* ptr_c;
    int m;
    int n;
    int k;
    int batch;
    int stride_a;
    int stride_b;
    int stride_c;
    int stride_a_batch;
    int stride_b_batch;
    int stride_c_batch;
} opus_gemm_kargs_a8w8;

/* C[b] = sum_kg sfa*sfb * (A[b] . B[b]^T)_kg   with fp32 scales.
 * Replaces the launch gemm_a8w8_blockscale_kernel<Traits><<<grid, 512>>>(kargs)
 * (opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_host.cc:257; group_n = 128)
 * and gemm_a8w8_1x128x1_blockscale_kernel<Traits><<<...>>>(kargs)
 * (opus_gemm/block_scale_1x128x1_gemm/gemm_a8w8_1x128x1_blockscale_host.cc:290;
 * group_n = 1).  The reference writes fp32 C; out_dtype also allows bf16.
 * Contract: k % 128 == 0, n % 16 == 0, stride_a/stride_b multiples of 16,
 * 16-byte aligned A/B/C; group_n = 1 also needs stride_sfb % 4 == 0.
 * log2_k_split: 0 = no split, > 0 = 2^L K-splits, < 0 = heuristic. */
B2G_API int b2g_gemm_a8w8_blockscale(const opus_gemm_kargs* kargs, int group_n, int out_dtype, int log2_k_split,
                             void* stream);

/* C[b] = alpha * A[b] . B[b]^T.  Replaces gemm_a8w8_kernel<Traits><<<...>>>(kargs)
 * (opus_gemm/fp8_gemm/gemm_a8w8_8wave.cc:780 launch, :261 kernel), which has no
 * scale: alpha = 1.0 reproduces it.  Contract: k % 16 == 0, n % 16 == 0. */
B2G_API int b2g_gemm_a8w8(const opus_gemm_kargs_a8w8* kargs, float alpha, int out_dtype, int log2_k_split, void* stream);

/* Same with B given in the flat-mm preshuffled layout [N/16][K/16][16][16]
 * (opus_fmm/flatmm_a8w8_gfx950.cc:638-681 shuffle_b output; kernel :244).
 * kargs->ptr_b points at the shuffled buffer; stride_b is ignored. */
B2G_API int b2g_gemm_a8w8_preshuffled(const opus_gemm_kargs_a8w8* kargs, float alpha, int out_dtype, int log2_k_split,
                              void* stream);

/* ------------------------------------------------------------ f4gemm ABI */
/* The packed 0x174-byte kernel argument block of asm_f4gemm/f4gemm.hpp:64-115:
 * every field in a 16-byte slot.  For MXFP8 one element is one byte, so the A/B
 * strides in elements are bytes. */
#if defined(_MSC_VER)
#pragma pack(push, 1)
#define B2G_PACKED
#else
#define B2G_PACKED __attribute__((packed))
#endif
typedef struct B2G_PACKED b2g_f4gemm_kargs {
    void* ptr_D;          unsigned int _p0[2];
    void* ptr_C;          unsigned int _p1[2];
    void* ptr_A;          unsigned int _p2[2];
    void* ptr_B;          unsigned int _p3[2];
    float alpha;          unsigned int _p4[3];
    float beta;           unsigned int _p5[3];
    unsigned int stride_D0; unsigned int _p6[3];
    unsigned int stride_D1; unsigned int _p7[3];
    unsigned int stride_C0; unsigned int _p8[3];   /* used for D, as the reference kernels do */
    unsigned int stride_C1; unsigned int _p9[3];
    unsigned int stride_A0; unsigned int _p10[3];
    unsigned int stride_A1; unsigned int _p11[3];
    unsigned int stride_B0; unsigned int _p12[3];
    unsigned int stride_B1; unsigned int _p13[3];
    unsigned int M;       unsigned int _p14[3];
    unsigned int N;       unsigned int _p15[3];
    unsigned int K;       unsigned int _p16[3];
    void* ptr_ScaleA;     unsigned int _p17[2];
    void* ptr_ScaleB;     unsigned int _p18[2];
    unsigned int stride_ScaleA0; unsigned int _p19[3];
    unsigned int stride_ScaleA1; unsigned int _p20[3];
    unsigned int stride_ScaleB0; unsigned int _p21[3];
    unsigned int stride_ScaleB1; unsigned int _p22[3];
    int log2_k_split;
} b2g_f4gemm_kargs;
#if defined(_MSC_VER)
#pragma pack(pop)
#endif

/* D[M, N] = alpha * A[M, K] . B[N, K]^T + beta * C[M, N] with MXFP8 operands (E4M3,
 * one UE8M0 scale per 1x32 block of K).  Replaces Kernel::launch (asm_f4gemm/f4gemm.hpp:297-309)
 * over the kernarg block filled by fill_args (f4gemm.hpp:355-392):
 *   - ScaleA/ScaleB in the reference's padded + shuffled layout
 *     (asm_f4gemm/f4gemm_ref.hpp:101-130), stride_Scale*0 = padded columns;
 *   - bpreshuffle = 1: B in the 16x16 preshuffled layout (f4gemm_ref.hpp:78-96);
 *   - log2_k_split > 0 splits K into 2^L parts (f4gemm.hpp:329-349); unlike the
 *     reference's bf16 atomics the partial sums are reduced in fp32, so the
 *     caller does NOT need to zero D first;
 *   - beta != 0 with ptr_C set adds beta * C as the reference CPU GEMM does
 *     (f4gemm_ref.hpp:179-210: v = alpha * acc in fp32, v += beta * C, one rounding
 *     to D's type); C has D's element type and D's row pitch stride_C0 (the
 *     reference kernel reads stride_C0 for both) and may be D itself; without
 *     ptr_C, beta is ignored, as there.
 * Contract: K % 32 == 0, N % 16 == 0. */
B2G_API int b2g_gemm_mxfp8_f4gemm(const b2g_f4gemm_kargs* args, int bpreshuffle, int out_dtype, void* stream);

/* The same entry with MXFP4 operands: the reference's own f4gemm element type.
 * A [M, K/2] and B [N, K/2] hold packed OCP E2M1, element 2i in the low nibble
 * of byte i (asm_f4gemm/f4gemm_ref.hpp:22-26); one UE8M0 scale per 1x32 block of
 * K, padded + shuffled as for MXFP8.  stride_A0 / stride_B0 count E2M1 elements
 * (fill_args sets them to K: f4gemm.hpp:351-353), so a row is stride/2 bytes;
 * bpreshuffle = 1 takes B through shuffle_weight_16x16 over its bytes
 * (f4gemm_ref.hpp:78-96), as the reference kernels do.  alpha, beta/C, the K
 * split and the output types behave as in b2g_gemm_mxfp8_f4gemm.
 * Contract: K % 256 == 0 (asm_f4gemm/main.cpp:141-150), N % 16 == 0. */
B2G_API int b2g_gemm_mxfp4_f4gemm(const b2g_f4gemm_kargs* args, int bpreshuffle, int out_dtype, void* stream);

/* Native MXFP8 entry: scales already in the sm_100 tensor-core atom layout
 * (b2g_sf_tc_bytes / b2g_sf_rowmajor_to_tc), so no per-call layout work.
 * ld* in elements.  b_preshuffled: B in the 16x16 preshuffled layout. */
typedef struct b2g_mxfp8_args {
    const void* a;
    const void* b;
    const void* sfa;
    const void* sfb;
    void* d;
    int m, n, k;
    long long lda, ldb, ldd;
    float alpha;
    int b_preshuffled;
    int out_dtype;
    int log2_k_split;
} b2g_mxfp8_args;

B2G_API int b2g_gemm_mxfp8(const b2g_mxfp8_args* args, void* stream);

/* Extra epilogue terms: D = alpha * A . B^T + beta * C + bias[n], evaluated in fp32
 * in that order (each step rounded once, the reference CPU GEMM's v = alpha * acc;
 * v += beta * C, asm_f4gemm/f4gemm_ref.hpp:179-210, then the per-output-column
 * bias of the split-K reduce, opus_gemm_dist/.../splitk_reduce_gfx950.cuh:49-60),
 * then one rounding to D's type.  C and the bias have D's element type; C may be
 * D itself.  Both are applied where D is written: in the GEMM epilogue, or in the
 * split-K reduce when log2_k_split > 0 (fp32 output then goes through the
 * workspace as well).  Bases 16-byte aligned, ldc >= N with a 16-byte row pitch. */
typedef struct b2g_epilogue {
    const void* c;        /* beta * C input, or NULL */
    long long ldc;        /* elements between rows of C */
    float beta;
    const void* bias;     /* per-column bias [N], or NULL */
} b2g_epilogue;

/* b2g_gemm_mxfp8 with the terms of *epi (epi may be NULL: no terms). */
B2G_API int b2g_gemm_mxfp8_ex(const b2g_mxfp8_args* args, const b2g_epilogue* epi, void* stream);

/* Native MXFP4 entry over the same argument block: a, b packed E2M1 (two per byte,
 * element 2i in the low nibble), scales in the tensor-core atom layout for K
 * elements (b2g_sf_tc_bytes(rows, k)).  k, lda and ldb count E2M1 elements (even;
 * a row is ld/2 bytes); K % 256 == 0. */
B2G_API int b2g_gemm_mxfp4(const b2g_mxfp8_args* args, void* stream);
B2G_API int b2g_gemm_mxfp4_ex(const b2g_mxfp8_args* args, const b2g_epilogue* epi, void* stream);

/* Column-parallel MXFP8 GEMM for one GPU of a multi-GPU job with the output
 * all-gather folded into the epilogue (no counterpart in the reference, whose
 * GEMM hosts run on one GPU; it replaces "GEMM, then all-gather the bf16 column
 * slabs"): C = alpha * A[M,K] . B[N,K]^T for this GPU's N columns is stored into
 * every GPU's full-width C, element (m, n) at peer_d[i] + m * ldd_full +
 * col_offset + n for i = 0 .. n_peers-1 (elements of out_dtype; args->d and
 * args->ldd are not used, args->log2_k_split is ignored).  peer_d[self] is this
 * GPU's own buffer, the others are the other GPUs' buffers mapped into this
 * process (CUDA IPC or symmetric memory over NVLink); at most 8.  Row pitch and
 * column offset must be whole 16 bytes.  Plain stores only: no kernel waits on
 * another GPU, so the caller orders every GPU's call before reading C (a
 * barrier on the stream, e.g. an NCCL all-reduce of one element). */
B2G_API int b2g_gemm_mxfp8_peer_out(const b2g_mxfp8_args* args, void* const* peer_d, int n_peers, int self,
                                    long long ldd_full, long long col_offset, void* stream);

/* MXFP8 GEMM with an all-to-all of its output folded into the epilogue: the
 * "GEMM -> direct A2A" step of opus_gemm_dist (splitk_reduce_gfx950.cuh:276-369,
 * which stores C column shard p into peer p's window at [src_rank, M, shard_n]).
 * This GPU computes C = alpha * A[M,K] . B[N,K]^T for its own M rows and all N
 * columns; column shard q (N / n_peers columns, a multiple of 64) goes to peer q
 * only, element (m, n) at peer_d[q] + (self * M + m) * shard_n + (n - q * shard_n)
 * (elements of out_dtype): every peer's window is [n_peers * M][shard_n], rows
 * grouped by source GPU.  args->d, args->ldd and args->log2_k_split are not used.
 * peer_d[i] is GPU i's window as mapped into this process (symmetric memory or
 * CUDA IPC over NVLink).  Plain stores, no waits on other GPUs: the caller orders
 * every GPU's call before reading a window (a barrier on the stream). */
B2G_API int b2g_gemm_mxfp8_a2a_out(const b2g_mxfp8_args* args, void* const* peer_d, int n_peers, int self,
                                   void* stream);

/* b2g_gemm_mxfp8 for callers that cannot allocate device memory.  No counterpart
 * in the reference (its host programs own every buffer and its kernels need no
 * scratch).  Some hosts hand all of the GPU's memory to their own pool at start-up
 * (serving engines, frameworks with a caching allocator): a cudaMalloc made inside
 * a library either fails for lack of free memory or hides memory the pool cannot
 * account for or reclaim.  This entry point allocates nothing: its scratch lives
 * in a fixed 32 MiB array that the library declares at file scope, which every GPU
 * that loads the library holds until the process exits.  The caller still passes
 * A, B, the scales and D.  What the array holds:
 *   - M <= 128 (the decode kernel): fp32 piece slots of its split tiles,
 *     2 * grid * MP * 128 * 4 bytes (MP = M rounded up to 16/32/64/128, grid <= the
 *     SM count): at most 18.5 MiB on a 148-SM B200, so every decode shape fits;
 *   - M > 128 with log2_k_split > 0 and bf16 output: the split-K fp32 partials,
 *     S * M * N * 4 bytes.  fp32 output adds its partials into D and needs none.
 *   - the first 256 bytes: the status word its kernels' bounded waits write.  It is
 *     sticky: b2g_device_status reports it (and, with clear, resets it), and that
 *     call allocates nothing either.
 * Scratch needs above 32 MiB - 256 B are rejected with B2G_ERR_WORKSPACE before any
 * device work is queued.  The first call on a device looks up that array's device
 * address; make that first call before any stream capture.  Every call on a device
 * shares the one array: calls that overlap on the GPU (concurrent streams) race on
 * it and must be serialised by the caller.  It never calls cudaMalloc, cudaFree or
 * any allocating routine. */
B2G_API int b2g_gemm_mxfp8_noalloc(const b2g_mxfp8_args* args, void* stream);

/* ------------------------------------------------- tile selection / manifest */
/* select_kernel (asm_f4gemm/f4gemm.hpp:210-267) over the library's own tile
 * manifest with the reference's tie-breaks.  Writes the chosen manifest index,
 * its tile and the log2 split; returns B2G_OK or B2G_ERR_UNSUPPORTED. */
B2G_API int b2g_select(int m, int n, int k, int num_sm, int log2_k_split, int bpreshuffle, int* index, int* tile_m,
               int* tile_n, int* log2_split);
B2G_API int b2g_manifest_size(void);
B2G_API int b2g_manifest_entry(int i, int* tile_m, int* tile_n, int* splitk, int* bpreshuffle, const char** name);

/* ------------------------------------------------------ layout helpers */
/* bytes of a UE8M0 scale buffer for `rows` rows of a K-long operand in the
 * tensor-core atom layout (128 rows x 4 scale columns per 512-byte atom). */
B2G_API long long b2g_sf_tc_bytes(int rows, int k);
/* row-major [rows, cols] (leading dimension ld) -> tensor-core atom layout */
B2G_API int b2g_sf_rowmajor_to_tc(const void* src, int rows, int cols, long long ld, void* dst, void* stream);
/* f4gemm shuffled layout (padded columns sn) -> tensor-core atom layout */
B2G_API int b2g_sf_f4gemm_to_tc(const void* src, int rows, int cols, int sn, void* dst, void* stream);
/* row-major [rows, cols] -> f4gemm padded + shuffled [sm, sn] (f4gemm_ref.hpp:108-130) */
B2G_API int b2g_shuffle_scale(const void* src, int rows, int cols, int sm, int sn, void* dst, void* stream);
/* [N, Kp] bytes <-> 16x16 preshuffled (f4gemm_ref.hpp:81-96); N % 16 == 0, Kp % 32 == 0 */
B2G_API int b2g_shuffle_weight_16x16(const void* src, void* dst, int n, int kp, void* stream);
B2G_API int b2g_unshuffle_weight_16x16(const void* src, void* dst, int n, int kp, void* stream);

/* ------------------------------------------------------------ quantisers */
/* fp32 x [rows, K] (leading dim ldx) -> E4M3 q [rows, K] (leading dim ldq) and
 * UE8M0 scales, s = 2^ceil(log2(amax/448)) per 1x32 block.  sf_tc (atom layout,
 * b2g_sf_tc_bytes(rows, K) bytes) and/or sf_rowmajor ([rows, K/32]) may be NULL. */
B2G_API int b2g_quant_mxfp8(const float* x, int rows, int k, long long ldx, void* q, long long ldq, void* sf_tc,
                    void* sf_rowmajor, void* stream);
/* The quantisers below take their input as fp32 or bf16 (x_dtype B2G_OUT_F32 or
 * B2G_OUT_BF16: the element type of the activations a caller holds; bf16 widens
 * to fp32 exactly, so the result is that of the fp32 quantiser on the widened
 * values).  x 16-byte aligned, ldx a multiple of 8 elements. */
B2G_API int b2g_quant_mxfp8_ex(const void* x, int x_dtype, int rows, int k, long long ldx, void* q, long long ldq,
                               void* sf_tc, void* sf_rowmajor, void* stream);
/* x [rows, K] -> packed E2M1 q [rows, K/2] (element 2i in the low nibble; ldq in
 * bytes, a multiple of 4) and UE8M0 scales s = 2^ceil(log2(amax/6)) per 1x32 block
 * (the MXFP8 rule with E2M1's largest value 6), elements rounded to nearest-even
 * onto the E2M1 grid with saturation.  K % 32 == 0; scale outputs as above. */
B2G_API int b2g_quant_mxfp4(const void* x, int x_dtype, int rows, int k, long long ldx, void* q, long long ldq,
                            void* sf_tc, void* sf_rowmajor, void* stream);
/* 1x128 fp32 scales (amax/448), sf [K/128, rows] */
B2G_API int b2g_quant_1x128(const float* x, int rows, int k, void* q, float* sf, void* stream);
B2G_API int b2g_quant_1x128_ex(const void* x, int x_dtype, int rows, int k, void* q, float* sf, void* stream);
/* 128x128 fp32 scales, sf [N/128, K/128] */
B2G_API int b2g_quant_128x128(const float* x, int n, int k, void* q, float* sf, void* stream);

/* ------------------------------------------------------------ diagnostics */
/* Synchronises the current device and reports (and with clear != 0 resets) the
 * device status word the kernels write when a bounded wait gives up: the
 * allocating entry points' word, or else b2g_gemm_mxfp8_noalloc's.  A nonzero
 * word cleared here also zeroes the decode kernel's tile counters.  Allocates
 * nothing (both words are file-scope device data). */
B2G_API int b2g_device_status(int* status, int clear);
/* Per-wait time limit of the kernels' barrier waits, in milliseconds (default 4000). */
B2G_API int b2g_set_wait_timeout_ms(int ms);

/* Static weights (no counterpart in the reference; a serving-loop setting).  When
 * on, the decode GEMM (M <= 128, MX / plain FP8) may read B and its scales before
 * the kernel preceding it on the stream has completed -- launched as a
 * programmatic dependent, its first weight loads overlap that kernel's tail; A,
 * A's scales and every write still wait for it.  Only for weights that no kernel
 * earlier on the stream writes while it is on (e.g. the layers of a model being
 * served).  Default off.  Process-wide; returns B2G_OK. */
B2G_API int b2g_set_static_weights(int on);
/* Test hook: while on, every GEMM launch makes its MMA issuer wait on a barrier
 * nothing arrives on, so the bounded wait runs out and the kernel reports
 * B2G_ERR_DEVICE_TIMEOUT through b2g_device_status. */
B2G_API int b2g_debug_force_stall(int on);
B2G_API const char* b2g_status_string(int status);
B2G_API const char* b2g_last_error(void);
B2G_API int b2g_version(void);

#ifdef __cplusplus
}
#endif
#endif /* B2G_GEMM_H */
