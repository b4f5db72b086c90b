/*
 * b2g_oracle.c -- CPU restatement of the reference's block-scaled FP8 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, smoke()
 * and bench.py's CPU-baseline leg compare the CUDA path against.  Nothing in the
 * product library (gcnasm_b200/) links, loads or calls it.
 *
 * Parity status: pinned.
 *   - The f4gemm conventions restated here (E8M0 decode, scale pad+shuffle,
 *     16x16 B preshuffle, f64 reference GEMM) are checked byte-for-byte against
 *     the reference's own f4gemm_ref.hpp compiled from its sources into
 *     oracle/_ref (see oracle/Makefile) and against the golden fixtures in
 *     tests/golden/ that were generated from it.
 *   - The opus gemm_ref loops (block_scale_gemm, block_scale_1x128x1_gemm,
 *     fp8_gemm, opus_fmm's flatmm) are restated loop-for-loop below; the
 *     reference's own loops are cut unchanged out of its host sources and
 *     compiled with an E4M3 stand-in for __hip_fp8_e4m3
 *     (oracle/extract_gemm_ref.py -> oracle/_ref/libopus_ref.so), and the
 *     restatements equal them bit for bit (fixtures:
 *     tests/golden/opus_gemm_ref_golden.npz).  The whole host programs cannot
 *     be compiled here (hipcc, hip/hip_fp8.h and the aiter OPUS headers).
 *
 * Every function cites the reference file:line it follows (paths relative to
 * the reference project root).
 *
 * Number formats (OCP MX v1.0):
 *   E4M3 ("fn"): bias 7, no infinities, 0x7F/0xFF are NaN, max finite 448,
 *   min normal 2^-6, subnormal step 2^-9.  gfx950's __hip_fp8_e4m3 is this
 *   format (wmma_opus_rdna4/opus/opus.hpp:858-866).
 *   UE8M0: bare biased exponent, 2^(e-127); e=0 decodes to 2^-126 and e=0xFF
 *   to NaN exactly as asm_f4gemm/f4gemm_ref.hpp:29-41 does.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* ------------------------------------------------------------------------- */
/* Scalar formats                                                            */
/* ------------------------------------------------------------------------- */

/* OCP E4M3 -> fp32.  Replaces static_cast<float>(__hip_fp8_e4m3) used by every
 * opus gemm_ref (e.g. opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_host.cc:84). */
ORC_API float orc_e4m3_to_f32(uint8_t v)
{
    const int s = v >> 7, e = (v >> 3) & 0xF, m = v & 7;
    float r;
    if (e == 0xF && m == 7) return bits_f32(0x7FC00000u); /* NaN */
    if (e == 0) r = ldexpf((float)m, -9);                  /* subnormal m*2^-9 */
    else        r = ldexpf((float)(8 + m), e - 10);        /* (1+m/8)*2^(e-7) */
    return s ? -r : r;
}

/* fp32 -> OCP E4M3, round-to-nearest-even, saturating to +-448 (the
 * __HIP_SATFINITE behaviour of the reference's host casts, used when it fills
 * A/B with static_cast<host_fp8_t>(float), e.g. gemm_a8w8_blockscale_host.cc:41).
 * NaN maps to 0x7F. */
ORC_API uint8_t orc_f32_to_e4m3(float x)
{
    uint32_t u = f32_bits(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    float a = fabsf(x);
    if (a != a) return 0x7F;
    if (a >= 448.0f) return sign | 0x7E;
    if (a < ldexpf(1.0f, -6)) {
        /* subnormal range: quantum 2^-9; rint() is round-half-even */
        float q = rintf(a * 512.0f);          /* exact scaling by a power of 2 */
        int qi = (int)q;                      /* 0..8; 8 == min normal 0x08 */
        return sign | (uint8_t)qi;
    }
    /* normal: keep 3 mantissa bits with RNE on the fp32 bit pattern */
    uint32_t ua = f32_bits(a);
    uint32_t lsb = (ua >> 20) & 1u;
    ua += 0x7FFFFu + lsb;                      /* round at bit 20 */
    int e32 = (int)(ua >> 23) - 127;           /* unbiased exponent after rounding */
    uint32_t man = (ua >> 20) & 7u;
    int e8 = e32 + 7;
    if (e8 > 15 || (e8 == 15 && man == 7)) return sign | 0x7E; /* rounded past 448 */
    return sign | (uint8_t)((e8 << 3) | man);
}

/* asm_f4gemm/f4gemm_ref.hpp:29-41 */
ORC_API float orc_e8m0_to_f32(uint8_t e)
{
    uint32_t bits;
    if (e == 0) bits = 0x00400000u;
    else if (e == 0xFF) bits = 0x7F800001u;
    else bits = (uint32_t)e << 23;
    return bits_f32(bits);
}

/* fp32 -> bf16 round-to-nearest-even (NaN kept quiet).  The inverse is
 * asm_f4gemm/f4gemm_ref.hpp:43-49 (bf16_to_f32). */
ORC_API uint16_t orc_f32_to_bf16(float x)
{
    uint32_t u = f32_bits(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

ORC_API float orc_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* ------------------------------------------------------------------------- */
/* Seeded N(0,1) generator: std::mt19937_64 (Matsumoto-Nishimura 2000 64-bit   */
/* Mersenne Twister, the C++11 <random> engine) + Box-Muller in double.        */
/* Seeds 1234 / 5678 follow asm_f4gemm/main.cpp:189-190.                      */
/* Rows are generated in blocks of 128; block rb uses seed + rb, so any row   */
/* range (one M-shard of a multi-GPU run) is reproducible on its own.         */
/* ------------------------------------------------------------------------- */
typedef struct { uint64_t mt[312]; int idx; } mt64_t;

static void mt64_seed(mt64_t* s, uint64_t seed)
{
    s->mt[0] = seed;
    for (int i = 1; i < 312; ++i)
        s->mt[i] = 6364136223846793005ULL * (s->mt[i - 1] ^ (s->mt[i - 1] >> 62)) + (uint64_t)i;
    s->idx = 312;
}

static uint64_t mt64_next(mt64_t* s)
{
    if (s->idx >= 312) {
        for (int i = 0; i < 312; ++i) {
            uint64_t x = (s->mt[i] & 0xFFFFFFFF80000000ULL) | (s->mt[(i + 1) % 312] & 0x7FFFFFFFULL);
            uint64_t xa = x >> 1;
            if (x & 1ULL) xa ^= 0xB5026F5AA96619E9ULL;
            s->mt[i] = s->mt[(i + 156) % 312] ^ xa;
        }
        s->idx = 0;
    }
    uint64_t y = s->mt[s->idx++];
    y ^= (y >> 29) & 0x5555555555555555ULL;
    y ^= (y << 17) & 0x71D67FFFEDA60000ULL;
    y ^= (y << 37) & 0xFFF7EEE000000000ULL;
    y ^= y >> 43;
    return y;
}

/* first n outputs of std::mt19937_64(seed) (for the engine self-test) */
ORC_API void orc_mt19937_64(uint64_t seed, uint64_t* out, size_t n)
{
    mt64_t s;
    mt64_seed(&s, seed);
    for (size_t i = 0; i < n; ++i) out[i] = mt64_next(&s);
}

/* out[(r - row0) * cols + c] for r in [row0, row0 + nrows) */
ORC_API void orc_normal_rows(uint64_t seed, int64_t row0, int64_t nrows, int64_t cols, float* out)
{
    const double two_pi = 6.283185307179586476925286766559;
    int64_t rb0 = row0 / 128, rb1 = (row0 + nrows + 127) / 128;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t rb = rb0; rb < rb1; ++rb) {
        mt64_t s;
        mt64_seed(&s, seed + (uint64_t)rb);
        int64_t total = 128 * cols;
        for (int64_t i = 0; i < total; i += 2) {
            double u1 = 1.0 - (double)(mt64_next(&s) >> 11) * 0x1.0p-53; /* (0,1] */
            double u2 = (double)(mt64_next(&s) >> 11) * 0x1.0p-53;       /* [0,1) */
            double rad = sqrt(-2.0 * log(u1));
            double z[2] = { rad * cos(two_pi * u2), rad * sin(two_pi * u2) };
            for (int j = 0; j < 2 && i + j < total; ++j) {
                int64_t r = rb * 128 + (i + j) / cols;
                int64_t c = (i + j) % cols;
                if (r >= row0 && r < row0 + nrows) out[(r - row0) * cols + c] = (float)z[j];
            }
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Quantisers (the data recipe of the benchmark configs)                     */
/* ------------------------------------------------------------------------- */

/* Exact UE8M0 exponent for one 1x32 block: the smallest e with 2^e*448 >= amax,
 * i.e. s = 2^ceil(log2(amax/448)) evaluated in real arithmetic (the rounding
 * of mla_agentic_v0/flash_mla/quant.py:28-37 without its fp32 division), then
 * biased and clamped to [1, 254]; an all-zero block gets 1 (2^-126, the
 * clamp(min=2**-126) of quant.py:34). */
ORC_API uint8_t orc_mx_scale_byte(float amax)
{
    if (!(amax > 0.0f)) return 1;
    int ex;
    float mant = frexpf(amax, &ex);        /* amax = mant * 2^ex, mant in [0.5,1) */
    int e = (mant <= 0.875f) ? ex - 9 : ex - 8; /* 448 = 0.875 * 2^9 */
    int b = e + 127;
    if (b < 1) b = 1;
    if (b > 254) b = 254;
    return (uint8_t)b;
}

/* MXFP8 quantiser: x [rows, K] fp32 -> q [rows, K] E4M3 and sf [rows, ceil(K/32)]
 * UE8M0 (plain row-major, the "unpadded [rows, K/32]" buffer that
 * asm_f4gemm/f4gemm_ref.hpp:141 calls `scales`). */
ORC_API void orc_quant_mx(const float* x, int64_t rows, int64_t K, uint8_t* q, uint8_t* sf)
{
    int64_t nb = (K + 31) / 32;
#pragma omp parallel for
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            float amax = 0.0f;
            int64_t k0 = b * 32, k1 = k0 + 32 < K ? k0 + 32 : K;
            for (int64_t k = k0; k < k1; ++k) { float a = fabsf(x[r * K + k]); if (a > amax) amax = a; }
            uint8_t e = orc_mx_scale_byte(amax);
            sf[r * nb + b] = e;
            float inv = ldexpf(1.0f, 127 - (int)e); /* exact 1/s */
            for (int64_t k = k0; k < k1; ++k) q[r * K + k] = orc_f32_to_e4m3(x[r * K + k] * inv);
        }
    }
}

/* fp32 scale of one block: amax/448 (fp32 division), 1.0 for an all-zero block. */
static inline float blk_scale(float amax) { return amax > 0.0f ? amax / 448.0f : 1.0f; }

/* 1x128 quantiser for activations (GROUP_M=1, GROUP_K=128):
 * x [rows, K] -> q, sf laid out [K/128, rows] (stride_sfa = rows, the layout of
 * opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_host.cc:78,244).  Also the
 * GROUP_N=1 weight quantiser (SFB [K/128, N], block_scale_1x128x1 host.cc:90,278). */
ORC_API void orc_quant_1x128(const float* x, int64_t rows, int64_t K, uint8_t* q, float* sf)
{
    int64_t nb = K / 128;
#pragma omp parallel for
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            float amax = 0.0f;
            for (int64_t k = b * 128; k < b * 128 + 128; ++k) { float a = fabsf(x[r * K + k]); if (a > amax) amax = a; }
            float s = blk_scale(amax);
            sf[b * rows + r] = s;
            for (int64_t k = b * 128; k < b * 128 + 128; ++k) q[r * K + k] = orc_f32_to_e4m3(x[r * K + k] / s);
        }
    }
}

/* 128x128 quantiser for weights (GROUP_N=128, GROUP_K=128): x [N, K] -> q and
 * sf laid out [N/128, K/128] (stride_sfb = K/128, gemm_a8w8_blockscale_host.cc:79,245). */
ORC_API void orc_quant_128x128(const float* x, int64_t N, int64_t K, uint8_t* q, float* sf)
{
    int64_t nbn = N / 128, nbk = K / 128;
#pragma omp parallel for collapse(2)
    for (int64_t bn = 0; bn < nbn; ++bn) {
        for (int64_t bk = 0; bk < nbk; ++bk) {
            float amax = 0.0f;
            for (int64_t n = bn * 128; n < bn * 128 + 128; ++n)
                for (int64_t k = bk * 128; k < bk * 128 + 128; ++k) { float a = fabsf(x[n * K + k]); if (a > amax) amax = a; }
            float s = blk_scale(amax);
            sf[bn * nbk + bk] = s;
            for (int64_t n = bn * 128; n < bn * 128 + 128; ++n)
                for (int64_t k = bk * 128; k < bk * 128 + 128; ++k) q[n * K + k] = orc_f32_to_e4m3(x[n * K + k] / s);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Reference GEMMs                                                           */
/* ------------------------------------------------------------------------- */

static float g_e4m3[256];
static int g_e4m3_ready = 0;
static void e4m3_table(void)
{
    if (g_e4m3_ready) return;
    for (int i = 0; i < 256; ++i) g_e4m3[i] = orc_e4m3_to_f32((uint8_t)i);
    g_e4m3_ready = 1;
}

/* opus_gemm/block_scale_gemm/gemm_a8w8_blockscale_host.cc:66-90 (gemm_ref):
 * fp32 running sum of a*b*(sa*sb) in k order, SFA[kg*stride_sfa + m/group_m],
 * SFB[(n/group_n)*stride_sfb + kg].  `rows` limits the computed rows (the CPU
 * baseline samples a row subset); pass m for the full product. */
ORC_API void orc_gemm_blockscale(const uint8_t* a, const uint8_t* b, const float* sfa, const float* sfb,
                                 float* c, int m, int n, int k, int lda, int ldb, int ldc,
                                 int stride_sfa, int stride_sfb, int group_m, int group_n, int group_k)
{
    e4m3_table();
#pragma omp parallel for collapse(2)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t* a_row = a + (int64_t)i * lda;
            const uint8_t* b_row = b + (int64_t)j * ldb;
            const int m_group = i / group_m;
            const int n_group = j / group_n;
            float sum = 0.0f;
            for (int kg = 0; kg < k / group_k; ++kg) {
                const float scale = sfa[(int64_t)kg * stride_sfa + m_group] * sfb[(int64_t)n_group * stride_sfb + kg];
                for (int p = kg * group_k; p < kg * group_k + group_k; ++p)
                    sum += g_e4m3[a_row[p]] * g_e4m3[b_row[p]] * scale;
            }
            c[(int64_t)i * ldc + j] = sum;
        }
    }
}

/* opus_gemm/block_scale_1x128x1_gemm/gemm_a8w8_1x128x1_blockscale_host.cc:77-101:
 * identical loop, SFB indexed [kg*stride_sfb + n/group_n] (layout [K/128, N]). */
ORC_API void orc_gemm_blockscale_1x128x1(const uint8_t* a, const uint8_t* b, const float* sfa, const float* sfb,
                                         float* c, int m, int n, int k, int lda, int ldb, int ldc,
                                         int stride_sfa, int stride_sfb, int group_m, int group_n, int group_k)
{
    e4m3_table();
#pragma omp parallel for collapse(2)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t* a_row = a + (int64_t)i * lda;
            const uint8_t* b_row = b + (int64_t)j * ldb;
            const int m_group = i / group_m;
            const int n_group = j / group_n;
            float sum = 0.0f;
            for (int kg = 0; kg < k / group_k; ++kg) {
                const float scale = sfa[(int64_t)kg * stride_sfa + m_group] * sfb[(int64_t)kg * stride_sfb + n_group];
                for (int p = kg * group_k; p < kg * group_k + group_k; ++p)
                    sum += g_e4m3[a_row[p]] * g_e4m3[b_row[p]] * scale;
            }
            c[(int64_t)i * ldc + j] = sum;
        }
    }
}

/* f64-accumulate variant of the two block-scale loops above (tighter checker);
 * sfb_kmajor = 0 -> SFB[(n/gn)*stride_sfb + kg], 1 -> SFB[kg*stride_sfb + n/gn]. */
ORC_API void orc_gemm_blockscale_f64(const uint8_t* a, const uint8_t* b, const float* sfa, const float* sfb,
                                     double* c, int m, int n, int k, int lda, int ldb, int ldc,
                                     int stride_sfa, int stride_sfb, int group_m, int group_n, int group_k,
                                     int sfb_kmajor)
{
    e4m3_table();
#pragma omp parallel for collapse(2)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            double sum = 0.0;
            for (int kg = 0; kg < k / group_k; ++kg) {
                double sb = sfb_kmajor ? sfb[(int64_t)kg * stride_sfb + j / group_n]
                                       : sfb[(int64_t)(j / group_n) * stride_sfb + kg];
                double part = 0.0;
                for (int p = kg * group_k; p < kg * group_k + group_k; ++p)
                    part += (double)g_e4m3[a[(int64_t)i * lda + p]] * (double)g_e4m3[b[(int64_t)j * ldb + p]];
                sum += part * (double)sfa[(int64_t)kg * stride_sfa + i / group_m] * sb;
            }
            c[(int64_t)i * ldc + j] = sum;
        }
    }
}

/* opus_gemm/fp8_gemm/gemm_a8w8_8wave.cc:601-613 (no scales; the B200 library's
 * per-tensor alpha is applied by the caller of this checker). */
ORC_API void orc_gemm_a8w8(const uint8_t* a, const uint8_t* b, float* c, int m, int n, int k,
                           int lda, int ldb, int ldc)
{
    e4m3_table();
#pragma omp parallel for collapse(2)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int p = 0; p < k; ++p)
                sum += g_e4m3[a[(int64_t)i * lda + p]] * g_e4m3[b[(int64_t)j * ldb + p]];
            c[(int64_t)i * ldc + j] = sum;
        }
    }
}

/* opus_fmm/flatmm_a8w8_gfx950.cc:586-597: gemm_ref with B stored [K, N]
 * (b[p*ldb + j]), the source layout its shuffle_b consumes. */
ORC_API void orc_gemm_a8w8_kn(const uint8_t* a, const uint8_t* b, float* c, int m, int n, int k,
                              int lda, int ldb, int ldc)
{
    e4m3_table();
#pragma omp parallel for collapse(2)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int p = 0; p < k; ++p)
                sum += g_e4m3[a[(int64_t)i * lda + p]] * g_e4m3[b[(int64_t)p * ldb + j]];
            c[(int64_t)i * ldc + j] = sum;
        }
    }
}

/* MXFP8 reference: dequantise every element as decode(q) * 2^(e-127) (the
 * make_operand dequant of asm_f4gemm/f4gemm_ref.hpp:167-173 with E4M3 in place
 * of the e2m1 LUT), then D = alpha * A.B^T accumulated like
 * f4gemm_ref.hpp:181-222.  acc_f64 = 1 reproduces reference_gemm's double
 * accumulation; 0 accumulates in fp32 (the fp32-accumulate acceptance form).
 * sfa/sfb are plain row-major [rows, sf_ld] UE8M0 (sf_ld >= ceil(K/32)). */
ORC_API void orc_gemm_mx(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb,
                         int m, int n, int k, int lda, int ldb, int sfa_ld, int sfb_ld,
                         float alpha, int acc_f64, float* d, int ldd)
{
    e4m3_table();
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t* ar = a + (int64_t)i * lda;
            const uint8_t* br = b + (int64_t)j * ldb;
            double acc64 = 0.0;
            float acc32 = 0.0f;
            for (int p0 = 0; p0 < k; p0 += 32) {
                /* the block's two scales, decoded once (same values per element) */
                const float s_a = orc_e8m0_to_f32(sfa[(int64_t)i * sfa_ld + p0 / 32]);
                const float s_b = orc_e8m0_to_f32(sfb[(int64_t)j * sfb_ld + p0 / 32]);
                const int p1 = p0 + 32 < k ? p0 + 32 : k;
                for (int p = p0; p < p1; ++p) {
                    const float va = g_e4m3[ar[p]] * s_a;   /* dequantised element, exact */
                    const float vb = g_e4m3[br[p]] * s_b;
                    if (acc_f64) acc64 += (double)va * (double)vb;
                    else acc32 += va * vb;
                }
            }
            d[(int64_t)i * ldd + j] = acc_f64 ? alpha * (float)acc64 : alpha * acc32;
        }
    }
}

/* MXFP4 (OCP e2m1) element decode: the nibble -> value table of
 * asm_f4gemm/f4gemm_ref.hpp:24-26.  Byte i of a packed row holds element 2i in
 * its low nibble and element 2i+1 in its high nibble (f4gemm_ref.hpp:22-23). */
static const float k_e2m1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                 -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

ORC_API float orc_e2m1_to_f32(uint8_t nib) { return k_e2m1[nib & 15]; }

/* fp32 -> e2m1 nibble, round to nearest with ties to the even code (codes 0, 2, 4,
 * 6 have a zero mantissa bit), saturating at 6: the thresholds are the midpoints
 * of the e2m1 grid {0, 0.5, 1, 1.5, 2, 3, 4, 6}, all exact in fp32.  The sign
 * bit follows the sign of x (so -0.1 gives -0).  NaN maps to code 7 | sign. */
ORC_API uint8_t orc_f32_to_e2m1(float x)
{
    uint8_t sign = (f32_bits(x) >> 31) ? 8 : 0;
    float a = fabsf(x);
    uint8_t c;
    if (a != a) c = 7;
    else if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return sign | c;
}

/* MXFP4 block scale: the reference's MX rule s = 2^ceil(log2(amax / max_elem))
 * (mla_agentic_v0/flash_mla/quant.py:28-37, E4M3's 448) with e2m1's largest value
 * 6 in its place, so every |x / s| <= 6; biased and clamped to [1, 254]; an
 * all-zero block gets 1 (2^-126).  The reference ships no MXFP4 quantiser of its
 * own (aiter's dynamic_mxfp4_quant is not part of it). */
ORC_API uint8_t orc_mxfp4_scale_byte(float amax)
{
    if (!(amax > 0.0f)) return 1;
    int ex;
    float mant = frexpf(amax, &ex);        /* amax = mant * 2^ex, mant in [0.5,1) */
    int e = (mant <= 0.75f) ? ex - 3 : ex - 2; /* 6 = 0.75 * 2^3 */
    int b = e + 127;
    if (b < 1) b = 1;
    if (b > 254) b = 254;
    return (uint8_t)b;
}

/* MXFP4 quantiser: x [rows, K] fp32 -> packed e2m1 q [rows, K/2] (element 2i in the
 * low nibble) and sf [rows, K/32] UE8M0.  K % 32 == 0. */
ORC_API void orc_quant_mxfp4(const float* x, int64_t rows, int64_t K, uint8_t* q, uint8_t* sf)
{
    int64_t nb = K / 32;
#pragma omp parallel for
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            float amax = 0.0f;
            for (int64_t k = b * 32; k < b * 32 + 32; ++k) { float a = fabsf(x[r * K + k]); if (a > amax) amax = a; }
            uint8_t e = orc_mxfp4_scale_byte(amax);
            sf[r * nb + b] = e;
            float inv = ldexpf(1.0f, 127 - (int)e); /* exact 1/s */
            for (int64_t k = b * 32; k < b * 32 + 32; k += 2) {
                uint8_t lo = orc_f32_to_e2m1(x[r * K + k] * inv);
                uint8_t hi = orc_f32_to_e2m1(x[r * K + k + 1] * inv);
                q[r * (K / 2) + k / 2] = (uint8_t)((hi << 4) | lo);
            }
        }
    }
}

/* MXFP4 reference GEMM, the f4gemm path itself: every element dequantised as
 * e2m1(nibble) * 2^(e-127) (make_operand, f4gemm_ref.hpp:150-177), then
 * D = alpha * A.B^T accumulated in f64 like reference_gemm (f4gemm_ref.hpp:181-222)
 * when acc_f64 = 1, or in fp32.  a/b are packed [rows][lda_bytes] with K
 * elements per row (K even); sfa/sfb plain row-major [rows][sf_ld] UE8M0. */
ORC_API void orc_gemm_mxfp4(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb,
                            int m, int n, int k, int lda_bytes, int ldb_bytes, int sfa_ld, int sfb_ld,
                            float alpha, int acc_f64, float* d, int ldd)
{
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            const uint8_t* ar = a + (int64_t)i * lda_bytes;
            const uint8_t* br = b + (int64_t)j * ldb_bytes;
            double acc64 = 0.0;
            float acc32 = 0.0f;
            for (int p0 = 0; p0 < k; p0 += 32) {
                const float s_a = orc_e8m0_to_f32(sfa[(int64_t)i * sfa_ld + p0 / 32]);
                const float s_b = orc_e8m0_to_f32(sfb[(int64_t)j * sfb_ld + p0 / 32]);
                const int p1 = p0 + 32 < k ? p0 + 32 : k;
                for (int p = p0; p < p1; ++p) {
                    const uint8_t ba = ar[p >> 1], bb = br[p >> 1];
                    const float va = k_e2m1[(p & 1) ? (ba >> 4) : (ba & 15)] * s_a;  /* exact */
                    const float vb = k_e2m1[(p & 1) ? (bb >> 4) : (bb & 15)] * s_b;
                    if (acc_f64) acc64 += (double)va * (double)vb;
                    else acc32 += va * vb;
                }
            }
            d[(int64_t)i * ldd + j] = acc_f64 ? alpha * (float)acc64 : alpha * acc32;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Layout transforms                                                         */
/* ------------------------------------------------------------------------- */

/* asm_f4gemm/f4gemm_ref.hpp:81-96: view(N/16, 16, Kp/32, 2, 16).permute(0,2,3,1,4)
 * on a byte buffer [N, Kp].  For MXFP8 one element is one byte, so Kp = K. */
ORC_API void orc_shuffle_weight_16x16(const uint8_t* src, uint8_t* dst, int N, int Kp)
{
    const int nk = Kp / 32;
    for (int n0 = 0; n0 < N / 16; n0++)
        for (int n1 = 0; n1 < 16; n1++)
            for (int k0 = 0; k0 < nk; k0++)
                for (int k1 = 0; k1 < 2; k1++)
                    for (int k2 = 0; k2 < 16; k2++) {
                        size_t s = (size_t)(n0 * 16 + n1) * Kp + k0 * 32 + k1 * 16 + k2;
                        size_t d = ((((size_t)n0 * nk + k0) * 2 + k1) * 16 + n1) * 16 + k2;
                        dst[d] = src[s];
                    }
}

/* asm_f4gemm/f4gemm_ref.hpp:108-130: pad [rows, cols] to [sm, sn] with 0x7F, then
 * view(sm/32, 2, 16, sn/8, 2, 4).permute(0, 3, 5, 2, 4, 1). */
ORC_API void orc_shuffle_scale(const uint8_t* src, int rows, int cols, int sm, int sn, uint8_t* dst)
{
    uint8_t* padded = (uint8_t*)malloc((size_t)sm * sn);
    memset(padded, 0x7F, (size_t)sm * sn);
    for (int r = 0; r < rows; r++) memcpy(&padded[(size_t)r * sn], &src[(size_t)r * cols], cols);
    const int n3 = sn / 8;
    for (int d0 = 0; d0 < sm / 32; d0++)
        for (int d1 = 0; d1 < 2; d1++)
            for (int d2 = 0; d2 < 16; d2++)
                for (int d3 = 0; d3 < n3; d3++)
                    for (int d4 = 0; d4 < 2; d4++)
                        for (int d5 = 0; d5 < 4; d5++) {
                            size_t s = (size_t)(d0 * 32 + d1 * 16 + d2) * sn + d3 * 8 + d4 * 4 + d5;
                            size_t d = (((((size_t)d0 * n3 + d3) * 4 + d5) * 16 + d2) * 2 + d4) * 2 + d1;
                            dst[d] = padded[s];
                        }
    free(padded);
}

/* opus_fmm/flatmm_a8w8_gfx950.cc:638-681 (shuffle_b) for fp8 with W_N=16,
 * W_K=128, wave64: ItemsPerAccess = min(16, 128/4) = 16, so
 * out[n/16][k/16][n%16][k%16] = in[k*N + n] with in stored [K, N]. */
ORC_API void orc_flatmm_shuffle_b(const uint8_t* in_kn, uint8_t* out, int N, int K)
{
    for (int d0 = 0; d0 < N / 16; ++d0)
        for (int d2 = 0; d2 < K / 16; ++d2)
            for (int d1 = 0; d1 < 16; ++d1)
                for (int d3 = 0; d3 < 16; ++d3)
                    out[(((size_t)d0 * (K / 16) + d2) * 16 + d1) * 16 + d3] =
                        in_kn[(size_t)(d2 * 16 + d3) * N + d0 * 16 + d1];
}

/* Plain row-major UE8M0 scales [rows, cols] -> the sm_100 tensor-core scale
 * layout the B200 library consumes natively: 128-row x 4-column atoms of 512 B,
 * byte (r%32)*16 + ((r/32)%4)*4 + (c%4) inside an atom, atoms ordered
 * [row_block][col_block] (col blocks fastest).  Padding is filled with 0x7F
 * (1.0), as f4gemm_ref.hpp:106-107 pads.  dst holds
 * ceil(rows/128) * ceil(cols/4) * 512 bytes. */
ORC_API void orc_sf_to_tc_layout(const uint8_t* src, int rows, int cols, uint8_t* dst)
{
    int rb_n = (rows + 127) / 128, cb_n = (cols + 3) / 4;
    memset(dst, 0x7F, (size_t)rb_n * cb_n * 512);
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) {
            size_t atom = (size_t)(r / 128) * cb_n + (c / 4);
            size_t off = atom * 512 + (size_t)(r % 32) * 16 + ((r / 32) % 4) * 4 + (c % 4);
            dst[off] = src[(size_t)r * cols + c];
        }
}

ORC_API int orc_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
