/*
 * CPU restatement of the NVFP4 path — TEST INFRASTRUCTURE ONLY (see the header
 * nvfp4_oracle.h for what may load it and what it restates).
 *
 * Build: oracle/build_oracle.py (gcc -O2 -fopenmp -ffp-contract=off, no
 * fast-math).  The quantizer part must be IEEE-exact: every fp32 operation is
 * a single correctly-rounded op, matching the __f*_rn intrinsics used on the GPU.
 */
#include "nvfp4_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

int nvfp4o_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static inline int pick_threads(int nthreads) {
    return nthreads > 0 ? nthreads : nvfp4o_max_threads();
}

/* ---------------------------------------------------------------------------
 * e2m1 (FP4): sign bit 3, exponent bits 2:1 (bias 1), mantissa bit 0.
 * Magnitudes by code 0..7: 0, 0.5, 1, 1.5, 2, 3, 4, 6.  No inf/NaN.
 * ------------------------------------------------------------------------- */
static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float nvfp4o_e2m1_decode(uint8_t code) {
    float m = kE2M1[code & 7];
    return (code & 8) ? -m : m;
}

/* Round-to-nearest-even onto the e2m1 grid, saturating at 6 (so +-inf -> +-6).
 * The sign is kept for values that round to zero (-0.1 -> code 8).  NaN maps to
 * code 7 | sign (inputs are required to be finite; this only fixes a value). */
uint8_t nvfp4o_e2m1_encode(float x) {
    uint8_t sign = (f2u(x) >> 31) ? 8 : 0;
    float a = fabsf(x);
    uint8_t c;
    if (a != a) return (uint8_t)(sign | 7);
    /* midpoints between neighbours; ties go to the even code */
    if (a <= 0.25f) c = 0;            /* 0.25 tie -> 0 (even)   */
    else if (a < 0.75f) c = 1;        /* 0.75 tie -> 1.0 (c=2)  */
    else if (a <= 1.25f) c = 2;       /* 1.25 tie -> 1.0 (c=2)  */
    else if (a < 1.75f) c = 3;        /* 1.75 tie -> 2.0 (c=4)  */
    else if (a <= 2.5f) c = 4;        /* 2.5 tie  -> 2.0 (c=4)  */
    else if (a < 3.5f) c = 5;         /* 3.5 tie  -> 4.0 (c=6)  */
    else if (a <= 5.0f) c = 6;        /* 5.0 tie  -> 4.0 (c=6)  */
    else c = 7;                       /* >5 -> 6, saturating     */
    return (uint8_t)(sign | c);
}

/* ---------------------------------------------------------------------------
 * e4m3 (OCP E4M3FN): bias 7, max finite 448 (0x7E), 0x7F = NaN, subnormal
 * quantum 2^-9.
 * ------------------------------------------------------------------------- */
float nvfp4o_e4m3_decode(uint8_t code) {
    int s = code >> 7, e = (code >> 3) & 0xF, m = code & 7;
    float v;
    if (e == 0xF && m == 7) return s ? -NAN : NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf((float)(8 + m), e - 10);
    return s ? -v : v;
}

/* Round-to-nearest-even, saturate finite overflow (and inf) to +-448, NaN -> 0x7F. */
uint8_t nvfp4o_e4m3_encode(float x) {
    uint8_t sign = (f2u(x) >> 31) ? 0x80 : 0;
    float a = fabsf(x);
    if (a != a) return 0x7F;
    if (a >= 448.0f) return (uint8_t)(sign | 0x7E);
    if (a < 0.015625f) {                       /* < 2^-6: subnormal grid 2^-9 */
        float q = nearbyintf(a * 512.0f);      /* exact scaling, RN-even      */
        return (uint8_t)(sign | (uint8_t)q);   /* q==8 is exactly code 0x08   */
    }
    int e;
    frexpf(a, &e);                             /* a = f * 2^e, f in [0.5,1)   */
    e -= 1;                                    /* a in [2^e, 2^(e+1))         */
    float q = nearbyintf(ldexpf(a, 3 - e));    /* mantissa with 3 frac bits   */
    int m = (int)q;
    if (m == 16) { m = 8; e += 1; }
    return (uint8_t)(sign | (uint8_t)(((e + 7) << 3) | (m - 8)));
}

float nvfp4o_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t nvfp4o_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

/* ---------------------------------------------------------------------------
 * Blocked scale layout (matmul/sm100_nvfp4/main.py:16-22): for a [R, K/16]
 * scale tensor with R padded to 128 and rest_k = K/64,
 *   sf.reshape(R/128, 4, 32, rest_k, 4).permute(0, 3, 2, 1, 4)
 * gives offset = ((r/128)*rest_k + k16/4)*512 + (r%32)*16 + ((r/32)%4)*4 + k16%4.
 * ------------------------------------------------------------------------- */
size_t nvfp4o_sf_offset(int64_t r, int64_t k16, int64_t K) {
    int64_t rest_k = K / 64;
    return (size_t)(((r >> 7) * rest_k + (k16 >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (k16 & 3));
}

size_t nvfp4o_sf_bytes(int64_t rows, int64_t K) {
    return (size_t)(((rows + 127) / 128) * 128) * (size_t)(K / 16);
}

void nvfp4o_sf_pack(const uint8_t *src, uint8_t *dst, int64_t rows, int64_t K) {
    int64_t rp = ((rows + 127) / 128) * 128, kb = K / 16;
    memset(dst, 0, nvfp4o_sf_bytes(rows, K));
    for (int64_t r = 0; r < rp && r < rows; r++)
        for (int64_t k = 0; k < kb; k++) dst[nvfp4o_sf_offset(r, k, K)] = src[r * kb + k];
}

void nvfp4o_sf_unpack(const uint8_t *src, uint8_t *dst, int64_t rows, int64_t K) {
    int64_t kb = K / 16;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t k = 0; k < kb; k++) dst[r * kb + k] = src[nvfp4o_sf_offset(r, k, K)];
}

/* ---------------------------------------------------------------------------
 * Quantizer specification (bf16 X[M,K] -> e2m1 Q[M,K/2] + e4m3 SF blocked).
 * For each row r and each 16-element block b (elements x_0..x_15 as fp32):
 *   amax  = max_i |x_i|                          (exact)
 *   sfv   = (amax / 6) / gs                      (two IEEE fp32 divisions)
 *   sf    = e4m3_rn_satfinite(sfv)               (stored scale byte)
 *   denom = float(sf) * gs                       (IEEE fp32 multiply)
 *   inv   = denom == 0 ? 0 : 1 / denom           (IEEE fp32 division)
 *   q_i   = e2m1_rn_satfinite(x_i * inv)         (IEEE fp32 multiply, then RN-even)
 * gs is the fp32 global scale such that x ~= q * sf * gs (typically
 * amax(X) / (6 * 448)); the GEMM's alpha is gs_A * gs_B.  A gs outside
 * [2^-100, FLT_MAX] (zero, negative, NaN, inf, absurdly small) is unusable and
 * every block becomes sf = 0, q = e2m1(x * 0).  With a usable gs and finite x,
 * inv is finite, so x * inv is never NaN.  Padding rows of SF (M..pad128(M))
 * are written as 0.
 * ------------------------------------------------------------------------- */
static void quantize_block(const uint16_t *x, uint8_t *q, uint8_t *sf, float gs) {
    float v[16], amax = 0.0f;
    for (int i = 0; i < 16; i++) {
        v[i] = nvfp4o_bf16_to_f32(x[i]);
        float a = fabsf(v[i]);
        if (a > amax) amax = a;
    }
    uint8_t code = 0;
    float inv = 0.0f;
    if (gs >= 0x1p-100f && gs <= 0x1.fffffep127f) {   /* usable global scale */
        volatile float t = amax / 6.0f;              /* keep the two divisions separate */
        float sfv = t / gs;
        code = nvfp4o_e4m3_encode(sfv);
        float denom = nvfp4o_e4m3_decode(code) * gs;
        inv = (denom == 0.0f) ? 0.0f : 1.0f / denom;
    }
    for (int i = 0; i < 8; i++) {
        uint8_t lo = nvfp4o_e2m1_encode(v[2 * i] * inv);
        uint8_t hi = nvfp4o_e2m1_encode(v[2 * i + 1] * inv);
        q[i] = (uint8_t)(lo | (hi << 4));
    }
    *sf = code;
}

void nvfp4o_quantize(const uint16_t *X, uint8_t *Q, uint8_t *SF, float gs, int64_t M, int64_t K,
                     int nthreads) {
    int64_t kb = K / 16;
    memset(SF, 0, nvfp4o_sf_bytes(M, K));
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t r = 0; r < M; r++) {
        for (int64_t b = 0; b < kb; b++) {
            uint8_t code;
            quantize_block(X + r * K + b * 16, Q + r * (K / 2) + b * 8, &code, gs);
            SF[nvfp4o_sf_offset(r, b, K)] = code;
        }
    }
}

float nvfp4o_amax_bf16(const uint16_t *X, int64_t n, int nthreads) {
    float amax = 0.0f;
#pragma omp parallel for reduction(max : amax) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < n; i++) {
        float a = fabsf(nvfp4o_bf16_to_f32(X[i]));
        if (a > amax) amax = a;
    }
    return amax;
}

/* ---------------------------------------------------------------------------
 * Dequantisation: a[r,k] = e2m1(Q nibble) * e4m3(SF[r, k/16]) in fp32.
 * ------------------------------------------------------------------------- */
static void dequant_rows(const uint8_t *Q, const uint8_t *SF, float *out, int64_t r0, int64_t nrows,
                         int64_t K, int nthreads) {
    int64_t kb = K / 16;
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < nrows; i++) {
        int64_t r = r0 + i;
        const uint8_t *q = Q + r * (K / 2);
        float *o = out + i * K;
        for (int64_t b = 0; b < kb; b++) {
            float s = nvfp4o_e4m3_decode(SF[nvfp4o_sf_offset(r, b, K)]);
            for (int j = 0; j < 8; j++) {
                uint8_t byte = q[b * 8 + j];
                o[b * 16 + 2 * j] = nvfp4o_e2m1_decode(byte & 0xF) * s;
                o[b * 16 + 2 * j + 1] = nvfp4o_e2m1_decode(byte >> 4) * s;
            }
        }
    }
}

void nvfp4o_dequant(const uint8_t *Q, const uint8_t *SF, float *out, int64_t rows, int64_t K,
                    int nthreads) {
    dequant_rows(Q, SF, out, 0, rows, K, nthreads);
}

/* ---------------------------------------------------------------------------
 * fp32 GEMM on dequantised rows: C[i,j] += dot(A[i,:], B[j,:]) (both K-major).
 * ------------------------------------------------------------------------- */
static float dot_scalar(const float *a, const float *b, int64_t n) {
    float acc[8] = {0};
    int64_t k = 0;
    for (; k + 8 <= n; k += 8)
        for (int l = 0; l < 8; l++) acc[l] += a[k + l] * b[k + l];
    float s = 0.0f;
    for (int l = 0; l < 8; l++) s += acc[l];
    for (; k < n; k++) s += a[k] * b[k];
    return s;
}

#if defined(__x86_64__)
__attribute__((target("avx2,fma"))) static inline float hsum256(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    lo = _mm_add_ps(lo, hi);
    lo = _mm_add_ps(lo, _mm_movehl_ps(lo, lo));
    lo = _mm_add_ss(lo, _mm_movehdup_ps(lo));
    return _mm_cvtss_f32(lo);
}

/* 2 rows of A x 4 rows of B over kc elements (kc % 8 == 0), accumulating into C. */
__attribute__((target("avx2,fma"))) static void micro_2x4(const float *a0, const float *a1,
                                                          const float *b0, const float *b1,
                                                          const float *b2, const float *b3,
                                                          int64_t kc, float *c0, float *c1) {
    __m256 s00 = _mm256_setzero_ps(), s01 = s00, s02 = s00, s03 = s00;
    __m256 s10 = s00, s11 = s00, s12 = s00, s13 = s00;
    for (int64_t k = 0; k < kc; k += 8) {
        __m256 x0 = _mm256_loadu_ps(a0 + k), x1 = _mm256_loadu_ps(a1 + k);
        __m256 y = _mm256_loadu_ps(b0 + k);
        s00 = _mm256_fmadd_ps(x0, y, s00); s10 = _mm256_fmadd_ps(x1, y, s10);
        y = _mm256_loadu_ps(b1 + k);
        s01 = _mm256_fmadd_ps(x0, y, s01); s11 = _mm256_fmadd_ps(x1, y, s11);
        y = _mm256_loadu_ps(b2 + k);
        s02 = _mm256_fmadd_ps(x0, y, s02); s12 = _mm256_fmadd_ps(x1, y, s12);
        y = _mm256_loadu_ps(b3 + k);
        s03 = _mm256_fmadd_ps(x0, y, s03); s13 = _mm256_fmadd_ps(x1, y, s13);
    }
    c0[0] += hsum256(s00); c0[1] += hsum256(s01); c0[2] += hsum256(s02); c0[3] += hsum256(s03);
    c1[0] += hsum256(s10); c1[1] += hsum256(s11); c1[2] += hsum256(s12); c1[3] += hsum256(s13);
}
#endif

/* C[mrows, ncols] = A[mrows,K] . B[ncols,K]^T, cache-blocked, OpenMP over tiles. */
static void sgemm_nt(const float *A, const float *B, float *C, int64_t mrows, int64_t ncols, int64_t K,
                     int nthreads) {
    const int64_t MB = 32, NB = 128, KC = 512;
    int64_t mt = (mrows + MB - 1) / MB, nt = (ncols + NB - 1) / NB;
    int use_avx2 = 0;
#if defined(__x86_64__)
    __builtin_cpu_init();
    use_avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#endif
    memset(C, 0, (size_t)mrows * (size_t)ncols * sizeof(float));
#pragma omp parallel for schedule(dynamic) collapse(2) num_threads(pick_threads(nthreads))
    for (int64_t ti = 0; ti < mt; ti++) {
        for (int64_t tj = 0; tj < nt; tj++) {
            int64_t i0 = ti * MB, i1 = i0 + MB < mrows ? i0 + MB : mrows;
            int64_t j0 = tj * NB, j1 = j0 + NB < ncols ? j0 + NB : ncols;
            for (int64_t k0 = 0; k0 < K; k0 += KC) {
                int64_t kc = k0 + KC < K ? KC : K - k0;
                int64_t i = i0;
#if defined(__x86_64__)
                if (use_avx2 && kc % 8 == 0) {
                    for (; i + 2 <= i1; i += 2) {
                        int64_t j = j0;
                        for (; j + 4 <= j1; j += 4)
                            micro_2x4(A + i * K + k0, A + (i + 1) * K + k0, B + j * K + k0,
                                      B + (j + 1) * K + k0, B + (j + 2) * K + k0, B + (j + 3) * K + k0,
                                      kc, C + i * ncols + j, C + (i + 1) * ncols + j);
                        for (; j < j1; j++) {
                            C[i * ncols + j] += dot_scalar(A + i * K + k0, B + j * K + k0, kc);
                            C[(i + 1) * ncols + j] += dot_scalar(A + (i + 1) * K + k0, B + j * K + k0, kc);
                        }
                    }
                }
#endif
                for (; i < i1; i++)
                    for (int64_t j = j0; j < j1; j++)
                        C[i * ncols + j] += dot_scalar(A + i * K + k0, B + j * K + k0, kc);
            }
        }
    }
}

void nvfp4o_sgemm_nt(const float *A, const float *B, float alpha, int64_t mrows, int64_t ncols, int64_t K,
                     float *D32, uint16_t *D16, int nthreads) {
    float *C = (float *)malloc((size_t)mrows * (size_t)ncols * sizeof(float));
    if (!C) return;
    sgemm_nt(A, B, C, mrows, ncols, K, nthreads);
    int64_t total = mrows * ncols;
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < total; i++) {
        float v = alpha * C[i];
        if (D32) D32[i] = v;
        if (D16) D16[i] = nvfp4o_f32_to_bf16(v);
    }
    free(C);
}

void nvfp4o_dequant_rows(const uint8_t *Q, const uint8_t *SF, float *out, int64_t r0, int64_t nrows, int64_t K,
                         int nthreads) {
    dequant_rows(Q, SF, out, r0, nrows, K, nthreads);
}

void nvfp4o_gemm_rows(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                      float alpha, int64_t M, int64_t N, int64_t K, int64_t m0, int64_t mrows,
                      float *D32, uint16_t *D16, int nthreads) {
    (void)M;
    float *Af = (float *)malloc((size_t)mrows * (size_t)K * sizeof(float));
    float *Bf = (float *)malloc((size_t)N * (size_t)K * sizeof(float));
    float *C = (float *)malloc((size_t)mrows * (size_t)N * sizeof(float));
    if (!Af || !Bf || !C) { free(Af); free(Bf); free(C); return; }
    dequant_rows(A, SFA, Af, m0, mrows, K, nthreads);
    dequant_rows(B, SFB, Bf, 0, N, K, nthreads);
    sgemm_nt(Af, Bf, C, mrows, N, K, nthreads);
    int64_t total = mrows * N;
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < total; i++) {
        float v = alpha * C[i];
        if (D32) D32[i] = v;
        if (D16) D16[i] = nvfp4o_f32_to_bf16(v);
    }
    free(Af); free(Bf); free(C);
}

/* ---------------------------------------------------------------------------
 * Fused GEMM epilogue (the product's nvfp4_gemm_epilogue; the reference has no
 * epilogue beyond fp16 conversion).  Per element, each fp32 step one IEEE
 * round-to-nearest operation (this file is built with -ffp-contract=off):
 *   y = alpha * acc;  y = y + bias[n];  y = act(y);  out = bf16_rn(y)
 * act: 0 none, 1 relu max(y, 0), 2 silu y / (1 + exp(-y)),
 *      3 gelu (tanh form) 0.5 y (1 + tanh(0.7978845608028654 (y + 0.044715 y^3))).
 * exp/tanh are the C library's; the GPU uses its approximate exp, reciprocal and
 * tanh instructions, so silu/gelu agree within the GEMM tolerance, not bit for bit.
 * ------------------------------------------------------------------------- */
void nvfp4o_epilogue(const float *acc, const uint16_t *bias, int act, float alpha, int64_t rows, int64_t N,
                     float *Y32, uint16_t *Y16, int nthreads) {
    const int64_t total = rows * N;
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < total; i++) {
        float y = alpha * acc[i];
        if (bias) y = y + nvfp4o_bf16_to_f32(bias[i % N]);
        if (act == 1) {
            y = fmaxf(y, 0.0f);
        } else if (act == 2) {
            y = y / (1.0f + expf(-y));
        } else if (act == 3) {
            const float y3 = (y * y) * y;
            const float u = 0.7978845608028654f * (y + 0.044715f * y3);
            y = (0.5f * y) * (1.0f + tanhf(u));
        }
        if (Y32) Y32[i] = y;
        if (Y16) Y16[i] = nvfp4o_f32_to_bf16(y);
    }
}

/* SwiGLU epilogue over gate / up columns interleaved in blocks of 16: output column
 * c of [rows, N/2] (N % 32 == 0) takes gate column 32*(c/16) + c%16 and up column
 * 32*(c/16) + 16 + c%16 of the accumulator; with y = alpha * acc (+ bias[col]) for
 * each, out = silu(y_gate) * y_up = y_gate / (1 + exp(-y_gate)) * y_up in fp32, then
 * bf16 (round to nearest even).  The GPU computes silu with tanh.approx, so the two
 * agree within the GEMM tolerance, not bit for bit. */
void nvfp4o_epilogue_swiglu(const float *acc, const uint16_t *bias, float alpha, int64_t rows, int64_t N,
                            float *Y32, uint16_t *Y16, int nthreads) {
    const int64_t half = N / 2, total = rows * half;
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < total; i++) {
        const int64_t r = i / half, c = i % half;
        const int64_t g = 32 * (c / 16) + c % 16, u = g + 16;
        float yg = alpha * acc[r * N + g], yu = alpha * acc[r * N + u];
        if (bias) {
            yg = yg + nvfp4o_bf16_to_f32(bias[g]);
            yu = yu + nvfp4o_bf16_to_f32(bias[u]);
        }
        const float y = yg / (1.0f + expf(-yg)) * yu;
        if (Y32) Y32[i] = y;
        if (Y16) Y16[i] = nvfp4o_f32_to_bf16(y);
    }
}

/* ---------------------------------------------------------------------------
 * Deterministic inputs: splitmix64 counter stream + Box-Muller in double.
 * ------------------------------------------------------------------------- */
static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static inline double unit_open(uint64_t bits) {  /* (0,1) */
    return ((double)(bits >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

static inline double normal_at(uint64_t seed, uint64_t i) {
    uint64_t base = splitmix64(seed ^ 0x5851F42D4C957F2Dull) + 2 * i;
    double u1 = unit_open(splitmix64(base)), u2 = unit_open(splitmix64(base + 1));
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

void nvfp4o_fill_normal_bf16(uint16_t *X, int64_t n, uint64_t seed, float stddev, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < n; i++) X[i] = nvfp4o_f32_to_bf16((float)(stddev * normal_at(seed, (uint64_t)i)));
}

/* Student-t with 3 degrees of freedom: Z / sqrt(chi2_3 / 3), chi2_3 = sum of three
 * squared normals; n_outlier_cols distinct columns (seeded choice) are multiplied
 * by outlier_gain. */
void nvfp4o_fill_student_t3_bf16(uint16_t *X, int64_t rows, int64_t cols, uint64_t seed,
                                 int n_outlier_cols, float outlier_gain, int nthreads) {
    char *is_out = (char *)calloc((size_t)cols, 1);
    uint64_t s = seed ^ 0xD1B54A32D192ED03ull;
    for (int c = 0; c < n_outlier_cols && c < cols;) {
        s = splitmix64(s);
        int64_t col = (int64_t)(s % (uint64_t)cols);
        if (!is_out[col]) { is_out[col] = 1; c++; }
    }
    int64_t n = rows * cols;
#pragma omp parallel for schedule(static) num_threads(pick_threads(nthreads))
    for (int64_t i = 0; i < n; i++) {
        uint64_t j = (uint64_t)i * 4;
        double z = normal_at(seed, j);
        double c1 = normal_at(seed, j + 1), c2 = normal_at(seed, j + 2), c3 = normal_at(seed, j + 3);
        double chi = (c1 * c1 + c2 * c2 + c3 * c3) / 3.0;
        double t = z / sqrt(chi);
        if (is_out[i % cols]) t *= outlier_gain;
        X[i] = nvfp4o_f32_to_bf16((float)t);
    }
    free(is_out);
}
