/*
 * CPU restatement of the NVFP4 block-scaled GEMM path — TEST INFRASTRUCTURE ONLY.
 *
 * This library is the parity checker for the CUDA product in gpu-kernels_b200/.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * leg may load it.  The product never calls it and has no CPU fallback.
 *
 * What it restates (reference = Parth-Badgujar/gpu-kernels):
 *   - NVFP4 operand encoding: e2m1 codes, two per byte, element 2i in the low
 *     nibble (torch float4_e2m1fn_x2, matmul/sm100_nvfp4/main.py:12-13);
 *   - e4m3 block scales, one per 16 contiguous K elements, stored in the 128x4
 *     "blocked" layout built by reshape(rest_m,4,32,rest_k,4).permute(0,3,2,1,4)
 *     (matmul/sm100_nvfp4/main.py:16-22);
 *   - the GEMM semantics of the reference's oracle torch._scaled_mm
 *     (matmul/sm100_nvfp4/main.py:25-34): D = sum_k a*sfa * b*sfb, fp32
 *     accumulate, here followed by alpha and bf16 rounding;
 *   - the bf16 -> NVFP4 quantizer.  The reference has none; its specification
 *     (fp32 op order fixed here and mirrored bit-for-bit by the CUDA kernel) is
 *     given at nvfp4o_quantize() below.
 *
 * Parity pin: tests/golden/ holds torch._scaled_mm outputs generated on a B200
 * by tests/golden/make_golden.py; tests/test_oracle_golden.py checks this
 * library against them.
 */
#ifndef NVFP4_ORACLE_H
#define NVFP4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar codecs ---------------------------------------------------- */
float   nvfp4o_e2m1_decode(uint8_t code);            /* code in [0,16)            */
uint8_t nvfp4o_e2m1_encode(float x);                 /* RN-even, saturate to +-6  */
float   nvfp4o_e4m3_decode(uint8_t code);            /* OCP E4M3FN, 0x7F/0xFF NaN */
uint8_t nvfp4o_e4m3_encode(float x);                 /* RN-even, saturate to +-448 */
float   nvfp4o_bf16_to_f32(uint16_t h);
uint16_t nvfp4o_f32_to_bf16(float f);                /* RN-even                    */

/* ---- scale-factor layout ---------------------------------------------- */
/* Byte offset of the scale of (row r, 16-element block k16) in the blocked
 * layout of a [pad128(rows), K/16] scale tensor.  K must be a multiple of 64. */
size_t  nvfp4o_sf_offset(int64_t r, int64_t k16, int64_t K);
size_t  nvfp4o_sf_bytes(int64_t rows, int64_t K);    /* pad128(rows) * K/16        */
void    nvfp4o_sf_pack(const uint8_t *sf_rowmajor, uint8_t *sf_blocked, int64_t rows, int64_t K);
void    nvfp4o_sf_unpack(const uint8_t *sf_blocked, uint8_t *sf_rowmajor, int64_t rows, int64_t K);

/* ---- quantizer ---------------------------------------------------------- */
void    nvfp4o_quantize(const uint16_t *X, uint8_t *Q, uint8_t *SF, float global_scale,
                        int64_t M, int64_t K, int nthreads);
float   nvfp4o_amax_bf16(const uint16_t *X, int64_t n, int nthreads);

/* ---- dequantize + GEMM ---------------------------------------------------- */
void    nvfp4o_dequant(const uint8_t *Q, const uint8_t *SF, float *out,
                       int64_t rows, int64_t K, int nthreads);
/* D[m,n] = alpha * sum_k A[m,k] B[n,k] over rows [m0, m0+mrows) of A.
 * Writes fp32 (D32, may be NULL) and bf16 (D16, may be NULL), both row-major
 * [mrows, N].  Dequantisation of the needed A rows and all of B is part of
 * the call, as in a host dequant-then-GEMM. */
void    nvfp4o_gemm_rows(const uint8_t *A, const uint8_t *SFA, const uint8_t *B,
                         const uint8_t *SFB, float alpha, int64_t M, int64_t N, int64_t K,
                         int64_t m0, int64_t mrows, float *D32, uint16_t *D16, int nthreads);

/* The two halves of nvfp4o_gemm_rows, for callers that dequantise B once:
 * rows [r0, r0+nrows) of a quantized matrix -> fp32, and D = alpha * A . B^T on fp32
 * row-major A [mrows, K], B [ncols, K] (fp32 and/or bf16 out). */
void    nvfp4o_dequant_rows(const uint8_t *Q, const uint8_t *SF, float *out, int64_t r0, int64_t nrows,
                            int64_t K, int nthreads);
void    nvfp4o_sgemm_nt(const float *A, const float *B, float alpha, int64_t mrows, int64_t ncols,
                        int64_t K, float *D32, uint16_t *D16, int nthreads);

/* ---- fused epilogue -------------------------------------------------------- */
/* Y = act(alpha * acc + bias[n]) over rows x N (bias bf16 [N] or NULL; act 0 none,
 * 1 relu, 2 silu, 3 gelu-tanh), fp32 and/or bf16 out. */
void    nvfp4o_epilogue(const float *acc, const uint16_t *bias, int act, float alpha, int64_t rows,
                        int64_t N, float *Y32, uint16_t *Y16, int nthreads);
void nvfp4o_epilogue_swiglu(const float *acc, const uint16_t *bias, float alpha, int64_t rows, int64_t N,
                            float *Y32, uint16_t *Y16, int nthreads);

/* ---- deterministic synthetic inputs -------------------------------------- */
/* Counter-based (splitmix64) so that any slice can be generated alone. */
void    nvfp4o_fill_normal_bf16(uint16_t *X, int64_t n, uint64_t seed, float stddev,
                                int nthreads);
void    nvfp4o_fill_student_t3_bf16(uint16_t *X, int64_t rows, int64_t cols, uint64_t seed,
                                    int n_outlier_cols, float outlier_gain, int nthreads);

int     nvfp4o_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
