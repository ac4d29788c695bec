/*
 * nvfp4_diag.h — diagnostic entry points of libnvfp4_diag.so, a separate build of the
 * NVFP4 library (gpu-kernels_b200/nvfp4_diag/) used to measure the kernels, never by
 * the product path.  It holds every entry point of nvfp4_b200.h as well, built from
 * the same sources with the cycle-trace kernel variants compiled in (NVFP4_DIAG).
 * No counterpart in the reference, which only has a host timer and an unused per-SM
 * event recorder (matmul/sm100_nvfp4/profiler.cuh:4-72).
 */
#ifndef NVFP4_DIAG_H
#define NVFP4_DIAG_H

#include "../../include/nvfp4_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * nvfp4_gemm_trace: the CTA-pair GEMM with a per-CTA cycle trace written to `trace`
 * (device, #SMs x 12 uint64; the grid is at most one CTA per SM): [0] MMA wait on full
 * stages, [1] MMA wait on a free accumulator, [2] producer wait on empty stages, [3]
 * epilogue wait on a full accumulator, [4] epilogue drain + stores, [5] tiles, [6]
 * MMA-thread span in cycles, [7] the same in ns, [8]/[9] %globaltimer at CTA
 * entry/exit, [10]/[11] at the first MMA issue / last accumulator commit.
 */
NVFP4_API int nvfp4_gemm_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                               float alpha, uint16_t *D, int M, int N, int K, uint64_t *trace, void *stream);
/* nvfp4_gemm_trace with a fused epilogue (nvfp4_gemm_epilogue's arguments; epi may be
 * NULL): the same trace, for the cost of the epilogue per tile ([3], [4]). */
NVFP4_API int nvfp4_gemm_trace_epilogue(const uint8_t *A, const uint8_t *SFA, const uint8_t *B,
                                        const uint8_t *SFB, float alpha, uint16_t *D, int M, int N, int K,
                                        const nvfp4_epilogue *epi, uint64_t *trace, void *stream);
/* nvfp4_gemm_decode with per-CTA %globaltimer stamps in `trace` (device, grid x 9
 * uint64, grid = min(#SMs, ceil(N/128) * ceil(K/256))): [0] CTA entry, [1] release of
 * the wait on the preceding kernel, [2] first and [3] last ring slot reaching the
 * MMA thread, [4] CTA exit, [5] k-block iterations of the CTA; for its last segment
 * [6] accumulator in registers, [7] arrival counted (a cut tile), [8] partials summed
 * (the tile's last contributor); 0 where a stamp does not apply. */
NVFP4_API int nvfp4_gemm_decode_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                                      float alpha, uint16_t *D, int M, int N, int K, void *workspace,
                                      size_t workspace_bytes, uint64_t *trace, void *stream);
/*
 * nvfp4_probe_mma_rate: measured kind::mxf4nvf4 tensor rate on every SM with operands
 * resident in shared memory (mode 0/1: single CTA without/with the scale copies; 2/3:
 * CTA pair without/with; 4: pair, scale copies batched per 4-MMA stage; 5: pair with
 * N = 192 and the scale copies; 6-9 measure the issuing thread: 6 scale copies alone,
 * 7 N = 64 MMAs, 8 N = 64 MMA + 2 commits, 9 copies + N = 64 MMA + 2 commits; 10 and
 * 11 are modes 4 and 2 with pseudo-random operands and scales instead of zeros).
 * Synchronous; returns TFLOP/s and cycles per iteration (one MMA, or one group of
 * copies in mode 6).
 */
NVFP4_API int nvfp4_probe_mma_rate(int mode, int iters, double *tflops, double *cycles_per_mma);
/* nvfp4_scale_codes: the e4m3 scale code of n blocks given each block's bf16 amax
 * (device, sign ignored) and the device fp32 global scale, computed the way the fused
 * GEMM epilogue computes them for NVFP4 output — from per-launch threshold tables,
 * without a division per block — so that path can be checked against the
 * specification for every bf16 amax. */
NVFP4_API int nvfp4_scale_codes(const uint16_t *amax_bf16, int64_t n, const float *global_scale, uint8_t *codes,
                                void *stream);

#ifdef __cplusplus
}
#endif
#endif
