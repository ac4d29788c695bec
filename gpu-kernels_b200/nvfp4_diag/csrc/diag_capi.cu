// diag_capi.cu — the diagnostic entry points of libnvfp4_diag.so (nvfp4_diag.h): the
// traced GEMM launches, the scale-code check of the fused epilogue's tables.  This
// library is the product's sources built again with NVFP4_DIAG (the traced kernel
// variants) plus this file and probe.cu; the product library holds none of them.
#include <algorithm>

#include "../nvfp4_diag.h"
#include "common.cuh"
#include "epilogue.cuh"
#include "gemm_decode.cuh"
#include "quant_common.cuh"

int epilogue_from(const nvfp4_epilogue *epi, int N, nvfp4::Epi *out);  // capi.cu

namespace nvfp4 {

int gemm_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D, int M,
               int N, int K, unsigned long long *trace, cudaStream_t stream, const Epi &epi);  // gemm_pair.cu
int gemm_validate(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const void *D, int M,
                  int N, int K);

// Decode GEMM with per-CTA %globaltimer stamps (trace: grid x kDecodeTraceSlots u64,
// grid = min(#SMs, tiles x k-blocks)): the launch timeline.
static int decode_trace_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                                 float alpha, uint16_t *D, int M, int N, int K, void *ws, size_t ws_bytes,
                                 unsigned long long *trace, cudaStream_t stream) {
    int st = gemm_validate(A, SFA, B, SFB, D, M, N, K);
    if (st) return st;
    if (M > 128 || !trace) return M > 128 ? NVFP4_ERR_SHAPE : NVFP4_ERR_INVALID;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    if (!ws || ws_bytes < decode::workspace_bytes(M, N, di.sm_count) || (reinterpret_cast<uintptr_t>(ws) & 255u))
        return NVFP4_ERR_WORKSPACE;
    return decode::launch_for(M, false, A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, Epi(), trace, nullptr,
                              nullptr, 0);
}

// Scale codes of blocks with the given bf16 amax values, taken the way the fused GEMM
// epilogue takes them: per-CTA threshold tables of the global scale, no division.
__global__ void __launch_bounds__(256) scale_codes_kernel(const uint16_t *__restrict__ amax, int64_t n,
                                                          const float *__restrict__ gs_ptr,
                                                          uint8_t *__restrict__ codes) {
    __shared__ ScaleTables tab;
    const float gs = *gs_ptr;
    build_scale_tables(&tab, gs, threadIdx.x, blockDim.x);
    __syncthreads();
    const ScaleGuess guess = scale_guess_factor(gs);
    const bool ok = gs_usable(gs);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        codes[i] = (uint8_t)table_scale_code(fabsf(__uint_as_float((uint32_t)amax[i] << 16)), guess, &tab, ok);
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

int nvfp4_gemm_decode_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                            uint16_t *D, int M, int N, int K, void *workspace, size_t workspace_bytes, uint64_t *trace,
                            void *stream) {
    return decode_trace_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, workspace, workspace_bytes,
                                 reinterpret_cast<unsigned long long *>(trace), static_cast<cudaStream_t>(stream));
}

int nvfp4_gemm_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                     uint16_t *D, int M, int N, int K, uint64_t *trace, void *stream) {
    return gemm_trace(A, SFA, B, SFB, alpha, D, M, N, K, reinterpret_cast<unsigned long long *>(trace),
                      static_cast<cudaStream_t>(stream), Epi());
}

int nvfp4_gemm_trace_epilogue(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                              float alpha, uint16_t *D, int M, int N, int K, const nvfp4_epilogue *epi,
                              uint64_t *trace, void *stream) {
    Epi e;
    if (epi) {
        int st = epilogue_from(epi, N, &e);
        if (st) return st;
    }
    return gemm_trace(A, SFA, B, SFB, alpha, e.q ? static_cast<void *>(e.q) : D, M, N, K,
                      reinterpret_cast<unsigned long long *>(trace), static_cast<cudaStream_t>(stream), e);
}

int nvfp4_scale_codes(const uint16_t *amax_bf16, int64_t n, const float *global_scale, uint8_t *codes, void *stream) {
    if (!amax_bf16 || !global_scale || !codes) return NVFP4_ERR_INVALID;
    if (n < 1) return NVFP4_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(amax_bf16) & 1u) || (reinterpret_cast<uintptr_t>(global_scale) & 3u))
        return NVFP4_ERR_ALIGN;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, di.sm_count);
    scale_codes_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(amax_bf16, n, global_scale,
                                                                                          codes);
    count_launch();
    return cuda_status(cudaGetLastError());
}

}  // extern "C"
