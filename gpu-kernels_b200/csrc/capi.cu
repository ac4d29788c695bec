// capi.cu — the extern "C" GEMM entry points of libnvfp4_b200 (declared in
// include/nvfp4_b200.h).  Argument checking lives in gemm_validate; kernels in
// gemm.cu, quantize.cu; shared plumbing in runtime.cu.
#include <atomic>

#include "common.cuh"

namespace nvfp4 {
int gemm_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16);
}  // namespace nvfp4

using namespace nvfp4;

static std::atomic<int> g_last_status{NVFP4_OK};

extern "C" {

int nvfp4_gemm(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, uint16_t *D,
               int M, int N, int K, void *stream) {
    return gemm_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, static_cast<cudaStream_t>(stream), false);
}

int nvfp4_gemm_f16(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                   uint16_t *D, int M, int N, int K, void *stream) {
    return gemm_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, static_cast<cudaStream_t>(stream), true);
}

// Reference signature (matmul/sm100_nvfp4/block_scaled_nvfp4.cuh:15-16): note the
// argument order c, sfa, sfb, a, b.
void matmul_nvfp4_b200(void *c, const uint8_t *sfa, const uint8_t *sfb, const uint8_t *a, const uint8_t *b, int M,
                       int N, int K) {
    g_last_status.store(gemm_dispatch(a, sfa, b, sfb, 1.0f, c, M, N, K, nullptr, true));
}

int nvfp4_last_status(void) { return g_last_status.load(); }

}  // extern "C"
