// decode_inst.cu — the decode kernel's instantiations for one padded row count,
// NVFP4_DECODE_MPAD (8, 16, 32, 64 or 128; the build compiles this file once per
// value), plain and grouped.
#include "gemm_decode.cuh"

#ifndef NVFP4_DECODE_MPAD
#error "NVFP4_DECODE_MPAD must be defined (8, 16, 32, 64 or 128)"
#endif

namespace nvfp4 {
namespace decode {

template <int MPAD, bool GROUPED>
int launch_mpad(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, uint16_t *D,
                int M, int N, int K, void *ws, cudaStream_t stream, const DeviceInfo &di, const Epi &epi,
                unsigned long long *trace, const int *m_offsets, const float *alphas, int groups) {
    return launch<MPAD, GROUPED>(A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, epi, trace, m_offsets, alphas,
                                 groups);
}

template int launch_mpad<NVFP4_DECODE_MPAD, false>(const uint8_t *, const uint8_t *, const uint8_t *,
                                                   const uint8_t *, float, uint16_t *, int, int, int, void *,
                                                   cudaStream_t, const DeviceInfo &, const Epi &,
                                                   unsigned long long *, const int *, const float *, int);
template int launch_mpad<NVFP4_DECODE_MPAD, true>(const uint8_t *, const uint8_t *, const uint8_t *,
                                                  const uint8_t *, float, uint16_t *, int, int, int, void *,
                                                  cudaStream_t, const DeviceInfo &, const Epi &,
                                                  unsigned long long *, const int *, const float *, int);

}  // namespace decode
}  // namespace nvfp4
