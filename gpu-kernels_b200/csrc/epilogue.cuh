// epilogue.cuh — the fused GEMM epilogue shared by the persistent (single-CTA,
// CTA-pair) and decode kernels: per output element
//   y = alpha * acc                  (fp32, one IEEE multiply)
//   y = y + float(bias[n])           (bf16 bias over N, optional)
//   y = act(y)                       (none, relu, silu, gelu with the tanh form)
// then either D = bf16_rn(y), or the bf16_rn(y) row segment quantized to NVFP4 with
// a given global scale (the standalone quantizer's arithmetic, quant_common.cuh),
// so a fused NVFP4 output equals nvfp4_quantize of the fused bf16 output byte for byte.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "quant_common.cuh"

namespace nvfp4 {

enum : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActGeluTanh = 3 };

struct Epi {
    const uint16_t *bias = nullptr;  // bf16 [N], or nullptr
    int act = kActNone;
    uint8_t *q = nullptr;            // NVFP4 output codes [M, N/2]; nullptr = bf16 D
    uint8_t *sf = nullptr;           // blocked e4m3 scales of the output [pad128(M) * N/16]
    const float *gs = nullptr;       // device fp32 global scale of the output
    __host__ __device__ bool plain() const { return bias == nullptr && act == kActNone && q == nullptr; }
};

__device__ __forceinline__ float bf16_bits_to_float(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ float round_bf16(float y) { return __bfloat162float(__float2bfloat16_rn(y)); }

__device__ __forceinline__ float epi_value(float acc, float alpha, const Epi &e, int n) {
    float y = __fmul_rn(acc, alpha);
    if (e.bias) y = __fadd_rn(y, bf16_bits_to_float(e.bias[n]));
    if (e.act == kActRelu) {
        y = fmaxf(y, 0.0f);
    } else if (e.act == kActSilu) {
        // y * sigmoid(y) = y / (1 + exp(-y))
        y = __fdiv_rn(y, __fadd_rn(1.0f, expf(-y)));
    } else if (e.act == kActGeluTanh) {
        // 0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3)))
        const float y3 = __fmul_rn(__fmul_rn(y, y), y);
        const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(y, __fmul_rn(0.044715f, y3)));
        y = __fmul_rn(__fmul_rn(0.5f, y), __fadd_rn(1.0f, tanhf(u)));
    }
    return y;
}

}  // namespace nvfp4
