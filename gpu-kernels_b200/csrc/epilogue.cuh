// epilogue.cuh — the fused GEMM epilogue shared by the persistent (single-CTA,
// CTA-pair) and decode kernels: per output element
//   y = alpha * acc                  (fp32, one IEEE multiply)
//   y = y + float(bias[n])           (bf16 bias over N, optional; one IEEE add)
//   y = act(y)                       (none, relu, silu, gelu with the tanh form)
// then either D = bf16_rn(y), or the bf16_rn(y) row segment quantized to NVFP4 with
// a given global scale (the standalone quantizer's arithmetic, quant_common.cuh),
// so a fused NVFP4 output equals nvfp4_quantize of the fused bf16 output byte for byte.
// silu and gelu use the hardware approximations ex2.approx, rcp.approx and
// tanh.approx (relative error below 2^-10 for tanh): the epilogue runs in the shadow
// of the next tile's MMAs only while it stays this cheap.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "quant_common.cuh"

namespace nvfp4 {

enum : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActGeluTanh = 3 };

struct Epi {
    const uint16_t *bias = nullptr;  // bf16 [N] (16-byte aligned), or nullptr
    int act = kActNone;
    uint8_t *q = nullptr;            // NVFP4 output codes [M, N/2]; nullptr = bf16 D
    uint8_t *sf = nullptr;           // blocked e4m3 scales of the output [pad128(M) * N/16]
    const float *gs = nullptr;       // device fp32 global scale of the output
    __host__ __device__ bool plain() const { return bias == nullptr && act == kActNone && q == nullptr; }
};

__device__ __forceinline__ float bf16_bits_to_float(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ float round_bf16(float y) { return __bfloat162float(__float2bfloat16_rn(y)); }

__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// act(alpha * acc + bias) for one element; `bias` is the element's bf16 bias as fp32
// (not added when the epilogue has no bias).
__device__ __forceinline__ float epi_value(float acc, float alpha, const Epi &e, float bias) {
    float y = __fmul_rn(acc, alpha);
    if (e.bias) y = __fadd_rn(y, bias);
    if (e.act == kActRelu) {
        y = fmaxf(y, 0.0f);
    } else if (e.act == kActSilu) {
        // y * sigmoid(y) = y / (1 + exp(-y))
        y = __fdividef(y, 1.0f + __expf(-y));
    } else if (e.act == kActGeluTanh) {
        // 0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3)))
        const float u = 0.7978845608028654f * (y + 0.044715f * (y * y * y));
        y = (0.5f * y) * (1.0f + tanh_approx(u));
    }
    return y;
}

}  // namespace nvfp4
