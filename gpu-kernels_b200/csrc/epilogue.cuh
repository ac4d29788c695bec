// epilogue.cuh — the fused GEMM epilogue shared by the persistent (single-CTA,
// CTA-pair) and decode kernels: per output element
//   y = alpha * acc                  (fp32, one IEEE multiply)
//   y = y + float(bias[n])           (bf16 bias over N, optional; one IEEE add)
//   y = act(y)                       (none, relu, silu, gelu with the tanh form)
// then either D = bf16_rn(y), or the bf16_rn(y) row segment quantized to NVFP4 with
// a given global scale (the standalone quantizer's arithmetic, quant_common.cuh),
// so a fused NVFP4 output equals nvfp4_quantize of the fused bf16 output byte for byte.
// silu and gelu use the hardware tanh.approx (relative error below 2^-10): the
// epilogue runs in the shadow of the next tile's MMAs only while it stays this cheap.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "quant_common.cuh"

namespace nvfp4 {

// kActSwiglu: silu(gate) * up over gate / up columns interleaved in blocks of 16
// (columns 32j .. 32j+15 gate, 32j+16 .. 32j+31 up); the output has half the columns.
enum : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActGeluTanh = 3, kActSwiglu = 4 };

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

// act(y) for a compile-time activation.
//   silu: y * sigmoid(y) = h + h * tanh(h) with h = y / 2 (one tanh.approx)
//   gelu: 0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3))) = h + h * tanh(u)
template <int ACT>
__device__ __forceinline__ float activate(float y) {
    if constexpr (ACT == kActRelu) {
        return fmaxf(y, 0.0f);
    } else if constexpr (ACT == kActSilu) {
        const float h = 0.5f * y;
        return fmaf(h, tanh_approx(h), h);
    } else if constexpr (ACT == kActGeluTanh) {
        const float h = 0.5f * y;
        const float u = 0.7978845608028654f * fmaf(0.044715f * y * y, y, y);
        return fmaf(h, tanh_approx(u), h);
    } else {
        return y;
    }
}

// SwiGLU of one gate / up pair (gate and up already alpha-scaled and biased):
// silu(gate) * up, silu as in activate<kActSilu>.
__device__ __forceinline__ float swiglu(float gate, float up) {
    return __fmul_rn(activate<kActSilu>(gate), up);
}

// act(alpha * acc + bias) for one element with the epilogue fixed at compile time
// (straight-line code: the per-tile epilogue of the persistent kernels).
template <int ACT, bool BIAS>
__device__ __forceinline__ float epi_t(float acc, float alpha, float bias) {
    float y = __fmul_rn(acc, alpha);
    if constexpr (BIAS) y = __fadd_rn(y, bias);
    return activate<ACT>(y);
}

// act(alpha * acc + bias) for one element; `bias` is the element's bf16 bias as fp32
// (not added when the epilogue has no bias).  Same arithmetic as epi_t.
__device__ __forceinline__ float epi_value(float acc, float alpha, const Epi &e, float bias) {
    float y = __fmul_rn(acc, alpha);
    if (e.bias) y = __fadd_rn(y, bias);
    switch (e.act) {
        case kActRelu: return activate<kActRelu>(y);
        case kActSilu: return activate<kActSilu>(y);
        case kActGeluTanh: return activate<kActGeluTanh>(y);
        default: return y;
    }
}

}  // namespace nvfp4
