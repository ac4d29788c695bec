// quant_common.cuh — the NVFP4 block-quantization arithmetic, shared by the
// standalone quantizer (quantize.cu) and the GEMM epilogues that write NVFP4
// output, so both give the same bytes for the same bf16 values.
//
// Specification (the CPU oracle's nvfp4o_quantize, each fp32 step one IEEE
// round-to-nearest operation):
//   sf  = e4m3_rn_sat((amax / 6) / gs)          amax over the 16-element block
//   inv = 1 / (float(sf) * gs), 0 if that product is 0
//   q   = e2m1_rn_sat(x * inv)
// A gs outside [2^-100, FLT_MAX] is unusable: every block gets sf = 0, inv = 0.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace nvfp4 {

__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
    return static_cast<uint32_t>(__nv_cvt_float2_to_fp4x2(make_float2(lo, hi), __NV_E2M1, cudaRoundNearest));
}

__device__ __forceinline__ float e4m3_to_float(uint8_t code) {
    __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(code), __NV_E4M3);
    return __half2float(__half(h));
}

__device__ __forceinline__ bool gs_usable(float gs) { return gs >= 0x1p-100f && gs <= 0x1.fffffep127f; }

// e4m3 scale code of a block whose absolute maximum is amax.
__device__ __forceinline__ uint32_t block_scale_code(float amax, float gs, bool gs_ok) {
    if (!gs_ok) return 0;
    const float sfv = __fdiv_rn(__fdiv_rn(amax, 6.0f), gs);
    return static_cast<uint32_t>(__nv_cvt_float_to_fp8(sfv, __NV_SATFINITE, __NV_E4M3));
}

// 1 / (float(sf) * gs) for scale code `code` (0 when the product is 0 or gs unusable).
__device__ __forceinline__ float block_inverse(uint32_t code, float gs, bool gs_ok) {
    const float denom = __fmul_rn(e4m3_to_float((uint8_t)code), gs);
    return (!gs_ok || denom == 0.0f) ? 0.0f : __fdiv_rn(1.0f, denom);
}

// Codes of 16 values given the block's reciprocal: element 2i in the low nibble;
// bytes 0-3 in lo, 4-7 in hi.
__device__ __forceinline__ void block_codes(const float (&v)[16], float inv, uint32_t &lo, uint32_t &hi) {
    lo = 0;
    hi = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        lo |= e2m1x2(__fmul_rn(v[2 * i], inv), __fmul_rn(v[2 * i + 1], inv)) << (8 * i);
        hi |= e2m1x2(__fmul_rn(v[8 + 2 * i], inv), __fmul_rn(v[8 + 2 * i + 1], inv)) << (8 * i);
    }
}

// Scale codes without divisions, for kernels that quantize many blocks with one
// global scale gs.  The code is a non-decreasing step function of the block's
// amax (each step of block_scale_code is monotone), and amax is a bf16 value, so
//   thr[c] = the smallest non-negative bf16 amax whose code is >= c   (c = 1..126)
// determines it exactly: code = max{c : amax >= thr[c]}.  thr[0] = 0; thr[c] is NaN
// where no amax reaches c (every comparison with it is false), thr[127] likewise.
// inv[c] = block_inverse(c).  A first guess amax * (1 / (6 gs)) rounded to e4m3 is
// within one code of the exact one (its relative error is a few fp32 ulps, an e4m3
// step 2^-3; where it underflows the exact code is 0 too), so two table comparisons
// correct it.
struct ScaleTables {
    float thr[128];
    float inv[128];
};

// thr[c] for 1 <= c <= 126 and a usable gs, as bf16 bits: the smallest bf16 pattern
// in [0, +inf] whose code is >= c (code(+inf) = 126, saturated).  Starts from the
// amax whose quotient is the midpoint between the e4m3 values of codes c-1 and c and
// steps one bf16 value at a time (a few steps); a binary search over all patterns
// if that has not settled after 64 steps.
__device__ __forceinline__ uint32_t scale_threshold_bits(uint32_t c, float gs) {
    auto reaches = [&](uint32_t bits) { return block_scale_code(__uint_as_float(bits << 16), gs, true) >= c; };
    const float mid = 0.5f * (e4m3_to_float((uint8_t)(c - 1)) + e4m3_to_float((uint8_t)c));
    const float x = mid * 6.0f * gs;  // >= 0, possibly +inf
    uint32_t b = x >= __uint_as_float(0x7F800000u) ? 0x7F80u : (__float_as_uint(x) >> 16);
    int steps = 0;
    if (reaches(b)) {
        while (b > 0 && steps < 64 && reaches(b - 1)) b--, steps++;
    } else {
        while (steps < 64 && !reaches(b)) b++, steps++;  // stops at 0x7F80 at the latest
    }
    if (steps < 64) return b;
    uint32_t lo = 0, hi = 0x7F80u;
    while (lo < hi) {
        const uint32_t m = (lo + hi) >> 1;
        if (reaches(m)) hi = m;
        else lo = m + 1;
    }
    return lo;
}

// Fill the tables for gs; thread `tid` of `nthreads` (>= 1) threads, followed by a
// barrier of the caller's before any use.
__device__ __forceinline__ void build_scale_tables(ScaleTables *t, float gs, int tid, int nthreads) {
    const bool ok = gs_usable(gs);
    for (int i = tid; i < 256; i += nthreads) {
        const int c = i & 127;
        if (i < 128) {
            float thr;
            if (c == 0) thr = 0.0f;
            else if (!ok || c == 127) thr = __uint_as_float(0x7FC00000u);
            else thr = __uint_as_float(scale_threshold_bits((uint32_t)c, gs) << 16);
            t->thr[c] = thr;
        } else {
            t->inv[c] = block_inverse((uint32_t)c, gs, ok);
        }
    }
}

// 1 / (6 gs) for the first guess as k * s with gs = m * 2^e (m in [0.5, 1)):
// k = 1 / (6 m), s = 2^-e, exact for every usable gs (e in [-99, 128]), so the guess
// neither overflows (6 gs can) nor loses precision in a subnormal factor.  k = 0
// when gs is unusable.
struct ScaleGuess {
    float k, s;
};
__device__ __forceinline__ ScaleGuess scale_guess_factor(float gs) {
    ScaleGuess g{0.0f, 1.0f};
    if (gs_usable(gs)) {
        int e;
        const float m = frexpf(gs, &e);
        g.k = 1.0f / (6.0f * m);
        g.s = ldexpf(1.0f, -e);
    }
    return g;
}

// block_scale_code(amax, gs, gs_ok) from the tables (amax >= 0, not NaN).
__device__ __forceinline__ uint32_t table_scale_code(float amax, ScaleGuess guess, const ScaleTables *t,
                                                     bool gs_ok) {
    const float approx = (amax * guess.k) * guess.s;
    uint32_t c = static_cast<uint32_t>(__nv_cvt_float_to_fp8(approx, __NV_SATFINITE, __NV_E4M3));
    c = c > 126u ? 126u : c;  // an inf * 0 guess (unusable gs) converts to the NaN code
    const float below = t->thr[c], above = t->thr[c + 1];
    c = amax < below ? c - 1 : (amax >= above ? c + 1 : c);
    return gs_ok ? c : 0u;
}

// Byte offset of the scale of (row r, 64-element k-group kg) in the blocked layout
// of a [pad128(rows), K/16] scale tensor with rest_k = K / 64; the k-group's four
// scales are the four bytes from there.
__device__ __forceinline__ int64_t sf_group_offset(int64_t r, int64_t kg, int64_t rest_k) {
    return ((r >> 7) * rest_k + kg) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4;
}

}  // namespace nvfp4
