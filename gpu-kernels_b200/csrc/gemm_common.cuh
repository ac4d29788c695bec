// gemm_common.cuh — pieces shared by the persistent NVFP4 GEMM kernels (gemm.cu,
// gemm_pair.cu): launch parameters, the epilogue's row store, operand tensor maps.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "ptx.cuh"

namespace nvfp4 {
namespace gemm {

constexpr int kBlockM = 128;
constexpr int kBlockKBytes = 128;               // one 128-byte swizzle row = 256 fp4
constexpr int kKGroups = 4;                     // 64-element MMA k-steps per 128-byte stage
constexpr int kEpiWarps = 8;
constexpr int kGroupM = 16;                     // m-tiles per raster group (single-CTA kernel)
constexpr int kMaxGroups = 256;                 // experts of a grouped (MoE) GEMM

// Grouped GEMM (pair kernel): group g covers rows [m_offsets[g], m_offsets[g+1]) of
// A and D and uses weight rows [g*N, (g+1)*N) of B; its A scales start at 128-row
// block sum_{h<g} ceil(M_h / 128) of SFA.  Device arrays.
struct Grouped {
    const int *m_offsets = nullptr;  // [groups + 1]
    const float *alphas = nullptr;   // [groups]
    int groups = 0;                  // 0: not grouped
    int m_total = 0;                 // rows of A / D (offsets are clamped to it)
};

// Column-parallel GEMM with the all-gather fused into the epilogue: this rank's
// [M, N] output shard is written straight into the full [M, ld] output of every rank
// at column col_off — through NVLink stores to each rank's buffer, or one multimem
// store to an NVLink multicast address that the switch delivers to all of them.
constexpr int kMaxGatherRanks = 8;
struct Gather {
    uint64_t dst[kMaxGatherRanks] = {};  // full-D base of each rank, or dst[0] = the multicast address
    int n_dst = 0;                       // 0: no gather
    int multicast = 0;
    int64_t ld = 0;                      // row pitch of the full D in elements
    int col_off = 0;                     // this rank's first column in the full D
};

struct Params {
    const uint8_t *sfa;
    const uint8_t *sfb;
    void *d;
    int M, N, K;
    float alpha;
    int num_m_tiles, num_n_tiles, num_tiles;
    int num_kb;       // ceil(K / 256)
    int k_groups;     // K / 64
    int vec32_store;  // D 32-byte aligned and N % 16 == 0
    KernelCtl ctl;
    // Optional per-CTA cycle trace (nullptr = off), kTraceSlots u64 per CTA:
    // [0] MMA wait on full  [1] MMA wait on acc_empty  [2] producer wait on empty
    // [3] epilogue wait on acc_full  [4] epilogue drain+store  [5] tiles
    // [6] MMA-thread cycles from first issue to last commit  [7] the same span in ns
    // [8] %globaltimer at CTA entry  [9] at CTA exit  [10] at the first MMA issue
    // [11] at the last accumulator commit; hand-off sample (%globaltimer ns): [12] the
    // MMA thread seeing tile 3's first slot landed, [13] its return from the
    // accumulator wait of tile 3, [14] epilogue warp 2 woken by tile 2's accumulator, [15] the last
    // epilogue warp of the CTA with tile 2 read out of tensor memory
    unsigned long long *trace;
    int group_m;  // pair kernel: 256-row tile rows per raster group
    int clc;      // pair kernel: tiles handed out by cluster launch control (else static persistent)
    int tma_store;  // pair kernel: plain D stored through shared memory by TMA (else direct stores)
    int spin;       // pair kernel: MMA thread and epilogue poll their barriers (test_wait)
    int l2hint;     // pair kernel: 1 = D stored evict-first in L2, 2 = also A/B loaded evict-last
    Epi epi;      // fused epilogue (plain: alpha and bf16/fp16 rounding only)
    Grouped grouped;
    Gather gather;
};
constexpr int kTraceSlots = 16;

__device__ __forceinline__ uint32_t pack2(float a, float b, bool f16) {
    if (f16) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Convert this thread's kCols accumulator columns (one output row) with alpha and
// store them to D[row, col0 .. col0+kCols), clipped to N; rows >= row_end are skipped.
// With store_hint, the 32-byte stores carry the L2 policy `policy`.
template <int kCols, bool F16>
__device__ __forceinline__ void store_row(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                          int row_end, float alpha, bool store_hint = false, uint64_t policy = 0) {
    if (row >= row_end) return;
    uint8_t *drow = static_cast<uint8_t *>(p.d) + ((int64_t)row * p.N + col0) * 2;
    if (p.vec32_store) {
#pragma unroll
        for (int c = 0; c < kCols / 16; c++) {
            if (col0 + c * 16 < p.N) {
                uint32_t v[8];
#pragma unroll
                for (int i = 0; i < 8; i++)
                    v[i] = pack2(__uint_as_float(acc[c * 16 + 2 * i]) * alpha,
                                 __uint_as_float(acc[c * 16 + 2 * i + 1]) * alpha, F16);
                if (store_hint) st_global_v8_hint(drow + c * 32, v, policy);
                else st_global_v8(drow + c * 32, v);
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < kCols / 8; c++) {
            if (col0 + c * 8 < p.N) {
                uint4 v;
                v.x = pack2(__uint_as_float(acc[c * 8 + 0]) * alpha, __uint_as_float(acc[c * 8 + 1]) * alpha, F16);
                v.y = pack2(__uint_as_float(acc[c * 8 + 2]) * alpha, __uint_as_float(acc[c * 8 + 3]) * alpha, F16);
                v.z = pack2(__uint_as_float(acc[c * 8 + 4]) * alpha, __uint_as_float(acc[c * 8 + 5]) * alpha, F16);
                v.w = pack2(__uint_as_float(acc[c * 8 + 6]) * alpha, __uint_as_float(acc[c * 8 + 7]) * alpha, F16);
                *reinterpret_cast<uint4 *>(drow + c * 16) = v;
            }
        }
    }
}

// The fused-epilogue form of store_row (bf16 or NVFP4 output, see epilogue.cuh).
// Called by all 32 lanes of a warp, each with its own row and the same col0: the
// tile's bias columns col0 .. col0+127 arrive as 4 bf16 per lane (bias_raw, lane l
// holding columns col0 + 4l .. +3) and are broadcast with shuffles, so every lane
// takes part whether or not its row is stored.  NVFP4 output needs col0 and N to be
// multiples of 64: each 64-column k-group of the row is then whole, its 32 bytes of
// codes leave as one 32-byte store and its 4 scale bytes as one 32-bit store.  Rows
// >= row_end are not stored (the caller zeroes the scale padding rows).
template <int kCols>
__device__ __forceinline__ void store_row_epi(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                              int row_end, float alpha, uint2 bias_raw) {
    static_assert(kCols <= 128, "bias is broadcast from 4 columns per lane");
    const Epi &e = p.epi;
    const bool row_ok = row < row_end;
    // bias of columns col0 + k, col0 + k + 1 (k even)
    auto bias2 = [&](int k, float &b0, float &b1) {
        const uint32_t w = __shfl_sync(0xffffffffu, ((k >> 1) & 1) ? bias_raw.y : bias_raw.x, k >> 2);
        b0 = __uint_as_float(w << 16);
        b1 = __uint_as_float(w & 0xFFFF0000u);
    };
    if (!e.q) {
        uint8_t *drow = static_cast<uint8_t *>(p.d) + ((int64_t)row * p.N + col0) * 2;
#pragma unroll
        for (int c = 0; c < kCols / 16; c++) {
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int k = c * 16 + 2 * i;
                float b0, b1;
                bias2(k, b0, b1);
                w[i] = pack2(epi_value(__uint_as_float(acc[k]), alpha, e, b0),
                             epi_value(__uint_as_float(acc[k + 1]), alpha, e, b1), false);
            }
            if (row_ok) {
                if (p.vec32_store) {
                    if (col0 + c * 16 < p.N) st_global_v8(drow + c * 32, w);
                } else {
                    if (col0 + c * 16 < p.N)
                        *reinterpret_cast<uint4 *>(drow + c * 32) = make_uint4(w[0], w[1], w[2], w[3]);
                    if (col0 + c * 16 + 8 < p.N)
                        *reinterpret_cast<uint4 *>(drow + c * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
        }
        return;
    }
    if constexpr (kCols % 64 == 0) {
        const float gs = *e.gs;
        const bool gs_ok = gs_usable(gs);
        const int64_t rest = p.N >> 6;
#pragma unroll
        for (int g = 0; g < kCols / 64; g++) {
            const int c0 = col0 + g * 64;
            uint32_t codes[8], scales = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                float v[16];
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const int k = g * 64 + b * 16 + i;
                    float b0, b1;
                    bias2(k, b0, b1);
                    v[i] = round_bf16(epi_value(__uint_as_float(acc[k]), alpha, e, b0));
                    v[i + 1] = round_bf16(epi_value(__uint_as_float(acc[k + 1]), alpha, e, b1));
                    amax = fmaxf(amax, fmaxf(fabsf(v[i]), fabsf(v[i + 1])));
                }
                const uint32_t code = block_scale_code(amax, gs, gs_ok);
                block_codes(v, block_inverse(code, gs, gs_ok), codes[2 * b], codes[2 * b + 1]);
                scales |= code << (8 * b);
            }
            if (row_ok && c0 < p.N) {
                st_global_v8(e.q + (int64_t)row * (p.N >> 1) + (c0 >> 1), codes);
                *reinterpret_cast<uint32_t *>(e.sf + sf_group_offset(row, c0 >> 6, rest)) = scales;
            }
        }
    }
}

// Bias of columns c .. c+7 (c % 8 == 0; N % 8 == 0, so the 16 bytes are inside the
// bias whenever c < N): the same address in every lane, one broadcast load.
__device__ __forceinline__ uint4 bias8(const uint16_t *bias, int N, int c) {
    return c < N ? __ldg(reinterpret_cast<const uint4 *>(bias + c)) : make_uint4(0u, 0u, 0u, 0u);
}

// Element j (0..7) of a bias8 vector as fp32.
__device__ __forceinline__ float bias_elem(const uint4 &b, int j) {
    const uint32_t w = (j >> 1) == 0 ? b.x : (j >> 1) == 1 ? b.y : (j >> 1) == 2 ? b.z : b.w;
    return (j & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
}

// store_row_epi with the activation and the bias fixed at compile time, bf16 output:
// straight-line code per 16-column chunk.  Lanes need not agree on anything here.
template <int kCols, int ACT, bool BIAS>
__device__ __forceinline__ void store_row_act(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                              int row_end, float alpha, const uint16_t *bias) {
    const bool row_ok = row < row_end;
    uint8_t *drow = static_cast<uint8_t *>(p.d) + ((int64_t)row * p.N + col0) * 2;
#pragma unroll
    for (int c = 0; c < kCols / 16; c++) {
        uint4 b0 = make_uint4(0u, 0u, 0u, 0u), b1 = b0;
        if constexpr (BIAS) {
            b0 = bias8(bias, p.N, col0 + c * 16);
            b1 = bias8(bias, p.N, col0 + c * 16 + 8);
        }
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint4 &b = i < 4 ? b0 : b1;
            w[i] = pack2(epi_t<ACT, BIAS>(__uint_as_float(acc[c * 16 + 2 * i]), alpha, bias_elem(b, (2 * i) & 7)),
                         epi_t<ACT, BIAS>(__uint_as_float(acc[c * 16 + 2 * i + 1]), alpha,
                                          bias_elem(b, (2 * i + 1) & 7)),
                         false);
        }
        if (row_ok) {
            if (p.vec32_store) {
                if (col0 + c * 16 < p.N) st_global_v8(drow + c * 32, w);
            } else {
                if (col0 + c * 16 < p.N)
                    *reinterpret_cast<uint4 *>(drow + c * 32) = make_uint4(w[0], w[1], w[2], w[3]);
                if (col0 + c * 16 + 8 < p.N)
                    *reinterpret_cast<uint4 *>(drow + c * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
            }
        }
    }
}

// The NVFP4-output form of store_row_act: per 16-element block the bf16-rounded
// values, their amax, the scale code from the per-CTA tables (no division) and the
// codes — the bytes store_row_epi (and nvfp4_quantize of the bf16 values) gives.
// col0 and N multiples of 64.  The row's scales go to row sf_row of the blocked
// scale tensor (the row itself, or its place in a grouped layout).
template <int kCols, int ACT, bool BIAS>
__device__ __forceinline__ void store_row_act_nvfp4(const uint32_t (&acc)[kCols], const Params &p, int row,
                                                    int col0, int row_end, float alpha, const uint16_t *bias,
                                                    int64_t sf_row, const ScaleTables *tab, ScaleGuess guess,
                                                    bool gs_ok) {
    static_assert(kCols % 64 == 0, "whole 64-column k-groups");
    const Epi &e = p.epi;
    const bool row_ok = row < row_end;
    const int64_t rest = p.N >> 6;
#pragma unroll
    for (int g = 0; g < kCols / 64; g++) {
        const int c0 = col0 + g * 64;
        uint32_t codes[8], scales = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            uint4 b0 = make_uint4(0u, 0u, 0u, 0u), b1 = b0;
            if constexpr (BIAS) {
                b0 = bias8(bias, p.N, c0 + b * 16);
                b1 = bias8(bias, p.N, c0 + b * 16 + 8);
            }
            uint32_t pk[8];
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int k = g * 64 + b * 16 + 2 * i;
                const uint4 &bb = i < 4 ? b0 : b1;
                pk[i] = pack2(epi_t<ACT, BIAS>(__uint_as_float(acc[k]), alpha, bias_elem(bb, (2 * i) & 7)),
                              epi_t<ACT, BIAS>(__uint_as_float(acc[k + 1]), alpha, bias_elem(bb, (2 * i + 1) & 7)),
                              false);
                amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(pk[i] << 16)),
                                         fabsf(__uint_as_float(pk[i] & 0xFFFF0000u))));
            }
            const uint32_t code = table_scale_code(amax, guess, tab, gs_ok);
            const float inv = tab->inv[code];
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                lo |= e2m1x2(__fmul_rn(__uint_as_float(pk[i] << 16), inv),
                             __fmul_rn(__uint_as_float(pk[i] & 0xFFFF0000u), inv)) << (8 * i);
                hi |= e2m1x2(__fmul_rn(__uint_as_float(pk[4 + i] << 16), inv),
                             __fmul_rn(__uint_as_float(pk[4 + i] & 0xFFFF0000u), inv)) << (8 * i);
            }
            codes[2 * b] = lo;
            codes[2 * b + 1] = hi;
            scales |= code << (8 * b);
        }
        if (row_ok && c0 < p.N) {
            st_global_v8(e.q + (int64_t)row * (p.N >> 1) + (c0 >> 1), codes);
            *reinterpret_cast<uint32_t *>(e.sf + sf_group_offset(sf_row, c0 >> 6, rest)) = scales;
        }
    }
}

// SwiGLU output of one row: accumulator columns [col0, col0 + kCols) (kCols % 32 == 0,
// col0 % 32 == 0) hold blocks of 16 gate then 16 up columns and become the kCols/2
// output columns from col0/2 of the [M, N/2] output: out = silu(gate) * up with
// y = alpha * acc (+ bias) for each.  Gate and up value 2i / 2i+1 of a block:
template <bool BIAS>
__device__ __forceinline__ void swiglu_block(const uint32_t *acc32, float alpha, const uint16_t *bias, int N,
                                             int c32, uint32_t (&pk)[8]) {
    uint4 bg0 = make_uint4(0u, 0u, 0u, 0u), bg1 = bg0, bu0 = bg0, bu1 = bg0;
    if constexpr (BIAS) {
        bg0 = bias8(bias, N, c32);
        bg1 = bias8(bias, N, c32 + 8);
        bu0 = bias8(bias, N, c32 + 16);
        bu1 = bias8(bias, N, c32 + 24);
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint4 &bg = i < 4 ? bg0 : bg1, &bu = i < 4 ? bu0 : bu1;
        const int j0 = (2 * i) & 7, j1 = (2 * i + 1) & 7;
        const float g0 = epi_t<kActNone, BIAS>(__uint_as_float(acc32[2 * i]), alpha, bias_elem(bg, j0));
        const float g1 = epi_t<kActNone, BIAS>(__uint_as_float(acc32[2 * i + 1]), alpha, bias_elem(bg, j1));
        const float u0 = epi_t<kActNone, BIAS>(__uint_as_float(acc32[16 + 2 * i]), alpha, bias_elem(bu, j0));
        const float u1 = epi_t<kActNone, BIAS>(__uint_as_float(acc32[16 + 2 * i + 1]), alpha, bias_elem(bu, j1));
        pk[i] = pack2(swiglu(g0, u0), swiglu(g1, u1), false);
    }
}

template <int kCols, bool BIAS>
__device__ __forceinline__ void store_row_swiglu(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                                 int row_end, float alpha, const uint16_t *bias) {
    static_assert(kCols % 32 == 0, "whole gate / up blocks");
    const int No = p.N >> 1;
    const bool row_ok = row < row_end;
    uint8_t *drow = static_cast<uint8_t *>(p.d) + ((int64_t)row * No + (col0 >> 1)) * 2;
#pragma unroll
    for (int j = 0; j < kCols / 32; j++) {
        uint32_t w[8];
        swiglu_block<BIAS>(&acc[32 * j], alpha, bias, p.N, col0 + 32 * j, w);
        if (row_ok && col0 + 32 * j < p.N) {
            if (p.vec32_store) {
                st_global_v8(drow + j * 32, w);
            } else {
                *reinterpret_cast<uint4 *>(drow + j * 32) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4 *>(drow + j * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
            }
        }
    }
}

// SwiGLU with NVFP4 output: kCols/2 output columns = whole 64-column k-groups of the
// [M, N/2] output (kCols % 128 == 0), the arithmetic of store_row_act_nvfp4.
template <int kCols, bool BIAS>
__device__ __forceinline__ void store_row_swiglu_nvfp4(const uint32_t (&acc)[kCols], const Params &p, int row,
                                                       int col0, int row_end, float alpha, const uint16_t *bias,
                                                       int64_t sf_row, const ScaleTables *tab, ScaleGuess guess,
                                                       bool gs_ok) {
    static_assert(kCols % 128 == 0, "whole 64-column output k-groups");
    const Epi &e = p.epi;
    const int No = p.N >> 1;
    const bool row_ok = row < row_end;
    const int64_t rest = No >> 6;
#pragma unroll
    for (int g = 0; g < kCols / 128; g++) {
        const int o0 = (col0 >> 1) + g * 64;  // first output column of the k-group
        uint32_t codes[8], scales = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            uint32_t pk[8];
            swiglu_block<BIAS>(&acc[g * 128 + b * 32], alpha, bias, p.N, col0 + g * 128 + b * 32, pk);
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++)
                amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(pk[i] << 16)), fabsf(__uint_as_float(pk[i] & 0xFFFF0000u))));
            const uint32_t code = table_scale_code(amax, guess, tab, gs_ok);
            const float inv = tab->inv[code];
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                lo |= e2m1x2(__fmul_rn(__uint_as_float(pk[i] << 16), inv),
                             __fmul_rn(__uint_as_float(pk[i] & 0xFFFF0000u), inv)) << (8 * i);
                hi |= e2m1x2(__fmul_rn(__uint_as_float(pk[4 + i] << 16), inv),
                             __fmul_rn(__uint_as_float(pk[4 + i] & 0xFFFF0000u), inv)) << (8 * i);
            }
            codes[2 * b] = lo;
            codes[2 * b + 1] = hi;
            scales |= code << (8 * b);
        }
        if (row_ok && o0 < No) {
            st_global_v8(e.q + (int64_t)row * (No >> 1) + (o0 >> 1), codes);
            *reinterpret_cast<uint32_t *>(e.sf + sf_group_offset(sf_row, o0 >> 6, rest)) = scales;
        }
    }
}

// The fused epilogue of one row, dispatched once per tile to the body compiled for
// this launch's activation, bias and output type.  tab / guess / gs_ok: the NVFP4
// output's scale tables (unused for bf16 output).  NVFP4 output needs kCols % 64 == 0
// (the launch rejects it otherwise).  bias: the bias row of this tile (the expert's
// in a grouped launch, nullptr for none); sf_row: the row's scale row.
template <int kCols>
__device__ __forceinline__ void store_row_epi_fast(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                                   int row_end, float alpha, const uint16_t *bias_row, int64_t sf_row,
                                                   const ScaleTables *tab, ScaleGuess guess, bool gs_ok) {
    const Epi &e = p.epi;
    const bool bias = bias_row != nullptr;
#define NVFP4_EPI_BODY(A)                                                                                         \
    if (e.q) {                                                                                                    \
        if constexpr (kCols % 64 == 0) {                                                                          \
            if (bias)                                                                                             \
                store_row_act_nvfp4<kCols, A, true>(acc, p, row, col0, row_end, alpha, bias_row, sf_row, tab,     \
                                                    guess, gs_ok);                                                \
            else                                                                                                  \
                store_row_act_nvfp4<kCols, A, false>(acc, p, row, col0, row_end, alpha, bias_row, sf_row, tab,    \
                                                     guess, gs_ok);                                               \
        }                                                                                                         \
    } else {                                                                                                      \
        if (bias) store_row_act<kCols, A, true>(acc, p, row, col0, row_end, alpha, bias_row);                     \
        else store_row_act<kCols, A, false>(acc, p, row, col0, row_end, alpha, bias_row);                         \
    }
    switch (e.act) {
        case kActRelu: NVFP4_EPI_BODY(kActRelu) break;
        case kActSilu: NVFP4_EPI_BODY(kActSilu) break;
        case kActGeluTanh: NVFP4_EPI_BODY(kActGeluTanh) break;
        case kActSwiglu:  // the launch admits it only where kCols % 128 == 0
            if constexpr (kCols % 128 == 0) {
                if (e.q) {
                    if (bias)
                        store_row_swiglu_nvfp4<kCols, true>(acc, p, row, col0, row_end, alpha, bias_row, sf_row, tab,
                                                            guess, gs_ok);
                    else
                        store_row_swiglu_nvfp4<kCols, false>(acc, p, row, col0, row_end, alpha, bias_row, sf_row,
                                                             tab, guess, gs_ok);
                } else {
                    if (bias) store_row_swiglu<kCols, true>(acc, p, row, col0, row_end, alpha, bias_row);
                    else store_row_swiglu<kCols, false>(acc, p, row, col0, row_end, alpha, bias_row);
                }
            }
            break;
        default: NVFP4_EPI_BODY(kActNone) break;
    }
#undef NVFP4_EPI_BODY
}

// The gather form of store_row (bf16 output): each 16-column chunk of this row goes
// to every destination of p.gather (32-byte stores, or two 16-byte multimem stores to
// the multicast address).  Rows >= row_end and columns >= N are not stored.
template <int kCols>
__device__ __forceinline__ void store_row_gather(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                                 int row_end, float alpha) {
    if (row >= row_end) return;
    const Gather &g = p.gather;
    const int64_t off = ((int64_t)row * g.ld + g.col_off + col0) * 2;
#pragma unroll
    for (int c = 0; c < kCols / 16; c++) {
        if (col0 + c * 16 < p.N) {
            uint32_t v[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                v[i] = pack2(__uint_as_float(acc[c * 16 + 2 * i]) * alpha,
                             __uint_as_float(acc[c * 16 + 2 * i + 1]) * alpha, false);
            if (g.multicast) {
                const uint64_t a = g.dst[0] + off + c * 32;
                multimem_st_bf16x8(a, v[0], v[1], v[2], v[3]);
                multimem_st_bf16x8(a + 16, v[4], v[5], v[6], v[7]);
            } else {
#pragma unroll
                for (int d = 0; d < kMaxGatherRanks; d++)
                    if (d < g.n_dst) st_global_v8(reinterpret_cast<void *>(g.dst[d] + off + c * 32), v);
            }
        }
    }
}

// Coalesced gather store of one warp's 32 rows x kCols columns (bf16), through the
// warp's 4 KB of shared memory `stage`: each 64-column chunk is written row by row
// (lane = row, 16-byte pieces XOR-swizzled by row so the 32 lanes hit every bank
// once per four rows), then read back four rows per instruction, eight lanes per row,
// so that every global store instruction writes four 128-byte row segments — to each
// destination, or once through the multicast address.  Rows >= row_end and columns
// >= N are not stored.  All 32 lanes call it.
template <int kCols>
__device__ __forceinline__ void store_rows_gather_staged(const uint32_t (&acc)[kCols], const Params &p, int row0,
                                                         int col0, int row_end, float alpha, uint32_t stage,
                                                         int lane) {
    static_assert(kCols % 64 == 0, "64-column chunks");
    const Gather &g = p.gather;
#pragma unroll
    for (int h = 0; h < kCols / 64; h++) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int k = h * 64 + j * 8;
            const uint32_t w0 = pack2(__uint_as_float(acc[k + 0]) * alpha, __uint_as_float(acc[k + 1]) * alpha, false);
            const uint32_t w1 = pack2(__uint_as_float(acc[k + 2]) * alpha, __uint_as_float(acc[k + 3]) * alpha, false);
            const uint32_t w2 = pack2(__uint_as_float(acc[k + 4]) * alpha, __uint_as_float(acc[k + 5]) * alpha, false);
            const uint32_t w3 = pack2(__uint_as_float(acc[k + 6]) * alpha, __uint_as_float(acc[k + 7]) * alpha, false);
            st_shared_v4(stage + (uint32_t)lane * 128u + 16u * ((uint32_t)j ^ ((uint32_t)lane & 7u)), w0, w1, w2, w3);
        }
        __syncwarp();
#pragma unroll
        for (int step = 0; step < 8; step++) {
            const int r = step * 4 + (lane >> 3), j = lane & 7;
            uint32_t v0, v1, v2, v3;
            ld_shared_v4(stage + (uint32_t)r * 128u + 16u * ((uint32_t)j ^ ((uint32_t)r & 7u)), v0, v1, v2, v3);
            const int grow = row0 + r, gcol = col0 + h * 64 + j * 8;
            if (grow < row_end && gcol < p.N) {
                const int64_t off = ((int64_t)grow * g.ld + g.col_off + gcol) * 2;
                if (g.multicast) {
                    multimem_st_bf16x8(g.dst[0] + off, v0, v1, v2, v3);
                } else {
#pragma unroll
                    for (int d = 0; d < kMaxGatherRanks; d++)
                        if (d < g.n_dst)
                            *reinterpret_cast<uint4 *>(g.dst[d] + off) = make_uint4(v0, v1, v2, v3);
                }
            }
        }
        __syncwarp();
    }
}

// This lane's 4 bias values of the columns col0 + 4 * lane .. +3 (zero without a
// bias or past N), for store_row_epi.
__device__ __forceinline__ uint2 load_bias_lane(const Epi &e, int N, int col0, int lane) {
    const int n = col0 + 4 * lane;
    if (!e.bias || n >= N) return make_uint2(0u, 0u);
    return __ldg(reinterpret_cast<const uint2 *>(e.bias + n));
}

// Encoded (and cached) 2-D tensor map over an NVFP4 operand [rows, K/2] bytes with a
// box of `box_bytes` x `box_rows` and the matching shared-memory swizzle.
int operand_map(const void *ptr, int64_t rows, int64_t K, int box_rows, int box_bytes, CUtensorMap *out);
// Encoded (and cached) store map over a 16-bit [M, N] output with boxes of 16 columns x
// box_rows rows and the 32-byte swizzle.
int output_map(const void *ptr, int64_t M, int64_t N, int box_rows, CUtensorMap *out);

}  // namespace gemm
}  // namespace nvfp4
