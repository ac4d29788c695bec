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
    // [11] at the last accumulator commit
    unsigned long long *trace;
    int group_m;  // pair kernel: 256-row tile rows per raster group
    int clc;      // pair kernel: tiles handed out by cluster launch control (else static persistent)
    int tma_store;  // pair kernel: plain D stored through shared memory by TMA (else direct stores)
    int spin;       // pair kernel: MMA thread and epilogue poll their barriers (test_wait)
    Epi epi;      // fused epilogue (plain: alpha and bf16/fp16 rounding only)
    Grouped grouped;
};
constexpr int kTraceSlots = 12;

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
template <int kCols, bool F16>
__device__ __forceinline__ void store_row(const uint32_t (&acc)[kCols], const Params &p, int row, int col0,
                                          int row_end, float alpha) {
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
                st_global_v8(drow + c * 32, v);
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
