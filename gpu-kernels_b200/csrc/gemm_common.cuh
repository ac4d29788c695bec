// gemm_common.cuh — pieces shared by the persistent NVFP4 GEMM kernels (gemm.cu,
// gemm_pair.cu): launch parameters, the epilogue's row store, operand tensor maps.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "ptx.cuh"

namespace nvfp4 {
namespace gemm {

constexpr int kBlockM = 128;
constexpr int kBlockKBytes = 128;               // one 128-byte swizzle row = 256 fp4
constexpr int kKGroups = 4;                     // 64-element MMA k-steps per 128-byte stage
constexpr int kEpiWarps = 8;
constexpr int kGroupM = 16;                     // m-tiles per raster group (single-CTA kernel)

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
// store them to D[row, col0 .. col0+kCols), clipped to N.
template <int kCols, bool F16>
__device__ __forceinline__ void store_row(const uint32_t (&acc)[kCols], const Params &p, int row, int col0) {
    if (row >= p.M) return;
    uint8_t *drow = static_cast<uint8_t *>(p.d) + ((int64_t)row * p.N + col0) * 2;
    if (p.vec32_store) {
#pragma unroll
        for (int c = 0; c < kCols / 16; c++) {
            if (col0 + c * 16 < p.N) {
                uint32_t v[8];
#pragma unroll
                for (int i = 0; i < 8; i++)
                    v[i] = pack2(__uint_as_float(acc[c * 16 + 2 * i]) * p.alpha,
                                 __uint_as_float(acc[c * 16 + 2 * i + 1]) * p.alpha, F16);
                st_global_v8(drow + c * 32, v);
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < kCols / 8; c++) {
            if (col0 + c * 8 < p.N) {
                uint4 v;
                v.x = pack2(__uint_as_float(acc[c * 8 + 0]) * p.alpha, __uint_as_float(acc[c * 8 + 1]) * p.alpha, F16);
                v.y = pack2(__uint_as_float(acc[c * 8 + 2]) * p.alpha, __uint_as_float(acc[c * 8 + 3]) * p.alpha, F16);
                v.z = pack2(__uint_as_float(acc[c * 8 + 4]) * p.alpha, __uint_as_float(acc[c * 8 + 5]) * p.alpha, F16);
                v.w = pack2(__uint_as_float(acc[c * 8 + 6]) * p.alpha, __uint_as_float(acc[c * 8 + 7]) * p.alpha, F16);
                *reinterpret_cast<uint4 *>(drow + c * 16) = v;
            }
        }
    }
}

// Encoded (and cached) 2-D tensor map over an NVFP4 operand [rows, K/2] bytes with a
// box of `box_bytes` x `box_rows` and the matching shared-memory swizzle.
int operand_map(const void *ptr, int64_t rows, int64_t K, int box_rows, int box_bytes, CUtensorMap *out);

}  // namespace gemm
}  // namespace nvfp4
