// grouped.cuh — row-group tables of the grouped (mixture-of-experts) kernels.
//
// A grouped operand stacks G groups of rows: group g is rows
// [m_offsets[g], m_offsets[g+1]) of a [m_total, K] matrix (m_offsets on the device,
// clamped here to [0, m_total]; an end before its start is an empty group).  Its
// block scales are laid out group by group, each group's blocked [pad128(M_g), K/16]
// tensor starting on a 128-row block: group g's first block is
// sum_{h<g} ceil(M_h / 128).  A scale buffer therefore needs room for
// ceil(m_total / 128) + G blocks of K/16 * 128 bytes.
#pragma once
#include <stdint.h>

namespace nvfp4 {

// One warp fills, in shared memory: r0[g], r1[g] (the group's rows), b0[g] (its
// first scale block, g <= G) and t0[g] (its first output tile, g <= G, counting
// ceil(M_g / 256) * tiles_per_row_block tiles per group; pass 0 to skip).
__device__ __forceinline__ void build_group_tables(const int *m_offsets, int G, int m_total, int tiles_per_row_block,
                                                   int lane, int *r0, int *r1, int *b0, int *t0) {
    int carry_t = 0, carry_b = 0;
    for (int base0 = 0; base0 < G; base0 += 32) {
        const int g = base0 + lane;
        int a = 0, z = 0;
        if (g < G) {
            a = min(max(m_offsets[g], 0), m_total);
            z = min(max(m_offsets[g + 1], a), m_total);
        }
        int tiles = (z - a + 255) / 256 * tiles_per_row_block, blocks = (z - a + 127) / 128;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, tiles, o), b = __shfl_up_sync(0xffffffffu, blocks, o);
            if (lane >= o) {
                tiles += t;
                blocks += b;
            }
        }
        if (g < G) {
            r0[g] = a;
            r1[g] = z;
            b0[g + 1] = carry_b + blocks;
            if (t0) t0[g + 1] = carry_t + tiles;
        }
        carry_t += __shfl_sync(0xffffffffu, tiles, 31);
        carry_b += __shfl_sync(0xffffffffu, blocks, 31);
    }
    if (lane == 0) {
        b0[0] = 0;
        if (t0) t0[0] = 0;
    }
}

// The last group g < G with key[g] <= x (key non-decreasing over non-empty groups).
__device__ __forceinline__ int last_group_at_or_before(const int *key, int G, int x) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (key[mid] <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}

}  // namespace nvfp4
