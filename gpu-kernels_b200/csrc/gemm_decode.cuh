// gemm_decode.cuh — the stream-K, swap-AB decode kernel and its launch templates.
//
// For M <= 128, D = alpha * A . B^T is HBM-bound: the weight B (N x K/2 bytes plus
// scales) is read once and dominates the traffic.  The reference cannot run these
// shapes at all (M < 128 gives zero tiles, matmul/sm100_nvfp4/nvfp4_v5.cu:163-176).
//
// Design:
//   * swap-AB: the MMA computes D^T tiles = B_tile[128 x K] . A[MPAD x K]^T with
//     tcgen05 kind::mxf4nvf4 (M = 128 weight rows, N = MPAD activation rows, MPAD in
//     {8,16,32,64,128}); weights stream from HBM (evict-first), the small activation
//     matrix stays L2-resident (evict-last);
//   * hybrid data-parallel + stream-K: with n_tiles >= grid, each CTA owns
//     floor(n_tiles / grid) whole tiles and the k-blocks of the remaining tiles are cut
//     into one contiguous range per CTA (grid = #SMs), so every SM streams the same
//     number of bytes; a CTA works through its cut tiles first and its whole tiles
//     last, so the cross-CTA reductions happen while the other CTAs still stream and
//     every CTA ends on a plain store;
//   * a tile whose k-range is split across CTAs is finished by the last contributor,
//     which adds the fp32 partials in CTA order (deterministic) — partials and
//     per-tile arrival counters live in a caller-provided workspace that the kernel
//     leaves zeroed again;
//   * deep TMA ring (up to 10 stages) to keep enough bytes in flight per SM;
//   * bounded waits as in gemm.cu.
#pragma once
#include <cuda_bf16.h>

#include <cstdlib>
#include <mutex>

#include "gemm_common.cuh"
#include "grouped.cuh"

namespace nvfp4 {
namespace decode {

constexpr int kTileN = 128;          // weight rows per tile (MMA M)
constexpr int kBlockKBytes = 128;    // 256 fp4 per stage row
constexpr int kKGroups = 4;
constexpr int kThreads = 32 * 6;     // producer, MMA, 4 epilogue warps
constexpr int kSmemBudget = 225 * 1024;
// Grouped form: activation rows are loaded in boxes of 16 (two 1 KB swizzle atoms;
// MPAD rows when MPAD is 8), only as many as the tile's group has rows.
constexpr int kXBoxRows = 16;

// Arrival counters of the cut tiles: a fixed region at the start of every decode
// workspace whatever the call's shape, with the fp32 partials after it.  A workspace
// is reused by calls of different shapes (nvfp4_gemm keeps one per stream), and the
// kernel leaves only its own counters zeroed: were the counters' place to depend on
// N, one call's partials would land where a later call with more tiles keeps its
// counters.  At most kCounterSlots tiles (x groups) per call.
constexpr int kCounterSlots = 65536;
constexpr size_t kCounterBytes = (size_t)kCounterSlots * sizeof(int);  // 256 KB

// Two CTAs per SM (COLOC): 228 KB of shared memory per SM, 1 KB of it reserved per CTA.
constexpr int kColocSmemMax = (233472 - 2 * 1024) / 2;

// GROUPED: the mixture-of-experts form (active experts' weight tiles only); its
// group tables take 4 KB of shared memory from the ring's budget.
// COLOC: a ring of half the size, so that two CTAs fit on an SM: the CTAs of the next
// call in the stream (a programmatic dependent) become resident while this call's
// CTAs still stream, and prefetch their first weight tiles into L2 before they wait.
template <int MPAD, bool GROUPED = false, bool COLOC = false>
struct Layout {
    static constexpr int kW = kTileN * kBlockKBytes;     // 16 KB
    static constexpr int kX = MPAD * kBlockKBytes;       // 1..16 KB
    static constexpr int kSfw = kKGroups * 512;          // 2 KB
    static constexpr int kSfx = kKGroups * 512;          // 2 KB (one 128-row scale block)
    static constexpr int kStage = kW + kX + kSfw + kSfx;
    static constexpr int kGroupBytes = GROUPED ? 4 * (gemm::kMaxGroups + 1) * 4 : 0;
    static constexpr int kBudget = COLOC ? kColocSmemMax - 1024 : kSmemBudget;
    static constexpr int STAGES = (kBudget - 2048 - kGroupBytes) / kStage > 10 ? 10
                                                                               : (kBudget - 2048 - kGroupBytes) / kStage;
    static constexpr int kOffW = 0;
    static constexpr int kOffX = kOffW + STAGES * kW;
    static constexpr int kOffSfw = kOffX + STAGES * kX;
    static constexpr int kOffSfx = kOffSfw + STAGES * kSfw;
    static constexpr int kOffBar = kOffSfx + STAGES * kSfx;
    static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 32;  // full, empty, acc_full x2, acc_empty x2, drain
    static constexpr int kOffGroups = (kOffBar + kBarBytes + 15) / 16 * 16;
    // the NVFP4 output's scale-code tables (quant_common.cuh), built by the epilogue warps
    static constexpr int kOffTable = kOffGroups + kGroupBytes;
    static constexpr int kDynamicSmem = kOffTable + (int)sizeof(ScaleTables) + 1024;
    static constexpr int kSfColsPerStage = kKGroups * 8;  // SFw 4 + SFx 4 per k-group
    // TMEM: two accumulators of MPAD columns (the MMAs of the next tile segment run
    // while the epilogue drains this one), then two sets of scale columns
    static constexpr int kSfBase = 2 * MPAD;
    static constexpr int kTmemNeed = 2 * MPAD + 2 * kSfColsPerStage;
    static constexpr int kTmemCols = kTmemNeed <= 128 ? 128 : (kTmemNeed <= 256 ? 256 : 512);
    static_assert(MPAD % 8 == 0 && MPAD <= 128, "MPAD");
    static_assert(kTmemNeed <= kTmemCols, "tensor memory budget");
    static_assert(kDynamicSmem <= (COLOC ? kColocSmemMax : 232448), "shared memory budget");
    static_assert(!COLOC || 2 * kTmemCols <= 512, "two CTAs' tensor memory on one SM");
    static_assert(STAGES >= 2, "ring depth");
};

struct Params {
    const uint8_t *sfa;  // activations' scales (blocked, pad128(M) rows)
    const uint8_t *sfb;  // weights' scales
    uint16_t *d;         // [M, N] bf16
    float *partials;     // [grid][2][MPAD][128] fp32
    int *counters;       // [n_tiles] of the workspace's fixed counter region, zero between calls
    int M, N, K;
    float alpha;
    int n_tiles, num_kb, k_groups;
    int64_t total_iters;
    int sk_tiles;         // tiles [0, sk_tiles) are cut across CTAs (stream-K)
    int64_t sk_iters;     // their k-blocks: sk_tiles * num_kb
    int dp_per_cta;       // whole tiles per CTA: tiles sk_tiles + c * dp_per_cta + j
    int rotate;           // process a cut last tile of the stream-K range first
    int grid;
    int prefetch;  // weight tiles prefetched into L2 before the dependency wait
    KernelCtl ctl;
    Epi epi;  // fused epilogue (plain: alpha and bf16 rounding only)
    // grouped (mixture-of-experts) form: B stacked [groups * N, K/2], A's rows grouped
    // by m_offsets, A's scales in the per-group layout (grouped.cuh)
    const int *m_offsets;
    const float *alphas;
    int groups;     // 0: not grouped
    int m_total;
    // Optional per-CTA %globaltimer stamps (nullptr = off), kDecodeTraceSlots u64 per
    // CTA: [0] entry [1] dependency wait released [2] first slot full (MMA thread)
    // [3] last slot full [4] epilogue done [5] iterations; of the CTA's last segment:
    // [6] accumulator in registers [7] arrival counted (cut tiles) [8] partials summed
    // (the tile's last contributor)
    unsigned long long *trace;
};
constexpr int kDecodeTraceSlots = 9;

// The tile schedule: host-computed for one weight matrix, computed on the device from
// the active groups in the grouped form (tiles = active experts x weight tiles).
struct Sched {
    int n_tiles;
    int64_t total_iters;
    int sk_tiles;
    int64_t sk_iters;
    int dp_per_cta;
    int grid;
};

__device__ __forceinline__ Sched make_sched(int n_tiles, int num_kb, int grid) {
    Sched s;
    s.n_tiles = n_tiles;
    s.total_iters = (int64_t)n_tiles * num_kb;
    s.grid = grid;
    s.dp_per_cta = grid > 0 ? n_tiles / grid : 0;
    s.sk_tiles = n_tiles - s.dp_per_cta * grid;
    s.sk_iters = (int64_t)s.sk_tiles * num_kb;
    return s;
}

// Stream-K range of CTA c over the cut tiles' k-blocks: [range_begin(c), range_begin(c+1)).
__device__ __forceinline__ int64_t range_begin(int64_t c, const Sched &q) { return c * q.sk_iters / q.grid; }

// CTA whose range holds iteration `it` (ranges are [begin(c), begin(c+1))).
__device__ __forceinline__ int owner_of(int64_t it, const Sched &q) {
    return (int)(((it + 1) * q.grid - 1) / q.sk_iters);
}

// Fused epilogue of one output column n (this thread's weight row) over the tile's
// activation rows m < rows, compiled per activation and bias.  bf16 output:
template <int MPAD, int ACT, bool BIAS>
__device__ __forceinline__ void store_col_act(const float (&sum)[MPAD], uint16_t *d, int N, int n, int rows,
                                              int d_row0, float alpha, float bias_n) {
    if (n >= N) return;
#pragma unroll
    for (int m = 0; m < MPAD; m++)
        if (m < rows) {
            __nv_bfloat16 v = __float2bfloat16_rn(epi_t<ACT, BIAS>(sum[m], alpha, bias_n));
            d[(int64_t)(d_row0 + m) * N + n] = *reinterpret_cast<uint16_t *>(&v);
        }
}

// NVFP4 output: a 16-element scale block of row m is 16 consecutive n, i.e. 16 lanes
// of the warp (N % 64 == 0, so a block is all in or all out of range); its amax by
// shuffles, its scale code from the per-CTA tables (no division).  Rows go in chunks
// of 8 computed unconditionally (only the stores check m < rows), so the shuffle
// chains of 8 rows overlap; `rows` is uniform over the warp, so every lane takes part
// in every shuffle.
template <int MPAD, int ACT, bool BIAS>
__device__ __forceinline__ void store_col_act_nvfp4(const float (&sum)[MPAD], const Epi &e, int N, int n, int lane,
                                                    int rows, int d_row0, int sf_row0, float alpha, float bias_n,
                                                    const ScaleTables *tab, ScaleGuess guess, bool gs_ok) {
    constexpr int kChunk = MPAD < 8 ? MPAD : 8;
    const bool valid = n < N;
    const int64_t rest = N >> 6;
#pragma unroll
    for (int m0 = 0; m0 < MPAD; m0 += kChunk) {
        if (m0 >= rows) break;
        float v[kChunk], amax[kChunk];
#pragma unroll
        for (int i = 0; i < kChunk; i++) {
            v[i] = valid ? round_bf16(epi_t<ACT, BIAS>(sum[m0 + i], alpha, bias_n)) : 0.0f;
            amax[i] = fabsf(v[i]);
        }
#pragma unroll
        for (int o = 8; o; o >>= 1)
#pragma unroll
            for (int i = 0; i < kChunk; i++) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], o));
#pragma unroll
        for (int i = 0; i < kChunk; i++) {
            const int m = m0 + i;
            const uint32_t code = table_scale_code(amax[i], guess, tab, gs_ok);
            const uint32_t q4 = e2m1x2(__fmul_rn(v[i], tab->inv[code]), 0.0f) & 0xFu;
            const uint32_t hi = __shfl_down_sync(0xffffffffu, q4, 1);
            if (m < rows && valid && !(lane & 1))
                e.q[(int64_t)(d_row0 + m) * (N >> 1) + (n >> 1)] = (uint8_t)(q4 | (hi << 4));
            if (m < rows && valid && !(lane & 15))
                e.sf[sf_group_offset(sf_row0 + m, n >> 6, rest) + ((n >> 4) & 3)] = (uint8_t)code;
        }
    }
}

// SwiGLU: a warp's 32 weight rows are one block of 16 gate rows (lanes 0-15) and the
// 16 matching up rows (lanes 16-31); lane l < 16 writes output column
// 16 * (n / 32) + l of the [M, N/2] output = silu(gate) * up, the up value shuffled
// down from lane l + 16 (N % 128 == 0, so a warp is all in or all out of range).
template <int MPAD, bool BIAS>
__device__ __forceinline__ void store_col_swiglu(const float (&sum)[MPAD], uint16_t *d, int N, int n, int lane,
                                                 int rows, int d_row0, float alpha, float bias_n) {
    const int No = N >> 1, o = (n >> 5) * 16 + (lane & 15);
    const bool valid = n < N && lane < 16;
#pragma unroll
    for (int m = 0; m < MPAD; m++) {
        if (m < rows) {  // uniform over the warp
            const float y = epi_t<kActNone, BIAS>(sum[m], alpha, bias_n);
            const float up = __shfl_down_sync(0xffffffffu, y, 16);
            if (valid) {
                __nv_bfloat16 v = __float2bfloat16_rn(swiglu(y, up));
                d[(int64_t)(d_row0 + m) * No + o] = *reinterpret_cast<uint16_t *>(&v);
            }
        }
    }
}

// SwiGLU with NVFP4 output: lanes 0-15 hold one 16-column scale block of the output
// row (amax shuffles stay within each half-warp), rows in chunks of 8 as in
// store_col_act_nvfp4.
template <int MPAD, bool BIAS>
__device__ __forceinline__ void store_col_swiglu_nvfp4(const float (&sum)[MPAD], const Epi &e, int N, int n, int lane,
                                                       int rows, int d_row0, int sf_row0, float alpha, float bias_n,
                                                       const ScaleTables *tab, ScaleGuess guess, bool gs_ok) {
    constexpr int kChunk = MPAD < 8 ? MPAD : 8;
    const int No = N >> 1, o = (n >> 5) * 16 + (lane & 15);
    const bool valid = n < N && lane < 16;
    const int64_t rest = No >> 6;
#pragma unroll
    for (int m0 = 0; m0 < MPAD; m0 += kChunk) {
        if (m0 >= rows) break;
        float v[kChunk], amax[kChunk];
#pragma unroll
        for (int i = 0; i < kChunk; i++) {
            const float y = epi_t<kActNone, BIAS>(sum[m0 + i], alpha, bias_n);
            const float up = __shfl_down_sync(0xffffffffu, y, 16);
            v[i] = valid ? round_bf16(swiglu(y, up)) : 0.0f;
            amax[i] = fabsf(v[i]);
        }
#pragma unroll
        for (int s = 8; s; s >>= 1)
#pragma unroll
            for (int i = 0; i < kChunk; i++) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], s));
#pragma unroll
        for (int i = 0; i < kChunk; i++) {
            const int m = m0 + i;
            const uint32_t code = table_scale_code(amax[i], guess, tab, gs_ok);
            const uint32_t q4 = e2m1x2(__fmul_rn(v[i], tab->inv[code]), 0.0f) & 0xFu;
            const uint32_t hi = __shfl_down_sync(0xffffffffu, q4, 1);
            if (m < rows && valid && !(lane & 1))
                e.q[(int64_t)(d_row0 + m) * (No >> 1) + (o >> 1)] = (uint8_t)(q4 | (hi << 4));
            if (m < rows && valid && lane == 0)
                e.sf[sf_group_offset(sf_row0 + m, o >> 6, rest) + ((o >> 4) & 3)] = (uint8_t)code;
        }
    }
}

template <int MPAD>
__device__ __forceinline__ void store_col_epi(const float (&sum)[MPAD], const Epi &e, uint16_t *d, int N, int n,
                                              int lane, int rows, int d_row0, int sf_row0, float alpha, float bias_n,
                                              const ScaleTables *tab, ScaleGuess guess, bool gs_ok) {
    const bool bias = e.bias != nullptr;
#define NVFP4_DECODE_EPI_BODY(A)                                                                                 \
    if (e.q) {                                                                                                   \
        if (bias)                                                                                                \
            store_col_act_nvfp4<MPAD, A, true>(sum, e, N, n, lane, rows, d_row0, sf_row0, alpha, bias_n, tab,    \
                                               guess, gs_ok);                                                    \
        else                                                                                                     \
            store_col_act_nvfp4<MPAD, A, false>(sum, e, N, n, lane, rows, d_row0, sf_row0, alpha, bias_n, tab,   \
                                                guess, gs_ok);                                                   \
    } else {                                                                                                     \
        if (bias) store_col_act<MPAD, A, true>(sum, d, N, n, rows, d_row0, alpha, bias_n);                       \
        else store_col_act<MPAD, A, false>(sum, d, N, n, rows, d_row0, alpha, bias_n);                          \
    }
    switch (e.act) {
        case kActRelu: NVFP4_DECODE_EPI_BODY(kActRelu) break;
        case kActSilu: NVFP4_DECODE_EPI_BODY(kActSilu) break;
        case kActGeluTanh: NVFP4_DECODE_EPI_BODY(kActGeluTanh) break;
        case kActSwiglu:
            if (e.q) {
                if (bias)
                    store_col_swiglu_nvfp4<MPAD, true>(sum, e, N, n, lane, rows, d_row0, sf_row0, alpha, bias_n, tab,
                                                       guess, gs_ok);
                else
                    store_col_swiglu_nvfp4<MPAD, false>(sum, e, N, n, lane, rows, d_row0, sf_row0, alpha, bias_n,
                                                        tab, guess, gs_ok);
            } else {
                if (bias) store_col_swiglu<MPAD, true>(sum, d, N, n, lane, rows, d_row0, alpha, bias_n);
                else store_col_swiglu<MPAD, false>(sum, d, N, n, lane, rows, d_row0, alpha, bias_n);
            }
            break;
        default: NVFP4_DECODE_EPI_BODY(kActNone) break;
    }
#undef NVFP4_DECODE_EPI_BODY
}

template <int MPAD, bool GROUPED, bool COLOC>
__global__ void __launch_bounds__(kThreads, COLOC ? 2 : 1)
    nvfp4_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                        const Params p) {
    using L = Layout<MPAD, GROUPED, COLOC>;
    constexpr int S = L::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sW = base + L::kOffW, sX = base + L::kOffX, sSfw = base + L::kOffSfw, sSfx = base + L::kOffSfx;
    const uint32_t bar_full = base + L::kOffBar, bar_empty = bar_full + 8 * S;
    const uint32_t bar_acc_full = bar_empty + 8 * S, bar_acc_empty = bar_acc_full + 16, bar_drain = bar_acc_empty + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base_ptr + L::kOffBar + (2 * S + 5) * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_flag = reinterpret_cast<volatile int *>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long *trace = p.trace ? p.trace + blockIdx.x * kDecodeTraceSlots : nullptr;
    if (trace && threadIdx.x == 0) trace[0] = global_timer_ns();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(bar_acc_full + 8 * b, 1);
            mbar_init(bar_acc_empty + 8 * b, 4);
        }
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint64_t tmo = p.ctl.wait_timeout_ns;
    const int64_t rest_k = p.K >> 6;

    // Grouped form: the schedule depends on the row offsets, an input, so wait for the
    // preceding kernel first; then one warp tabulates each group's rows and first scale
    // block and lists the groups that have rows (only their weights are read).
    int *g_r0 = reinterpret_cast<int *>(base_ptr + L::kOffGroups);
    int *g_r1 = g_r0 + (gemm::kMaxGroups + 1);
    int *g_b0 = g_r1 + (gemm::kMaxGroups + 1);
    int *g_act = g_b0 + (gemm::kMaxGroups + 1);  // [0] = number of active groups, then their ids
    const int tiles_per_group = (p.N + kTileN - 1) / kTileN;
    Sched q;
    if constexpr (GROUPED) {
        grid_dependency_wait();
        if (warp == 0) {
            build_group_tables(p.m_offsets, p.groups, p.m_total, 0, lane, g_r0, g_r1, g_b0, nullptr);
            __syncwarp();
            int count = 0;
            for (int base0 = 0; base0 < p.groups; base0 += 32) {
                const int g = base0 + lane;
                const bool act = g < p.groups && g_r1[g] > g_r0[g];
                const uint32_t mask = __ballot_sync(0xffffffffu, act);
                if (act) g_act[1 + count + __popc(mask & ((1u << lane) - 1u))] = g;
                count += __popc(mask);
            }
            if (lane == 0) g_act[0] = count;
        }
        __syncthreads();
        q = make_sched(g_act[0] * tiles_per_group, p.num_kb, (int)gridDim.x);
    } else {
        q.n_tiles = p.n_tiles;
        q.total_iters = p.total_iters;
        q.sk_tiles = p.sk_tiles;
        q.sk_iters = p.sk_iters;
        q.dp_per_cta = p.dp_per_cta;
        q.grid = p.grid;
    }
    // Where tile T's operands and output live.
    struct DTile {
        int w_row, x_row, d_row0, rows, ncol0;
        int64_t sfw_block, sfx_block;
        float alpha;
        int group;    // the tile's group (0 when not grouped): its bias row
        int sf_row0;  // NVFP4 output: scale row of the tile's first output row
    };
    auto dtile = [&](int T) {
        DTile d;
        if constexpr (GROUPED) {
            const int g = g_act[1 + T / tiles_per_group], t = T % tiles_per_group;
            d.w_row = g * p.N + t * kTileN;
            d.sfw_block = (int64_t)g * tiles_per_group + t;
            d.x_row = g_r0[g];
            d.sfx_block = g_b0[g];
            d.d_row0 = g_r0[g];
            d.rows = g_r1[g] - g_r0[g];
            d.ncol0 = t * kTileN;
            d.alpha = p.alphas[g];
            d.group = g;
            d.sf_row0 = g_b0[g] * 128;
        } else {
            d.w_row = T * kTileN;
            d.sfw_block = T;
            d.x_row = 0;
            d.sfx_block = 0;
            d.d_row0 = 0;
            d.rows = p.M;
            d.ncol0 = T * kTileN;
            d.alpha = p.alpha;
            d.group = 0;
            d.sf_row0 = 0;
        }
        return d;
    };
    const int64_t it_begin = range_begin(blockIdx.x, q), it_end = range_begin(blockIdx.x + 1, q);
    // Processing order of this CTA's work: its stream-K range [it_begin, it_end) over
    // the cut tiles — a last tile that is cut (shared with the next CTA) first, then
    // the range from its start — and then its whole tiles.  The cut tiles are thus
    // reduced across CTAs early, and a CTA with whole tiles ends on a plain store.
    // v in [0, n_iters) is the position in that order, iter(v) the k-block.
    const int64_t sk_len = it_end - it_begin;
    const int64_t n_iters = sk_len + (int64_t)q.dp_per_cta * p.num_kb;
    const int64_t dp_first = ((int64_t)q.sk_tiles + (int64_t)blockIdx.x * q.dp_per_cta) * p.num_kb;
    const int64_t last_tile0 = sk_len ? ((it_end - 1) / p.num_kb) * p.num_kb : 0;
    const bool rotate = GROUPED ? q.dp_per_cta > 0 : p.rotate != 0;
    const int64_t head =
        (rotate && sk_len && it_end % p.num_kb != 0 && last_tile0 > it_begin) ? it_end - last_tile0 : 0;
    auto iter = [&](int64_t v) {
        return v < head ? last_tile0 + v : (v < sk_len ? it_begin + (v - head) : dp_first + (v - sk_len));
    };
    // end (exclusive, in k-blocks) of the contiguous piece that k-block `it` belongs to
    auto piece_end = [&](int64_t it) {
        if (it >= q.sk_iters) return dp_first + (int64_t)q.dp_per_cta * p.num_kb;
        return (head && it >= last_tile0) ? it_end : (head ? last_tile0 : it_end);
    };

    // Launched as a programmatic dependent of the previous kernel in the stream:
    // everything above overlapped that kernel's tail.  Warm L2 with this CTA's first
    // weight tiles (a prefetch only fills L2, which stays coherent with any write the
    // previous kernel still makes), then wait for the previous kernel before touching
    // any input or output.
    if constexpr (!GROUPED) {
        if (warp == 0 && lane == 0) {
            for (int64_t v = 0; v < n_iters && v < p.prefetch; v++) {
                const int64_t it = iter(v);
                tma_prefetch_2d(&tmap_w, (int)(it % p.num_kb) * kBlockKBytes, (int)(it / p.num_kb) * kTileN);
            }
        }
        grid_dependency_wait();
    }
    if (trace && threadIdx.x == 0) {
        trace[1] = global_timer_ns();
        trace[5] = (unsigned long long)n_iters;
    }

    if (warp == 0) {
        if (elect_one()) {
            const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
            bool ok = true;
            uint32_t issued_mask = 0, issued_parity = 0, i = 0;
            for (int64_t v = 0; v < n_iters; v++, i++) {
                const int64_t it = iter(v);
                const int s = i % S;
                const uint32_t ph = (i / S) & 1;
                if (!wait_parity(bar_empty + 8 * s, ph ^ 1, tmo, abort_flag)) {
                    report_timeout(abort_flag, p.ctl.status);
                    ok = false;
                    break;
                }
                const int tile = (int)(it / p.num_kb), kb = (int)(it % p.num_kb);
                const DTile dt = dtile(tile);
                const int kg = min(kKGroups, p.k_groups - kb * kKGroups);
                // grouped: only the group's rows of activations (16-row boxes); the MMA
                // still reads MPAD rows, and the output rows past the group that the
                // stale ones feed are never stored
                constexpr int XB = MPAD < kXBoxRows ? MPAD : kXBoxRows;  // rows per activation box
                const int x_boxes = GROUPED ? min(MPAD / XB, (dt.rows + XB - 1) / XB) : 1;
                const uint32_t x_bytes = GROUPED ? (uint32_t)(x_boxes * XB * kBlockKBytes) : (uint32_t)L::kX;
                mbar_arrive_expect_tx(bar_full + 8 * s, L::kW + x_bytes + 2u * kg * 512u);
                issued_mask |= 1u << s;
                issued_parity = (issued_parity & ~(1u << s)) | (ph << s);
                tma_load_2d_hint(sW + s * L::kW, &tmap_w, bar_full + 8 * s, kb * kBlockKBytes, dt.w_row, pol_w);
                for (int xb = 0; xb < x_boxes; xb++)
                    tma_load_2d_hint(sX + s * L::kX + xb * XB * kBlockKBytes, &tmap_x, bar_full + 8 * s,
                                     kb * kBlockKBytes, dt.x_row + xb * XB, pol_x);
                bulk_load_hint(sSfw + s * L::kSfw, p.sfb + (dt.sfw_block * rest_k + kb * kKGroups) * 512, kg * 512u,
                               bar_full + 8 * s, pol_w);
                bulk_load_hint(sSfx + s * L::kSfx, p.sfa + (dt.sfx_block * rest_k + kb * kKGroups) * 512, kg * 512u,
                               bar_full + 8 * s, pol_x);
            }
            grid_launch_dependents();  // all loads issued: the next kernel may start its prologue
            if (!ok) {
                volatile int never = 0;
                for (int s = 0; s < S; s++)
                    if (issued_mask & (1u << s))
                        wait_parity(bar_full + 8 * s, (issued_parity >> s) & 1, p.ctl.drain_timeout_ns, &never);
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_mxf4nvf4(kTileN, MPAD);
            bool ok = true, any = false;
            uint32_t i = 0;
            int seg = 0;
            for (; ok && (int64_t)i < n_iters; seg++) {  // i: k-blocks consumed so far
                int64_t it = iter(i);
                const int tile = (int)(it / p.num_kb);
                const int64_t seg_end = min(piece_end(it), (int64_t)(tile + 1) * p.num_kb);
                const uint32_t buf = (uint32_t)(seg & 1), use = (uint32_t)(seg >> 1);
                const uint32_t d_tmem = tmem_base + buf * MPAD;
                if (!wait_parity(bar_acc_empty + 8 * buf, (use & 1) ^ 1, tmo, abort_flag)) {
                    report_timeout(abort_flag, p.ctl.status);
                    ok = false;
                    break;
                }
                tc_fence_after();
                bool first = true;
                for (; it < seg_end; it++, i++) {
                    const int s = i % S;
                    if (!wait_parity(bar_full + 8 * s, (i / S) & 1, tmo, abort_flag)) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (trace && (i == 0 || (int64_t)i + 1 == n_iters)) trace[i == 0 ? 2 : 3] = global_timer_ns();
                    const int kb = (int)(it % p.num_kb);
                    const int kg = min(kKGroups, p.k_groups - kb * kKGroups);
                    const uint32_t sf_cols = tmem_base + L::kSfBase + (i & 1) * L::kSfColsPerStage;
                    for (int j = 0; j < kg; j++) {
                        const uint32_t col = sf_cols + j * 8;
                        tmem_cp_32x128_x4(col, smem_desc(sSfw + s * L::kSfw + j * 512, 16, 128, 0));
                        tmem_cp_32x128_x4(col + 4, smem_desc(sSfx + s * L::kSfx + j * 512, 16, 128, 0));
                        mma_mxf4nvf4(d_tmem, smem_desc(sW + s * L::kW + j * 32, 16, 1024, 2),
                                     smem_desc(sX + s * L::kX + j * 32, 16, 1024, 2), idesc, col, col + 4,
                                     !(first && j == 0));
                    }
                    first = false;
                    any = true;
                    mma_commit(bar_empty + 8 * s);
                }
                if (!ok) break;
                mma_commit(bar_acc_full + 8 * buf);
            }
            if (!ok && any) {
                volatile int never = 0;
                mma_commit(bar_drain);
                wait_parity(bar_drain, 0, p.ctl.drain_timeout_ns, &never);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 2..5)
        const int quarter = warp & 3;
        const int nl = quarter * 32 + lane;  // row of the weight tile this thread owns
        const int etid = threadIdx.x - 64;   // 0..127
        // NVFP4 output: the scale-code tables of the output's global scale (read after
        // the wait on the preceding kernel, which may have written it)
        ScaleTables *tab = reinterpret_cast<ScaleTables *>(base_ptr + L::kOffTable);
        ScaleGuess guess{0.0f, 1.0f};
        bool gs_ok = false;
        if (p.epi.q) {
            const float gs = *p.epi.gs;
            gs_ok = gs_usable(gs);
            guess = scale_guess_factor(gs);
            build_scale_tables(tab, gs, etid, 128);
            named_barrier(1, 128);
        }
        int seg = 0;
        for (int64_t v = 0; v < n_iters; seg++) {
            const int64_t it = iter(v);
            const int tile = (int)(it / p.num_kb);
            const int64_t tile_first = (int64_t)tile * p.num_kb, tile_last = tile_first + p.num_kb - 1;
            const int64_t seg_end = min(piece_end(it), tile_last + 1);
            const bool whole = (it == tile_first) && (seg_end == tile_last + 1);
            // partials slot: 0 for the tile the range starts in, 1 for the one it ends in
            const int slot = (it == it_begin) ? 0 : 1;
            const int seg_len = (int)(seg_end - it);
            v += seg_len;

            bool ok = true;
            const uint32_t buf = (uint32_t)(seg & 1), use = (uint32_t)(seg >> 1);
            if (lane == 0) ok = wait_parity(bar_acc_full + 8 * buf, use & 1, tmo, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) report_timeout(abort_flag, p.ctl.status);
                break;
            }
            tc_fence_after();
            uint32_t acc[MPAD];
            tmem_ld_cols<MPAD>(tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * MPAD, acc);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acc_empty + 8 * buf);
            const bool last_seg = v >= n_iters;  // v already counts this segment
            if (trace && etid == 0 && last_seg) trace[6] = global_timer_ns();

            const DTile dt = dtile(tile);
            const int n = dt.ncol0 + nl;
            float sum[MPAD];
            if (whole) {
#pragma unroll
                for (int m = 0; m < MPAD; m++) sum[m] = __uint_as_float(acc[m]);
            } else {
                // publish this CTA's partial, then count arrivals on the tile
                float *mine = p.partials + ((int64_t)blockIdx.x * 2 + slot) * MPAD * kTileN;
#pragma unroll
                for (int m = 0; m < MPAD; m++) __stcg(mine + m * kTileN + nl, __uint_as_float(acc[m]));
                // The barrier orders every epilogue thread's partial stores before thread
                // 0's release-acquire increment, which publishes them to the other
                // contributors and, for the last one, orders their partials before the
                // loads that follow the second barrier: one L2 round trip instead of a
                // fence per thread plus the atomic.  The counter adds k-blocks, not
                // CTAs: with fewer cut k-blocks than CTAs some ranges are empty, so the
                // CTAs between the tile's first and last owner need not all contribute.
                named_barrier(1, 128);
                if (etid == 0) {
                    const int prev = atomic_add_acq_rel_gpu(p.counters + tile, seg_len);
                    *last_flag = (prev + seg_len == p.num_kb);
                    if (trace && last_seg) trace[7] = global_timer_ns();
                }
                named_barrier(1, 128);
                if (!*last_flag) continue;
                // last contributor: add every partial (its own included, re-read from L2)
                // in CTA order, so the result does not depend on who finished last.
                // This is the tail of a call whose tiles are all cut, so: the partials
                // of kCh contributors are loaded at once (one L2 round trip per kCh, the
                // loads unconditional — clamped to the tile's last owner, whose range is
                // never empty — and the unused ones dropped), range bounds in 32-bit
                // arithmetic where they fit, and a contributor's partial slot read off
                // its range start (slot 0: the range starts inside this tile) instead of
                // a division.
                constexpr int kCh = MPAD <= 16 ? 4 : (MPAD <= 32 ? 2 : 1);
                const bool narrow = q.sk_iters <= (int64_t)(0x7fffffff / q.grid);
                auto begin_of = [&](int c) -> int64_t {
                    return narrow ? (int64_t)((uint32_t)c * (uint32_t)q.sk_iters / (uint32_t)q.grid)
                                  : range_begin(c, q);
                };
                const int c_lo = owner_of(tile_first, q), c_hi = owner_of(tile_last, q);
#pragma unroll
                for (int m = 0; m < MPAD; m++) sum[m] = 0.0f;
                int64_t cb = begin_of(c_lo);
                for (int c0 = c_lo; c0 <= c_hi; c0 += kCh) {
                    float part_v[kCh][MPAD];
                    bool has[kCh];
#pragma unroll
                    for (int j = 0; j < kCh; j++) {
                        const int c = min(c0 + j, c_hi);
                        const int64_t ce = begin_of(c + 1);
                        has[j] = c0 + j <= c_hi && ce != cb;  // an empty range leaves no partial
                        const int cslot = cb >= tile_first ? 0 : 1;
                        const float *part = p.partials + ((int64_t)c * 2 + cslot) * MPAD * kTileN;
#pragma unroll
                        for (int m = 0; m < MPAD; m++) part_v[j][m] = __ldcg(part + m * kTileN + nl);
                        cb = ce;
                    }
#pragma unroll
                    for (int j = 0; j < kCh; j++)
                        if (has[j]) {
#pragma unroll
                            for (int m = 0; m < MPAD; m++) sum[m] += part_v[j][m];
                        }
                }
                if (etid == 0) {
                    p.counters[tile] = 0;  // reusable by the next call
                    if (trace && last_seg) trace[8] = global_timer_ns();
                }
            }
            if (p.epi.plain()) {
                if (n < p.N) {
#pragma unroll
                    for (int m = 0; m < MPAD; m++)
                        if (m < dt.rows) {
                            __nv_bfloat16 v = __float2bfloat16_rn(sum[m] * dt.alpha);
                            p.d[(int64_t)(dt.d_row0 + m) * p.N + n] = *reinterpret_cast<uint16_t *>(&v);
                        }
                }
            } else {
                const float bias_n = (n < p.N && p.epi.bias)
                                         ? bf16_bits_to_float(p.epi.bias[(int64_t)dt.group * p.N + n])
                                         : 0.0f;
                store_col_epi<MPAD>(sum, p.epi, p.d, p.N, n, lane, dt.rows, dt.d_row0, dt.sf_row0, dt.alpha, bias_n,
                                    tab, guess, gs_ok);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
    if (trace && threadIdx.x == 0) trace[4] = global_timer_ns();
}

inline int mpad_for(int M) {
    int m = 8;
    while (m < M) m *= 2;
    return m;
}

// Whether a call's tiles (x groups) fit the workspace's counter region.
inline bool tiles_fit(int N, int groups = 1) {
    return (int64_t)((N + kTileN - 1) / kTileN) * groups <= kCounterSlots;
}

inline size_t workspace_bytes(int M, int N, int sm_count, int groups = 1) {
    (void)N;
    (void)groups;
    return kCounterBytes + (size_t)sm_count * 2 * mpad_for(M) * kTileN * sizeof(float);
}

// Rotation of the stream-K range (cut last tile first): on by default when the CTA
// also owns whole tiles; NVFP4_DECODE_ROTATE=0|1 forces it.
static int decode_rotate(int dp_per_cta) {
    static int forced = [] {
        const char *e = std::getenv("NVFP4_DECODE_ROTATE");
        return e ? (std::atoi(e) ? 1 : 0) : -1;
    }();
    return forced >= 0 ? forced : (dp_per_cta > 0 ? 1 : 0);
}

// Two CTAs per SM (half-size ring) for MPAD <= 32, on by default;
// NVFP4_DECODE_COLOC=0 keeps one CTA per SM with the full ring.  Measured per call
// from a CUDA graph, W1 [28672, 8192]: M=1 26.9 -> 24.8 us, M=16 27.3 -> 25.2 us;
// at MPAD=64 the half ring holds 3 slots and is slower (29.3 -> 30.5 us).
static bool decode_coloc() {
    static int on = [] {
        const char *e = std::getenv("NVFP4_DECODE_COLOC");
        return e ? (std::atoi(e) ? 1 : 0) : 1;
    }();
    return on != 0;
}

// Weight tiles each CTA prefetches into L2 before waiting on the preceding kernel, or
// NVFP4_DECODE_PREFETCH (0..32).  Two CTAs per SM: the ring depth (the CTA is resident
// while the previous call still streams; 5 tiles measured best of 0/2/3/5/10/16).  One
// CTA per SM: 2 (the CTA only starts once the previous call's CTA on that SM has left,
// and a deeper prefetch measured slower: M=64 28.6 us with 2, 29.3 with 7).
static int decode_prefetch(int stages, bool coloc) {
    static int forced = [] {
        const char *e = std::getenv("NVFP4_DECODE_PREFETCH");
        return e ? std::min(32, std::max(0, std::atoi(e))) : -1;
    }();
    return forced >= 0 ? forced : (coloc ? stages : std::min(stages, 2));
}

// CTAs per call: one per SM, or at most NVFP4_DECODE_GRID (a diagnostic of how the
// streaming rate depends on the number of SMs that stream).
static int decode_max_ctas(int sm_count) {
    static int forced = [] {
        const char *e = std::getenv("NVFP4_DECODE_GRID");
        return e ? std::atoi(e) : 0;
    }();
    return forced > 0 ? std::min(forced, sm_count) : sm_count;
}

template <int MPAD, bool GROUPED, bool COLOC>
static int launch_ring(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                       uint16_t *D, int M, int N, int K, void *ws, cudaStream_t stream, const DeviceInfo &di,
                       const Epi &epi, unsigned long long *trace, const int *m_offsets, const float *alphas,
                       int groups) {
    using L = Layout<MPAD, GROUPED, COLOC>;
    auto kern = nvfp4_decode_kernel<MPAD, GROUPED, COLOC>;
    static int configured[64] = {};
    if (!configured[di.device]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDynamicSmem) != cudaSuccess)
            return NVFP4_ERR_CUDA;
        configured[di.device] = 1;
    }
    // grouped: B is [groups * N, K/2], A is [M = m_total, K/2] with groups of rows
    const int w_rows = GROUPED ? groups * N : N;
    CUtensorMap tw, tx;
    int st = gemm::operand_map(B, w_rows, K, kTileN, kBlockKBytes, &tw);  // cached tensor maps
    // grouped: activations in 16-row boxes, as many as the tile's group has rows
    if (!st) st = gemm::operand_map(A, M, K, GROUPED ? (MPAD < kXBoxRows ? MPAD : kXBoxRows) : MPAD, kBlockKBytes, &tx);
    if (st) return st;
    Params p;
    p.sfa = SFA;
    p.sfb = SFB;
    p.d = D;
    p.M = M;
    p.N = N;
    p.K = K;
    p.alpha = alpha;
    p.n_tiles = (N + kTileN - 1) / kTileN;
    p.num_kb = (K + 255) / 256;
    p.k_groups = K / 64;
    // grouped: the tile count is only known on the device; size the grid for the most
    p.total_iters = (int64_t)p.n_tiles * (GROUPED ? groups : 1) * p.num_kb;
    p.grid = (int)std::min<int64_t>(decode_max_ctas(di.sm_count), p.total_iters);
    p.dp_per_cta = p.n_tiles / p.grid;  // whole tiles per CTA (0 when tiles are fewer than CTAs)
    p.sk_tiles = p.n_tiles - p.dp_per_cta * p.grid;
    p.sk_iters = (int64_t)p.sk_tiles * p.num_kb;
    p.rotate = decode_rotate(p.dp_per_cta);
    p.prefetch = decode_prefetch(L::STAGES, COLOC);
    p.counters = static_cast<int *>(ws);
    p.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kCounterBytes);
    p.epi = epi;
    p.trace = trace;
    p.m_offsets = m_offsets;
    p.alphas = alphas;
    p.groups = GROUPED ? groups : 0;
    p.m_total = M;
    if ((st = kernel_ctl(&p.ctl))) return st;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kDynamicSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tw, tx, p) != cudaSuccess) return NVFP4_ERR_CUDA;
    count_launch();
    return cuda_status(cudaGetLastError());
}

template <int MPAD, bool GROUPED = false>
static int launch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                  uint16_t *D, int M, int N, int K, void *ws, cudaStream_t stream, const DeviceInfo &di,
                  const Epi &epi, unsigned long long *trace = nullptr, const int *m_offsets = nullptr,
                  const float *alphas = nullptr, int groups = 0) {
    if constexpr (MPAD <= 32) {
        if (decode_coloc())
            return launch_ring<MPAD, GROUPED, true>(A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, epi, trace,
                                                    m_offsets, alphas, groups);
    }
    return launch_ring<MPAD, GROUPED, false>(A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, epi, trace,
                                             m_offsets, alphas, groups);
}

// One launch of the decode kernel for activations padded to MPAD rows; explicitly
// instantiated in decode_inst.cu, which is compiled once per MPAD so that the kernel
// variants build in parallel.
template <int MPAD, bool GROUPED>
int launch_mpad(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, uint16_t *D,
                int M, int N, int K, void *ws, cudaStream_t stream, const DeviceInfo &di, const Epi &epi,
                unsigned long long *trace, const int *m_offsets, const float *alphas, int groups);


// The decode kernel for `rows` activation rows (padded to the next MPAD), plain or
// grouped; defined in gemm_decode.cu.
int launch_for(int rows, bool grouped, const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
               float alpha, uint16_t *D, int M, int N, int K, void *ws, cudaStream_t stream, const DeviceInfo &di,
               const Epi &epi, unsigned long long *trace, const int *m_offsets, const float *alphas, int groups);

}  // namespace decode
}  // namespace nvfp4

