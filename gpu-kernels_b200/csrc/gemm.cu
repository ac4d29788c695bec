// gemm.cu — persistent, warp-specialised NVFP4 block-scaled GEMM for sm_100a.
//
//   D[M,N] = alpha * sum_k (e2m1 A[m,k] * e4m3 SFA[m,k/16]) * (e2m1 B[n,k] * e4m3 SFB[n,k/16])
//
// Same contract as the reference's best B200 kernel (_matmul_nvfp4_v5,
// matmul/sm100_nvfp4/nvfp4_v5.cu:21-231 of Parth-Badgujar/gpu-kernels): e2m1 K-major
// operands, 128x4-blocked e4m3 scales, tcgen05 kind::mxf4nvf4 MMAs with the scales
// staged through tensor memory.  What is different, and why:
//   * the accumulator is released as soon as the epilogue has pulled it into
//     registers, so the next tile's MMAs overlap the conversion and stores
//     (the reference serialises the whole epilogue against the mainloop);
//   * 8 epilogue warps (two per TMEM lane quarter) drain 256 columns in one pass;
//   * a 4-stage, 54 KB/stage ring (BLOCK_K = 256) with per-stage scale columns;
//   * any M >= 1, N % 8 == 0, K % 64 == 0: TMA zero-fills ragged tiles, the last
//     k-stage issues only the k-groups that exist, stores are bounds-checked;
//   * grouped rasterisation for L2 reuse without the reference's divisibility rule;
//   * every wait is bounded; a timed-out CTA drains its in-flight copies and MMAs,
//     frees its tensor memory and returns (status latched for the host);
//   * alpha and bf16 (or fp16) output; explicit stream; tensor maps cached.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"

namespace nvfp4 {

namespace gemm {

constexpr int kBlockM = 128;
constexpr int kBlockKBytes = 128;               // one 128-byte swizzle row = 256 fp4
constexpr int kKGroups = 4;                     // 64-element MMA k-steps per stage
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);  // producer, MMA, 8 epilogue warps
constexpr int kGroupM = 16;                     // m-tiles per raster group

template <int BN, int STAGES>
struct Layout {
    static constexpr int kSfbBlocks = BN / 128;
    static constexpr int kA = kBlockM * kBlockKBytes;        // 16 KB
    static constexpr int kB = BN * kBlockKBytes;             // 32 KB at BN=256
    static constexpr int kSfa = kKGroups * 512;              // 2 KB
    static constexpr int kSfb = kSfbBlocks * kKGroups * 512; // 4 KB at BN=256
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + STAGES * kA;
    static constexpr int kOffSfa = kOffB + STAGES * kB;
    static constexpr int kOffSfb = kOffSfa + STAGES * kSfa;
    static constexpr int kOffBar = kOffSfb + STAGES * kSfb;
    // barriers: full[S], empty[S], acc_full, acc_empty, drain; then tmem slot + abort flag
    static constexpr int kBarBytes = (2 * STAGES + 3) * 8 + 16;
    static constexpr int kBytes = kOffBar + kBarBytes;
    static constexpr int kDynamicSmem = kBytes + 1024;       // manual 1024-B alignment slack
    // tensor memory: accumulator columns [0, BN), two sets of scale columns after it
    static constexpr int kSfColsPerGroup = 4 + 4 * kSfbBlocks;
    static constexpr int kSfColsPerStage = kKGroups * kSfColsPerGroup;
    static constexpr int kTmemCols = 512;
    static_assert(BN + 2 * kSfColsPerStage <= kTmemCols, "tensor memory budget");
    static_assert(kDynamicSmem <= 232448, "shared memory budget");
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
    // [6] MMA-thread cycles from first issue to last commit  [7] unused
    unsigned long long *trace;
    int group_m;  // pair kernel: 256-row tile rows per raster group
};
constexpr int kTraceSlots = 8;

__device__ __forceinline__ void tile_coords(int t, const Params &p, int &tm, int &tn) {
    const int per_group = kGroupM * p.num_n_tiles;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(p.num_m_tiles - first_m, kGroupM);
    const int local = t - g * per_group;
    tm = first_m + local % gm;
    tn = local / gm;
}

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

template <int BN, int STAGES, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const Params p) {
    using L = Layout<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sA = base + L::kOffA, sB = base + L::kOffB, sSfa = base + L::kOffSfa, sSfb = base + L::kOffSfb;
    const uint32_t bar_full = base + L::kOffBar;
    const uint32_t bar_empty = bar_full + 8 * STAGES;
    const uint32_t bar_acc_full = bar_empty + 8 * STAGES;
    const uint32_t bar_acc_empty = bar_acc_full + 8;
    const uint32_t bar_drain = bar_acc_empty + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base_ptr + L::kOffBar + (2 * STAGES + 3) * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        mbar_init(bar_acc_full, 1);
        mbar_init(bar_acc_empty, kEpiWarps);
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
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

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one()) {
            const int64_t rest_k = p.K >> 6;  // 64-element k-groups per 128-row scale block
            const int sfb_rows_padded = ((p.N + 127) / 128) * 128;
            uint32_t it = 0;
            bool ok = true;
            uint32_t issued_mask = 0, issued_parity = 0;
            for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, p, tm, tn);
                for (int kb = 0; kb < p.num_kb; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!wait_parity(bar_empty + 8 * s, ph ^ 1, tmo, abort_flag)) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    const int kg = min(kKGroups, p.k_groups - kb * kKGroups);
                    int sfb_blocks = 0;
                    for (int rb = 0; rb < L::kSfbBlocks; rb++)
                        if (tn * BN + rb * 128 < sfb_rows_padded) sfb_blocks++;
                    const uint32_t bytes = L::kA + L::kB + (uint32_t)kg * 512u * (1u + sfb_blocks);
                    mbar_arrive_expect_tx(bar_full + 8 * s, bytes);
                    issued_mask |= 1u << s;
                    issued_parity = (issued_parity & ~(1u << s)) | (ph << s);
                    tma_load_2d(sA + s * L::kA, &tmap_a, bar_full + 8 * s, kb * kBlockKBytes, tm * kBlockM);
                    tma_load_2d(sB + s * L::kB, &tmap_b, bar_full + 8 * s, kb * kBlockKBytes, tn * BN);
                    bulk_load(sSfa + s * L::kSfa, p.sfa + ((int64_t)tm * rest_k + kb * kKGroups) * 512,
                              kg * 512u, bar_full + 8 * s);
                    for (int rb = 0; rb < sfb_blocks; rb++)
                        bulk_load(sSfb + s * L::kSfb + rb * kKGroups * 512,
                                  p.sfb + ((int64_t)(tn * L::kSfbBlocks + rb) * rest_k + kb * kKGroups) * 512,
                                  kg * 512u, bar_full + 8 * s);
                }
            }
            if (!ok) {
                // Drain: every load already issued must land before the CTA exits.
                volatile int never = 0;
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s))
                        wait_parity(bar_full + 8 * s, (issued_parity >> s) & 1, p.ctl.drain_timeout_ns, &never);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_mxf4nvf4(kBlockM, BN);
            const uint32_t tmem_acc = tmem_base;
            uint32_t it = 0;
            int local = 0;
            bool ok = true, any_issued = false;
            for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, local++) {
                if (!wait_parity(bar_acc_empty, (local & 1) ^ 1, tmo, abort_flag)) {
                    report_timeout(abort_flag, p.ctl.status);
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < p.num_kb; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!wait_parity(bar_full + 8 * s, ph, tmo, abort_flag)) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int kg = min(kKGroups, p.k_groups - kb * kKGroups);
                    const uint32_t sf_cols = tmem_base + BN + (it & 1) * L::kSfColsPerStage;
                    for (int j = 0; j < kg; j++) {
                        const uint32_t col = sf_cols + j * L::kSfColsPerGroup;
                        tmem_cp_32x128_x4(col, smem_desc(sSfa + s * L::kSfa + j * 512, 16, 128, 0));
#pragma unroll
                        for (int rb = 0; rb < L::kSfbBlocks; rb++)
                            tmem_cp_32x128_x4(col + 4 + 4 * rb,
                                              smem_desc(sSfb + s * L::kSfb + (rb * kKGroups + j) * 512, 16, 128, 0));
                        const uint64_t adesc = smem_desc(sA + s * L::kA + j * 32, 16, 1024, 2);
                        const uint64_t bdesc = smem_desc(sB + s * L::kB + j * 32, 16, 1024, 2);
                        mma_mxf4nvf4(tmem_acc, adesc, bdesc, idesc, col, col + 4, (kb | j) != 0);
                    }
                    any_issued = true;
                    mma_commit(bar_empty + 8 * s);  // frees the smem slot once these MMAs finish
                }
                if (!ok) break;
                mma_commit(bar_acc_full);
            }
            if (!ok && any_issued) {
                volatile int never = 0;
                mma_commit(bar_drain);
                wait_parity(bar_drain, 0, p.ctl.drain_timeout_ns, &never);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;                 // TMEM lanes this warp may read
        const int half = (warp - 2) >> 2;             // column half of the tile
        constexpr int kCols = BN / 2;                 // columns per warp
        int local = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, local++) {
            int tm, tn;
            tile_coords(t, p, tm, tn);
            bool ok = true;
            if (lane == 0) ok = wait_parity(bar_acc_full, local & 1, tmo, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) report_timeout(abort_flag, p.ctl.status);
                break;
            }
            tc_fence_after();
            uint32_t acc[kCols];
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * kCols;
#pragma unroll
            for (int c = 0; c < kCols / 32; c++)
                tmem_ld_32x32b_x32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&acc[c * 32]));
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acc_empty);  // accumulator may be overwritten now

            store_row<kCols, F16>(acc, p, tm * kBlockM + quarter * 32 + lane, tn * BN + half * kCols);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}


// ---------------------------------------------------------------------------
// CTA-pair kernel: tcgen05 cta_group::2, one 256x256 output tile per pair.
//
// CTA rank r of the pair holds A rows [256*tm + 128*r, +128), B rows
// [256*tn + 128*r, +128), the 128-row scale block of its A rows and both 128-row
// scale blocks of the tile's B rows.  Its producer loads those into its own smem
// with cta_group::2 TMA loads whose bytes complete on the LEADER's (rank 0) full
// barrier; the leader's MMA thread issues the pair MMAs (M=256, N=256, K=64) and
// the scale copies, and commits separately to each CTA's empty / acc_full
// barriers.  Both CTAs' epilogues drain their own TMEM half and arrive on the
// leader's acc_empty barrier.  Per CTA and stage: 16 + 16 + 2 + 4 KB.
// ---------------------------------------------------------------------------
template <int STAGES>
struct PairLayout {
    static constexpr int kA = kBlockM * kBlockKBytes;   // 16 KB: this CTA's 128 A rows
    static constexpr int kB = 128 * kBlockKBytes;       // 16 KB: this CTA's 128 B rows
    static constexpr int kSfa = kKGroups * 512;         // 2 KB
    static constexpr int kSfb = 2 * kKGroups * 512;     // 4 KB: both 128-row blocks of the tile
    static constexpr int kStage = kA + kB + kSfa + kSfb;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + STAGES * kA;
    static constexpr int kOffSfa = kOffB + STAGES * kB;
    static constexpr int kOffSfb = kOffSfa + STAGES * kSfa;
    static constexpr int kOffBar = kOffSfb + STAGES * kSfb;
    static constexpr int kBarBytes = (2 * STAGES + 3) * 8 + 16;
    static constexpr int kDynamicSmem = kOffBar + kBarBytes + 1024;
    static constexpr int kSfColsPerGroup = 12;           // SFA 4 + SFB 8
    static constexpr int kSfColsPerStage = kKGroups * kSfColsPerGroup;
    static constexpr int kTmemCols = 512;
    static constexpr uint32_t kTxBytes = 2u * kStage;    // both CTAs complete on the leader's barrier
    // accumulator [0, 256), then one set of scale columns per ring stage
    static_assert(256 + STAGES * kSfColsPerStage <= kTmemCols, "tensor memory budget");
    static_assert(kDynamicSmem <= 232448, "shared memory budget");
};

template <int STAGES, bool F16, bool TRACE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    nvfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                           const Params p) {
    using L = PairLayout<STAGES>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sA = base + L::kOffA, sB = base + L::kOffB, sSfa = base + L::kOffSfa, sSfb = base + L::kOffSfb;
    const uint32_t bar_full = base + L::kOffBar;
    const uint32_t bar_empty = bar_full + 8 * STAGES;
    const uint32_t bar_acc_full = bar_empty + 8 * STAGES;
    const uint32_t bar_acc_empty = bar_acc_full + 8;
    const uint32_t bar_drain = bar_acc_empty + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base_ptr + L::kOffBar + (2 * STAGES + 3) * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const int n_m = (p.M + 255) / 256, n_n = (p.N + 255) / 256, n_tiles = n_m * n_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        mbar_init(bar_acc_full, 1);
        mbar_init(bar_acc_empty, 2 * kEpiWarps);
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        prefetch_tmap(&tmap_sfa);
        prefetch_tmap(&tmap_sfb);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint64_t tmo = p.ctl.wait_timeout_ns;
    const uint32_t lead_full = map_to_cta(bar_full, 0);

    // raster: groups of kGroupM/2 pair-rows of 256
    auto coords = [&](int t, int &tm, int &tn) {
        const int gm_max = p.group_m;
        const int per_group = gm_max * n_n;
        const int g = t / per_group, first = g * gm_max, gm = min(n_m - first, gm_max), local = t - g * per_group;
        tm = first + local % gm;
        tn = local / gm;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        if (elect_one()) {
            const int rest_k = p.K >> 6;
            uint32_t stage = 0, phase = 0;
            uint32_t dA = sA, dB = sB, dSfa = sSfa, dSfb = sSfb, emp = bar_empty, fb = lead_full, own_full = bar_full;
            bool ok = true;
            uint32_t issued_mask = 0, issued_parity = 0;
            long long t_wait = 0;
            for (int t = pair; ok && t < n_tiles; t += num_pairs) {
                int tm, tn;
                coords(t, tm, tn);
                const int arow = tm * 256 + rank * 128, brow = tn * 256 + rank * 128;
                // scale tensors viewed as rows of 256 bytes: one (128-row block, k-stage) = 8 rows
                const int ysa = (tm * 2 + (int)rank) * rest_k * 2, ysb0 = tn * 2 * rest_k * 2,
                          ysb1 = (tn * 2 + 1) * rest_k * 2;
                for (int kb = 0; kb < p.num_kb; kb++) {
                    const long long c0 = TRACE ? clock64() : 0;
                    if (!mbar_try_wait(emp, phase ^ 1) && !wait_parity(emp, phase ^ 1, tmo, abort_flag)) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    if (TRACE) t_wait += clock64() - c0;
                    if (rank == 0) {
                        mbar_arrive_expect_tx(own_full, L::kTxBytes);
                        issued_mask |= 1u << stage;
                        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    }
                    const int x = kb * kBlockKBytes, ysf = kb * kKGroups * 2;
                    tma_load_2d_pair(dA, &tmap_a, fb, x, arow);
                    tma_load_2d_pair(dB, &tmap_b, fb, x, brow);
                    tma_load_2d_pair(dSfa, &tmap_sfa, fb, 0, ysa + ysf);
                    tma_load_2d_pair(dSfb, &tmap_sfb, fb, 0, ysb0 + ysf);
                    tma_load_2d_pair(dSfb + kKGroups * 512, &tmap_sfb, fb, 0, ysb1 + ysf);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                        dA = sA;
                        dB = sB;
                        dSfa = sSfa;
                        dSfb = sSfb;
                        emp = bar_empty;
                        fb = lead_full;
                        own_full = bar_full;
                    } else {
                        dA += L::kA;
                        dB += L::kB;
                        dSfa += L::kSfa;
                        dSfb += L::kSfb;
                        emp += 8;
                        fb += 8;
                        own_full += 8;
                    }
                }
            }
            if (!ok && rank == 0) {
                volatile int never = 0;
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s))
                        wait_parity(bar_full + 8 * s, (issued_parity >> s) & 1, p.ctl.drain_timeout_ns, &never);
            }
            if (TRACE) p.trace[blockIdx.x * kTraceSlots + 2] = t_wait;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader only)
        // One thread issues every tcgen05 op of the pair, so its instruction count per
        // stage bounds the tensor rate: descriptors are advanced by constant strides
        // (never rebuilt), each ring stage owns a fixed set of scale columns in TMEM,
        // and a stage's 12 scale copies go out before its 4 MMAs.
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc = idesc_mxf4nvf4(256, 256);
            const uint32_t empty0 = map_to_cta(bar_empty, 0), empty1 = map_to_cta(bar_empty, 1);
            const uint32_t accf0 = map_to_cta(bar_acc_full, 0), accf1 = map_to_cta(bar_acc_full, 1);
            const uint64_t a_desc0 = smem_desc(sA, 16, 1024, 2), b_desc0 = smem_desc(sB, 16, 1024, 2);
            const uint64_t sfa_desc0 = smem_desc(sSfa, 16, 128, 0), sfb_desc0 = smem_desc(sSfb, 16, 128, 0);
            const uint32_t sf_col0 = tmem_base + 256;
            uint32_t stage = 0, phase = 0;
            uint64_t a_d = a_desc0, b_d = b_desc0, sfa_d = sfa_desc0, sfb_d = sfb_desc0;
            uint32_t sf_col = sf_col0, full_bar = bar_full, e0 = empty0, e1 = empty1;
            int local = 0;
            bool ok = true, any_issued = false;
            long long t_full = 0, t_acc = 0, t_first = 0;
            for (int t = pair; ok && t < n_tiles; t += num_pairs, local++) {
                long long c0 = TRACE ? clock64() : 0;
                if (!wait_parity(bar_acc_empty, (local & 1) ^ 1, tmo, abort_flag)) {
                    report_timeout(abort_flag, p.ctl.status);
                    ok = false;
                    break;
                }
                if (TRACE) {
                    const long long c1 = clock64();
                    t_acc += c1 - c0;
                    if (!t_first) t_first = c1;
                }
                tc_fence_after();
                for (int kb = 0; kb < p.num_kb; kb++) {
                    if (TRACE) c0 = clock64();
                    if (!mbar_try_wait(full_bar, phase) && !wait_parity(full_bar, phase, tmo, abort_flag)) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    if (TRACE) t_full += clock64() - c0;
                    tc_fence_after();
                    const uint32_t acc0 = kb != 0;
                    if (kb * kKGroups + kKGroups <= p.k_groups) {
                        // full stage: descriptor offsets are immediates (addr >> 4 units)
#pragma unroll
                        for (int j = 0; j < kKGroups; j++) {
                            const uint32_t col = sf_col + j * L::kSfColsPerGroup;
                            tmem_cp_32x128_x4_pair(col, sfa_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 4, sfb_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 8, sfb_d + (kKGroups + j) * 32);
                        }
#pragma unroll
                        for (int j = 0; j < kKGroups; j++) {
                            const uint32_t col = sf_col + j * L::kSfColsPerGroup;
                            mma_mxf4nvf4_pair(tmem_base, a_d + j * 2, b_d + j * 2, idesc, col, col + 4,
                                              j == 0 ? acc0 : 1u);
                        }
                    } else {
                        const int kg = p.k_groups - kb * kKGroups;  // last, partial stage
                        for (int j = 0; j < kg; j++) {
                            const uint32_t col = sf_col + j * L::kSfColsPerGroup;
                            tmem_cp_32x128_x4_pair(col, sfa_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 4, sfb_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 8, sfb_d + (kKGroups + j) * 32);
                            mma_mxf4nvf4_pair(tmem_base, a_d + j * 2, b_d + j * 2, idesc, col, col + 4,
                                              j == 0 ? acc0 : 1u);
                        }
                    }
                    any_issued = true;
                    mma_commit_pair(e0);  // frees the stage in both CTAs once these MMAs finish
                    mma_commit_pair(e1);
                    // advance the ring
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                        a_d = a_desc0;
                        b_d = b_desc0;
                        sfa_d = sfa_desc0;
                        sfb_d = sfb_desc0;
                        sf_col = sf_col0;
                        full_bar = bar_full;
                        e0 = empty0;
                        e1 = empty1;
                    } else {
                        a_d += L::kA >> 4;
                        b_d += L::kB >> 4;
                        sfa_d += L::kSfa >> 4;
                        sfb_d += L::kSfb >> 4;
                        sf_col += L::kSfColsPerStage;
                        full_bar += 8;
                        e0 += 8;
                        e1 += 8;
                    }
                }
                if (!ok) break;
                mma_commit_pair(accf0);
                mma_commit_pair(accf1);
            }
            if (!ok && any_issued) {
                volatile int never = 0;
                mma_commit_pair(map_to_cta(bar_drain, 0));
                wait_parity(bar_drain, 0, p.ctl.drain_timeout_ns, &never);
            }
            if (TRACE) {
                unsigned long long *tr = p.trace + blockIdx.x * kTraceSlots;
                tr[0] = t_full;
                tr[1] = t_acc;
                tr[5] = local;
                tr[6] = clock64() - t_first;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        constexpr int kCols = 128;
        const uint32_t lead_acc_empty = map_to_cta(bar_acc_empty, 0);
        int local = 0;
        long long t_accw = 0, t_store = 0, c_ready = 0;
        for (int t = pair; t < n_tiles; t += num_pairs, local++) {
            int tm, tn;
            coords(t, tm, tn);
            bool ok = true;
            const long long c0 = TRACE ? clock64() : 0;
            if (lane == 0) ok = wait_parity(bar_acc_full, local & 1, tmo, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (TRACE) {
                c_ready = clock64();
                t_accw += c_ready - c0;
            }
            if (!ok) {
                if (lane == 0) report_timeout(abort_flag, p.ctl.status);
                break;
            }
            tc_fence_after();
            uint32_t acc[kCols];
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * kCols;
#pragma unroll
            for (int c = 0; c < kCols / 32; c++)
                tmem_ld_32x32b_x32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&acc[c * 32]));
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(lead_acc_empty);
            store_row<kCols, F16>(acc, p, tm * 256 + (int)rank * 128 + quarter * 32 + lane, tn * 256 + half * kCols);
            if (TRACE && warp == 2 && lane == 0) t_store += clock64() - c_ready;
        }
        if (TRACE && warp == 2 && lane == 0) {
            p.trace[blockIdx.x * kTraceSlots + 3] = t_accw;
            p.trace[blockIdx.x * kTraceSlots + 4] = t_store;
        }
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, L::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct MapKey {
    int device;
    const void *ptr;
    int64_t rows, kbytes;
    int box_rows;
    bool operator==(const MapKey &o) const {
        return device == o.device && ptr == o.ptr && rows == o.rows && kbytes == o.kbytes && box_rows == o.box_rows;
    }
};

// Small LRU of encoded operand tensor maps (the reference re-encodes on every
// call, nvfp4_v5.cu:294-308).  Thread-safe.
static int operand_map(const void *ptr, int64_t rows, int64_t K, int box_rows, CUtensorMap *out) {
    static std::mutex mu;
    constexpr int kCap = 64;
    static MapKey keys[kCap];
    static CUtensorMap maps[kCap];
    static uint64_t stamp[kCap];
    static uint64_t clock = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    MapKey key{dev, ptr, rows, K / 2, box_rows};
    std::lock_guard<std::mutex> lock(mu);
    int victim = 0;
    for (int i = 0; i < kCap; i++) {
        if (stamp[i] && keys[i] == key) {
            stamp[i] = ++clock;
            *out = maps[i];
            return NVFP4_OK;
        }
        if (stamp[i] < stamp[victim]) victim = i;
    }
    CUtensorMap m;
    int st = encode_tiled_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, ptr, (uint64_t)(K / 2), (uint64_t)rows,
                             (uint64_t)(K / 2), kBlockKBytes, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    keys[victim] = key;
    maps[victim] = m;
    stamp[victim] = ++clock;
    *out = m;
    return NVFP4_OK;
}

template <int BN, int STAGES, bool F16>
static int launch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, const DeviceInfo &di) {
    using L = Layout<BN, STAGES>;
    auto kern = nvfp4_gemm_kernel<BN, STAGES, F16>;
    static int configured[64] = {};
    if (!configured[di.device]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDynamicSmem) != cudaSuccess)
            return NVFP4_ERR_CUDA;
        configured[di.device] = 1;
    }
    CUtensorMap ta, tb;
    int st = operand_map(A, M, K, kBlockM, &ta);
    if (!st) st = operand_map(B, N, K, BN, &tb);
    if (st) return st;
    Params p;
    p.sfa = SFA;
    p.sfb = SFB;
    p.d = D;
    p.M = M;
    p.N = N;
    p.K = K;
    p.alpha = alpha;
    p.num_m_tiles = (M + kBlockM - 1) / kBlockM;
    p.num_n_tiles = (N + BN - 1) / BN;
    p.num_tiles = p.num_m_tiles * p.num_n_tiles;
    p.num_kb = (K + 255) / 256;
    p.k_groups = K / 64;
    p.vec32_store = ((reinterpret_cast<uintptr_t>(D) & 31u) == 0) && (N % 16 == 0);
    p.trace = nullptr;
    if ((st = kernel_ctl(&p.ctl))) return st;
    const int grid = p.num_tiles < di.sm_count ? p.num_tiles : di.sm_count;
    kern<<<grid, kThreads, L::kDynamicSmem, stream>>>(ta, tb, p);
    count_launch();
    return cuda_status(cudaGetLastError());
}

// Raster group (256-row tile rows sharing a sweep over N) of the pair kernel;
// env NVFP4_GROUP_M overrides the default.
static int pair_group_m() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_GROUP_M");
        int x = e ? std::atoi(e) : 8;
        return x < 1 ? 1 : (x > 1024 ? 1024 : x);
    }();
    return v;
}

template <int STAGES, bool F16>
static int launch_pair(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                       void *D, int M, int N, int K, cudaStream_t stream, const DeviceInfo &di,
                       unsigned long long *trace = nullptr) {
    using L = PairLayout<STAGES>;
    auto kern = trace ? nvfp4_gemm_pair_kernel<STAGES, F16, true> : nvfp4_gemm_pair_kernel<STAGES, F16, false>;
    static int configured[2][64] = {};
    if (!configured[trace != nullptr][di.device]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDynamicSmem) != cudaSuccess)
            return NVFP4_ERR_CUDA;
        configured[trace != nullptr][di.device] = 1;
    }
    CUtensorMap ta, tb, tsa, tsb;
    int st = operand_map(A, M, K, kBlockM, &ta);
    if (!st) st = operand_map(B, N, K, 128, &tb);
    // scale tensors as [bytes/256, 256] so one (128-row block, 4 k-groups) chunk is an 8x256 box
    const uint64_t sfa_rows = (uint64_t)((M + 127) / 128) * (K / 64) * 2;
    const uint64_t sfb_rows = (uint64_t)((N + 127) / 128) * (K / 64) * 2;
    if (!st) st = encode_tiled_2d(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, SFA, 256, sfa_rows, 256, 256, 8,
                                  CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!st) st = encode_tiled_2d(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, SFB, 256, sfb_rows, 256, 256, 8,
                                  CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    Params p;
    p.sfa = SFA;
    p.sfb = SFB;
    p.d = D;
    p.M = M;
    p.N = N;
    p.K = K;
    p.alpha = alpha;
    p.num_m_tiles = (M + 255) / 256;
    p.num_n_tiles = (N + 255) / 256;
    p.num_tiles = p.num_m_tiles * p.num_n_tiles;
    p.num_kb = (K + 255) / 256;
    p.k_groups = K / 64;
    p.vec32_store = ((reinterpret_cast<uintptr_t>(D) & 31u) == 0) && (N % 16 == 0);
    p.trace = trace;
    p.group_m = pair_group_m();
    if ((st = kernel_ctl(&p.ctl))) return st;
    const int pairs = std::min(p.num_tiles, di.sm_count / 2);
    kern<<<2 * pairs, kThreads, L::kDynamicSmem, stream>>>(ta, tb, tsa, tsb, p);
    count_launch();
    return cuda_status(cudaGetLastError());
}

}  // namespace gemm

int gemm_validate(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const void *D, int M,
                  int N, int K) {
    if (!A || !SFA || !B || !SFB || !D) return NVFP4_ERR_INVALID;
    if (M < 1 || N < 8 || N % 8 || K < 64 || K % 64) return NVFP4_ERR_SHAPE;
    if (!aligned16(A) || !aligned16(SFA) || !aligned16(B) || !aligned16(SFB) || !aligned16(D)) return NVFP4_ERR_ALIGN;
    return NVFP4_OK;
}

// Kernel choice for the persistent path: the CTA-pair kernel for M > 128, the
// single-CTA kernel otherwise.  NVFP4_GEMM_VARIANT=single|pair forces one.
static int gemm_variant(int M) {
    static int forced = [] {
        const char *e = std::getenv("NVFP4_GEMM_VARIANT");
        if (!e) return 0;
        if (!std::strcmp(e, "single")) return 1;
        if (!std::strcmp(e, "pair")) return 2;
        return 0;
    }();
    if (forced) return forced;
    return M > 128 ? 2 : 1;
}

int gemm_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16) {
    int st = gemm_validate(A, SFA, B, SFB, D, M, N, K);
    if (st) return st;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    if (gemm_variant(M) == 2) {
        if (f16) return gemm::launch_pair<5, true>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di);
        return gemm::launch_pair<5, false>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di);
    }
    if (f16) return gemm::launch<256, 4, true>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di);
    return gemm::launch<256, 4, false>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di);
}

// Pair kernel with the per-CTA cycle trace on (trace: 148 x kTraceSlots u64 on the device).
int gemm_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D, int M,
               int N, int K, unsigned long long *trace, cudaStream_t stream) {
    int st = gemm_validate(A, SFA, B, SFB, D, M, N, K);
    if (st) return st;
    if (!trace) return NVFP4_ERR_INVALID;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    return gemm::launch_pair<5, false>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, trace);
}

}  // namespace nvfp4
