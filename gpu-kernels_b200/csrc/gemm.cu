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

#include "gemm_common.cuh"

namespace nvfp4 {

namespace gemm {

constexpr int kThreads = 32 * (2 + kEpiWarps);  // producer, MMA, 8 epilogue warps

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

__device__ __forceinline__ void tile_coords(int t, const Params &p, int &tm, int &tn) {
    const int per_group = kGroupM * p.num_n_tiles;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(p.num_m_tiles - first_m, kGroupM);
    const int local = t - g * per_group;
    tm = first_m + local % gm;
    tn = local / gm;
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
    // Launched as a programmatic dependent of the previous kernel in the stream: the
    // set-up above overlapped that kernel's tail; nothing of global memory is read or
    // written before it has completed.
    grid_dependency_wait();
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
            grid_launch_dependents();  // all loads issued: the next kernel may start its set-up
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

            if (p.epi.plain())
                store_row<kCols, F16>(acc, p, tm * kBlockM + quarter * 32 + lane, tn * BN + half * kCols, p.M,
                                      p.alpha);
            else
                store_row_epi<kCols>(acc, p, tm * kBlockM + quarter * 32 + lane, tn * BN + half * kCols, p.M,
                                     p.alpha, load_bias_lane(p.epi, p.N, tn * BN + half * kCols, lane));
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
// host side
// ---------------------------------------------------------------------------
struct MapKey {
    int device;
    int kind;  // 0: NVFP4 operand, 1: 16-bit output D
    const void *ptr;
    int64_t rows, row_bytes;
    int box_rows, box_bytes;
    bool operator==(const MapKey &o) const {
        return device == o.device && kind == o.kind && ptr == o.ptr && rows == o.rows && row_bytes == o.row_bytes &&
               box_rows == o.box_rows && box_bytes == o.box_bytes;
    }
};

// Small LRU of encoded tensor maps (the reference re-encodes on every call,
// nvfp4_v5.cu:294-308).  Thread-safe.
static int cached_map(const MapKey &key, CUtensorMapDataType dtype, uint64_t inner, CUtensorMapSwizzle swizzle,
                      uint32_t box_inner, CUtensorMap *out) {
    static std::mutex mu;
    constexpr int kCap = 64;
    static MapKey keys[kCap];
    static CUtensorMap maps[kCap];
    static uint64_t stamp[kCap];
    static uint64_t clock = 0;
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
    int st = encode_tiled_2d(&m, dtype, key.ptr, inner, (uint64_t)key.rows, (uint64_t)key.row_bytes, box_inner,
                             (uint32_t)key.box_rows, swizzle);
    if (st) return st;
    keys[victim] = key;
    maps[victim] = m;
    stamp[victim] = ++clock;
    *out = m;
    return NVFP4_OK;
}

int operand_map(const void *ptr, int64_t rows, int64_t K, int box_rows, int box_bytes, CUtensorMap *out) {
    int dev = 0;
    cudaGetDevice(&dev);
    const MapKey key{dev, 0, ptr, rows, K / 2, box_rows, box_bytes};
    return cached_map(key, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(K / 2),
                      box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, (uint32_t)box_bytes,
                      out);
}

// Store map of a 16-bit [M, N] output: boxes of 16 columns x box_rows rows, 32-byte swizzle.
int output_map(const void *ptr, int64_t M, int64_t N, int box_rows, CUtensorMap *out) {
    int dev = 0;
    cudaGetDevice(&dev);
    const MapKey key{dev, 1, ptr, M, N * 2, box_rows, 32};
    return cached_map(key, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)N, CU_TENSOR_MAP_SWIZZLE_32B, 16u, out);
}

template <int BN, int STAGES, bool F16>
static int launch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, const DeviceInfo &di, const Epi &epi) {
    using L = Layout<BN, STAGES>;
    auto kern = nvfp4_gemm_kernel<BN, STAGES, F16>;
    static int configured[64] = {};
    if (!configured[di.device]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDynamicSmem) != cudaSuccess)
            return NVFP4_ERR_CUDA;
        configured[di.device] = 1;
    }
    CUtensorMap ta, tb;
    int st = operand_map(A, M, K, kBlockM, kBlockKBytes, &ta);
    if (!st) st = operand_map(B, N, K, BN, kBlockKBytes, &tb);
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
    p.group_m = kGroupM;
    p.clc = 0;
    p.tma_store = 0;
    p.spin = 0;
    p.l2hint = 0;
    p.epi = epi;
    if ((st = kernel_ctl(&p.ctl))) return st;
    const int grid = p.num_tiles < di.sm_count ? p.num_tiles : di.sm_count;
    // A programmatic dependent of the previous kernel in the stream for M > 128: its
    // set-up then overlaps that kernel's tail (back-to-back 2048³ 14.6 -> 13.5 us,
    // 1024 x 1024 x 4096 14.4 -> 13.5 us).  Not for M <= 128, the weight-streaming
    // calls, where it measured 2 % slower (28672 x 8192 weights, M = 32-128, from
    // CUDA-graph replays: 24.9-26.4 against 25.4-27.0 us).  Env NVFP4_SINGLE_PDL=0|1
    // overrides.
    static const int pdl_env = [] {
        const char *e = std::getenv("NVFP4_SINGLE_PDL");
        return e ? (std::atoi(e) ? 1 : 0) : -1;
    }();
    const int pdl = pdl_env >= 0 ? pdl_env : (M > kBlockM ? 1 : 0);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kDynamicSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, ta, tb, p) != cudaSuccess) return NVFP4_ERR_CUDA;
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

int pair_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16, const DeviceInfo &di, const Epi &epi);

// Kernel choice for the persistent path: the single-CTA kernel for M <= 128 and for
// small grids with short K, the CTA-pair kernel otherwise.  The two give the same
// bits (each output element is one fp32 sum over K in the same order, then the same
// rounding).  A launch of at most one wave of 256 x 256 tiles is bound by fixed
// per-tile costs, which are lower in the single-CTA kernel (no cluster set-up, one
// accumulator hand-off inside the CTA): measured, 1024³ 10.2 against 13.3 us, 2048³
// 13.1 against 15.1 us, 512 x 2048 x 4096 16.4 against 17.2 us; with longer K the
// pair kernel's lower cost per k-block wins (1536 x 1536 x 8192: 23.4 against 22.0
// us).  NVFP4_GEMM_VARIANT=single|pair forces one.
static int gemm_variant(int M, int N, int K, int pairs, const Epi &epi) {
    static int forced = [] {
        const char *e = std::getenv("NVFP4_GEMM_VARIANT");
        if (!e) return 0;
        if (!std::strcmp(e, "single")) return 1;
        if (!std::strcmp(e, "pair")) return 2;
        return 0;
    }();
    if (forced) return forced;
    if (M <= 128) return 1;
    if (epi.act == kActSwiglu) return 2;  // the single-CTA epilogue has no SwiGLU
    const int64_t tiles = (int64_t)((M + 255) / 256) * ((N + 255) / 256);
    if (tiles <= pairs && (K <= 2048 || (K <= 4096 && tiles <= 32))) return 1;
    return 2;
}

// Persistent GEMM (single-CTA or CTA-pair kernel) with an optional fused epilogue;
// with NVFP4 output (epi.q) D is not written and may be null.
int gemm_dispatch_epi(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                      int M, int N, int K, cudaStream_t stream, bool f16, const Epi &epi) {
    int st = gemm_validate(A, SFA, B, SFB, epi.q ? epi.q : D, M, N, K);
    if (st) return st;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    if (gemm_variant(M, N, K, di.sm_count / 2, epi) == 2)
        return pair_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, stream, f16, di, epi);
    if (epi.act == kActSwiglu) return NVFP4_ERR_UNSUPPORTED;  // the single-CTA epilogue has no SwiGLU
    if (f16) return gemm::launch<256, 4, true>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, epi);
    return gemm::launch<256, 4, false>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, epi);
}

int gemm_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16) {
    return gemm_dispatch_epi(A, SFA, B, SFB, alpha, D, M, N, K, stream, f16, Epi());
}

}  // namespace nvfp4
