// gemm_pair.cu — CTA-pair (tcgen05 cta_group::2) persistent NVFP4 GEMM, one 256 x BN
// output tile per pair of SMs.  The kernel for M > 128.
//
// CTA rank r of the pair holds A rows [256*tm + 128*r, +128), B rows
// [BN*tn + BN/2*r, +BN/2), the 128-row scale block of its A rows and the two
// 128-row scale blocks that cover the tile's BN B rows (the MMA reads B's scales
// from each CTA's own TMEM).  Each CTA's producers load those with cta_group::2 TMA
// loads — each CTA fetches only its own tiles — whose bytes complete on the LEADER's
// (rank 0) full barrier; the leader's MMA thread issues the pair MMAs (M=256, N=BN,
// K=64) and the scale copies, and commits separately to each CTA's empty / acc_full
// barriers.  Both CTAs' epilogues drain their own 128 x BN TMEM half and arrive on
// the leader's acc_empty barrier.
//
// BN = 256 (one accumulator: the next tile's MMAs wait for the epilogue to read the
// previous one out of TMEM) or BN = 192 (two accumulators of 192 columns, so the
// MMAs of tile i+1 run while the epilogue drains tile i).  A 192-row B tile starts
// 64 rows into a 128-row scale block on odd tn; its scales are then read from the
// scale columns shifted by 2 (each TMEM scale column holds 32 rows).
//
// The ring is latency-bound: a slot is reloaded only after the MMAs that read it
// have completed, so throughput = slots / (queued MMA time + commit->producer
// wake-up + TMA issue + TMA latency, ~1.9K + 0.3K + 1.5K cycles measured).  Slot
// width is a template parameter: BKB = 128 bytes of K per row (256 fp4, the
// default) or BKB = 64 (128 fp4, 64-byte swizzle).  Two producer warps issue each
// slot's loads (A/B and the scales) in parallel, and a single MMA thread issues
// with strided (never rebuilt) descriptors.
#include <cstdlib>
#include <cstring>

#include "gemm_common.cuh"
#include "grouped.cuh"

namespace nvfp4 {
namespace gemm {

constexpr int kTileQ = 4;  // tile ids the scheduler may publish ahead of the slowest consumer

template <int STAGES, int BKB, int BN>
struct PairLayout {
    static_assert(BKB == 128 || BKB == 64, "slot width");
    static_assert(BN == 256 || BN == 192, "tile width");
    static constexpr int kKG = BKB / 32;                 // 64-element k-groups per slot
    static constexpr int kBRows = BN / 2;                // B rows held by each CTA
    static constexpr int kA = 128 * BKB;                 // this CTA's 128 A rows
    static constexpr int kB = kBRows * BKB;              // this CTA's BN/2 B rows
    static constexpr int kSfa = kKG * 512;               // A scales (one 128-row block)
    static constexpr int kSfb = 2 * kKG * 512;           // B scales (the two 128-row blocks covering the tile)
    static constexpr int kStage = kA + kB + kSfa + kSfb;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + STAGES * kA;
    static constexpr int kOffSfa = kOffB + STAGES * kB;
    static constexpr int kOffSfb = kOffSfa + STAGES * kSfa;
    static constexpr int kOffBar = kOffSfb + STAGES * kSfb;
    static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;  // full, empty, acc_full x2, acc_empty x2, drain
    // cluster-launch-control tile queue: response (16 B), its barrier, kTileQ entries
    // with full / empty barriers
    static constexpr int kOffSched = (kOffBar + kBarBytes + 127) / 128 * 128;
    static constexpr int kSchedBytes = 16 + 8 + kTileQ * (4 + 8 + 8) + 8;
    // One region, two uses that never meet: the grouped GEMM's tables (first row, end
    // row, first tile and first A-scale block of each group), or the epilogue's staging
    // — per epilogue warp 4 KB, holding either two 1 KB boxes of 32 rows x 16 16-bit
    // columns for TMA stores of D (32-byte swizzle) or a 32 x 64 chunk that the gather
    // epilogue writes out row-contiguously.  Staging only where the budget allows.
    static constexpr int kGroupBytes = 4 * (kMaxGroups + 1) * 4;
    static constexpr int kStageBox = 32 * 32;
    static constexpr int kStageWarp = 4096;
    static constexpr int kStageNeed = kEpiWarps * kStageWarp;
    static constexpr int kOffStage = (kOffSched + kSchedBytes + 1023) / 1024 * 1024;
    static constexpr int kOffGroups = kOffStage;
    static constexpr bool kHasStage = kOffStage + kStageNeed + 1024 <= 232448;
    static constexpr int kRegion = (kHasStage && kStageNeed > kGroupBytes) ? kStageNeed : kGroupBytes;
    // the NVFP4 output's scale-code tables (quant_common.cuh), built by the epilogue warps
    static constexpr int kOffTable = kOffStage + kRegion;
    static constexpr int kDynamicSmem = kOffTable + (int)sizeof(ScaleTables) + 1024;
    static constexpr uint32_t kTxBytes = 2u * kStage;    // both CTAs complete on the leader's barrier
    // shared-memory matrix descriptor: 128B or 64B swizzle, 8-row core groups
    static constexpr uint32_t kLayout = BKB == 128 ? 2 : 4;
    static constexpr uint32_t kSbo = 8 * BKB;
    // TMEM: kAccBufs accumulators of BN columns, then rotating sets of scale columns
    // (SFA 4 + SFB 8 per k-group); the tensor pipe executes copies and MMAs in issue
    // order, so a set is rewritten only after the MMAs that read it
    static constexpr int kSfColsPerGroup = 12;
    static constexpr int kSfCols = kKG * kSfColsPerGroup;
    static constexpr int kTmemCols = 512;
    static constexpr int kAccBufs = (2 * BN + kSfCols <= kTmemCols) ? 2 : 1;
    static constexpr int kSfBase = kAccBufs * BN;
    static constexpr int kSfSetsFit = (kTmemCols - kSfBase) / kSfCols;
    static constexpr int kSfSets = kSfSetsFit < STAGES ? kSfSetsFit : STAGES;
    static_assert(kSfSets >= 1 && kSfBase + kSfSets * kSfCols <= kTmemCols, "tensor memory budget");
    static_assert(kB % 1024 == 0, "B slot must keep 1024-byte alignment for the swizzle");
    static_assert(kOffSched % 16 == 0, "the cluster-launch-control response is read as 16 bytes");
    static_assert(kDynamicSmem <= 232448, "shared memory budget");
    static_assert(kDynamicSmem <= 232448, "shared memory budget");
};

// warps: 0 A/B producer, 1 MMA (+ TMEM owner), 2..9 epilogue, 10 scale producer,
// 11 tile scheduler (cluster launch control, leader CTA)
constexpr int kSfProducerWarp = 2 + kEpiWarps;
constexpr int kSchedWarp = kSfProducerWarp + 1;
constexpr int kPairThreads = 32 * (kSchedWarp + 1);
// consumers of each tile-queue entry: both producers of both CTAs, the leader's MMA
// thread, every epilogue warp of both CTAs
constexpr int kTileQConsumers = 2 * 2 + 1 + 2 * kEpiWarps;

// Output tile t of the persistent schedule: its coordinates and where its rows live.
struct TileInfo {
    int tm, tn;
    int a_row0;      // first A / D row of the 256-row tile
    int row_end;     // rows >= row_end are not stored
    int sfa_block0;  // 128-row A scale block of the tile's first row
    int b_row0;      // first B row of the tile's weight matrix
    int sfb_block0;  // its first 128-row scale block
    float alpha;
    int group;       // grouped launch: the tile's group (else 0)
    int sf_row_off;  // NVFP4 output: scale row of D row r is r + sf_row_off (per-group layout)
};

template <int STAGES, int BKB, int BN, bool F16, bool TRACE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    nvfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                           const __grid_constant__ CUtensorMap tmap_d, const Params p) {
    using L = PairLayout<STAGES, BKB, BN>;
    constexpr int KG = L::kKG;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t sA = base + L::kOffA, sB = base + L::kOffB, sSfa = base + L::kOffSfa, sSfb = base + L::kOffSfb;
    const uint32_t bar_full = base + L::kOffBar;
    const uint32_t bar_empty = bar_full + 8 * STAGES;
    const uint32_t bar_acc_full = bar_empty + 8 * STAGES;
    const uint32_t bar_acc_empty = bar_acc_full + 16;  // [2] each; buffer b at +8*b
    const uint32_t bar_drain = bar_acc_empty + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(base_ptr + L::kOffBar + (2 * STAGES + 5) * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *g_row0 = reinterpret_cast<int *>(base_ptr + L::kOffGroups);  // [groups] first row
    int *g_rend = g_row0 + (kMaxGroups + 1);                           // [groups] end row
    int *g_tile0 = g_rend + (kMaxGroups + 1);                          // [groups + 1] first tile
    int *g_sfa0 = g_tile0 + (kMaxGroups + 1);                          // [groups + 1] first scale block
    // tile queue (cluster launch control): response, its barrier, entries, full/empty
    const uint32_t clc_resp = base + L::kOffSched;  // 16-byte aligned
    const uint32_t clc_bar = clc_resp + 16;
    const uint32_t tq_full = clc_bar + 8;                // [kTileQ]
    const uint32_t tq_empty = tq_full + 8 * kTileQ;      // [kTileQ], leader only
    const uint32_t tq_tile = tq_empty + 8 * kTileQ;      // [kTileQ] int
    volatile int *tq_tile_ptr = reinterpret_cast<volatile int *>(base_ptr + L::kOffSched + 24 + 16 * kTileQ);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    if (TRACE && threadIdx.x == 0) p.trace[blockIdx.x * kTraceSlots + 8] = global_timer_ns();
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const int n_m = (p.M + 255) / 256, n_n = (p.N + BN - 1) / BN;
    const int G = p.grouped.groups;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(bar_acc_full + 8 * b, 1);
            mbar_init(bar_acc_empty + 8 * b, 2 * kEpiWarps);
        }
        mbar_init(bar_drain, 1);
        mbar_init(clc_bar, 1);
        for (int q = 0; q < kTileQ; q++) {
            mbar_init(tq_full + 8 * q, 1);
            mbar_init(tq_empty + 8 * q, kTileQConsumers);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        prefetch_tmap(&tmap_sfa);
        prefetch_tmap(&tmap_sfb);
        if (p.tma_store) prefetch_tmap(&tmap_d);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
        tmem_relinquish_pair();
    }
    // Launched as a programmatic dependent of the previous kernel in the stream: the
    // set-up above overlapped that kernel's tail; nothing of global memory is read or
    // written before it has completed.
    grid_dependency_wait();
    if (G > 0 && warp == 2)
        build_group_tables(p.grouped.m_offsets, G, p.grouped.m_total, n_n, lane, g_row0, g_rend, g_sfa0, g_tile0);
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint64_t tmo = p.ctl.wait_timeout_ns;
    const uint32_t lead_full = map_to_cta(bar_full, 0);
    const int n_tiles = G > 0 ? g_tile0[G] : n_m * n_n;

    // The k-th tile this pair works on (k = 0, 1, ...), or -1 when there is none.
    // Static schedule: pair + k * num_pairs.  Cluster launch control: k = 0 is the
    // cluster's own tile (its index in the grid), k >= 1 comes from the tile queue the
    // leader's scheduler fills with clusters it cancelled; every consumer frees the
    // entry on the leader's empty barrier once it has read it.
    const uint32_t lead_tq_empty = map_to_cta(tq_empty, 0);
    auto tile_at = [&](int k, bool &ok) -> int {
        if (!p.clc) {
            const int t = pair + k * num_pairs;
            return t < n_tiles ? t : -1;
        }
        if (k == 0) return pair < n_tiles ? pair : -1;
        const int j = k - 1, q = j % kTileQ;
        if (!wait_parity_cluster(tq_full + 8 * q, (uint32_t)(j / kTileQ) & 1u, tmo, abort_flag)) {
            report_timeout(abort_flag, p.ctl.status);
            ok = false;
            return -1;
        }
        const int t = tq_tile_ptr[q];
        mbar_arrive_cluster(lead_tq_empty + 8 * q);
        return t;
    };

    // raster: groups of p.group_m 256-row tile rows sweep N together (L2 reuse of A)
    auto coords = [&](int t, int nm, int &tm, int &tn) {
        const int gm_max = p.group_m;
        const int per_group = gm_max * n_n;
        const int g = t / per_group, first = g * gm_max, gm = min(nm - first, gm_max), local = t - g * per_group;
        tm = first + local % gm;
        tn = local / gm;
    };
    auto tile_info = [&](int t) {
        TileInfo ti;
        if (G == 0) {
            coords(t, n_m, ti.tm, ti.tn);
            ti.a_row0 = ti.tm * 256;
            ti.row_end = p.M;
            ti.sfa_block0 = ti.tm * 2;
            ti.b_row0 = 0;
            ti.sfb_block0 = 0;
            ti.alpha = p.alpha;
            ti.group = 0;
            ti.sf_row_off = 0;
        } else {
            const int g = last_group_at_or_before(g_tile0, G, t);  // g_tile0[g] <= t < g_tile0[g + 1]
            const int r0 = g_row0[g], r1 = g_rend[g];
            coords(t - g_tile0[g], (r1 - r0 + 255) / 256, ti.tm, ti.tn);
            ti.a_row0 = r0 + ti.tm * 256;
            ti.row_end = r1;
            ti.sfa_block0 = g_sfa0[g] + ti.tm * 2;
            ti.b_row0 = g * p.N;
            ti.sfb_block0 = g * (p.N >> 7);
            ti.alpha = p.grouped.alphas[g];
            ti.group = g;
            ti.sf_row_off = g_sfa0[g] * 128 - r0;
        }
        return ti;
    };

    if (warp == 0 || warp == kSfProducerWarp) {
        // ------------------------------------------------------------ producers (both CTAs)
        // warp 0: the A and B tiles (and, on the leader, the slot's expected bytes);
        // the last warp: the scale tiles.  Both wait on the same empty barrier.
        if (elect_one()) {
            const bool ab = warp == 0;
            const int rest_k = p.K >> 6;
            const uint64_t pol_ab = policy_evict_last();  // operands kept in L2 (l2hint >= 2)
            uint32_t stage = 0, phase = 0;
            uint32_t d0 = ab ? sA : sSfa, d1 = ab ? sB : sSfb, emp = bar_empty, fb = lead_full, own_full = bar_full;
            bool ok = true;
            uint32_t issued_mask = 0, issued_parity = 0;
            long long t_wait = 0;
            for (int k = 0; ok; k++) {
                const int t = tile_at(k, ok);
                if (t < 0) break;
                const TileInfo ti = tile_info(t);
                const int arow = ti.a_row0 + rank * 128, brow = ti.b_row0 + ti.tn * BN + rank * L::kBRows;
                // scale tensors viewed as rows of 256 bytes: one (128-row block, 64-K group) =
                // 2 rows; the tile's B rows lie in 128-row blocks sb and sb + 1
                const int sb = ti.sfb_block0 + ((ti.tn * BN) >> 7);
                const int ysa = (ti.sfa_block0 + (int)rank) * rest_k * 2, ysb0 = sb * rest_k * 2,
                          ysb1 = (sb + 1) * rest_k * 2;
                for (int kb = 0; kb < p.num_kb; kb++) {
                    const long long c0 = TRACE ? clock64() : 0;
                    if (!(p.spin >= 2 ? spin_parity(emp, phase ^ 1, tmo, abort_flag)
                                      : (mbar_try_wait(emp, phase ^ 1) || wait_parity(emp, phase ^ 1, tmo, abort_flag)))) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    if (TRACE) t_wait += clock64() - c0;
                    if (ab) {
                        if (rank == 0) {
                            mbar_arrive_expect_tx(own_full, L::kTxBytes);
                            issued_mask |= 1u << stage;
                            issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                        }
                        const int x = kb * BKB;
                        if (p.l2hint >= 2) {
                            tma_load_2d_pair_hint(d0, &tmap_a, fb, x, arow, pol_ab);
                            tma_load_2d_pair_hint(d1, &tmap_b, fb, x, brow, pol_ab);
                        } else {
                            tma_load_2d_pair(d0, &tmap_a, fb, x, arow);
                            tma_load_2d_pair(d1, &tmap_b, fb, x, brow);
                        }
                    } else {
                        const int ysf = kb * KG * 2;
                        tma_load_2d_pair(d0, &tmap_sfa, fb, 0, ysa + ysf);
                        tma_load_2d_pair(d1, &tmap_sfb, fb, 0, ysb0 + ysf);
                        tma_load_2d_pair(d1 + KG * 512, &tmap_sfb, fb, 0, ysb1 + ysf);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                        d0 = ab ? sA : sSfa;
                        d1 = ab ? sB : sSfb;
                        emp = bar_empty;
                        fb = lead_full;
                        own_full = bar_full;
                    } else {
                        d0 += ab ? L::kA : L::kSfa;
                        d1 += ab ? L::kB : L::kSfb;
                        emp += 8;
                        fb += 8;
                        own_full += 8;
                    }
                }
            }
            if (ab) grid_launch_dependents();  // all loads issued: the next kernel may start its set-up
            if (!ok && ab && rank == 0) {
                volatile int never = 0;
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s))
                        wait_parity(bar_full + 8 * s, (issued_parity >> s) & 1, p.ctl.drain_timeout_ns, &never);
            }
            if (TRACE && ab) p.trace[blockIdx.x * kTraceSlots + 2] = t_wait;
        }
    } else if (warp == kSchedWarp) {
        // ------------------------------------------------------------ tile scheduler (leader)
        // Cluster launch control: cancel a cluster that has not started yet and take over
        // its tile; publish the tile (or -1 once none is left) in both CTAs' queues.
        if (p.clc && rank == 0 && pair < n_tiles && elect_one()) {
            const uint32_t peer_tile = map_to_cta(tq_tile, 1), peer_full = map_to_cta(tq_full, 1);
            const uint32_t own_full = map_to_cta(tq_full, 0);
            for (int j = 0;; j++) {
                const int q = j % kTileQ;
                if (!wait_parity_cluster(tq_empty + 8 * q, ((uint32_t)(j / kTileQ) & 1u) ^ 1u, tmo, abort_flag)) {
                    report_timeout(abort_flag, p.ctl.status);
                    break;
                }
                mbar_arrive_expect_tx(clc_bar, 16);
                clc_try_cancel(clc_resp, clc_bar);
                if (!wait_parity(clc_bar, (uint32_t)j & 1u, tmo, abort_flag)) {
                    report_timeout(abort_flag, p.ctl.status);
                    break;
                }
                uint32_t x = 0;
                int t = clc_query(clc_resp, x) ? (int)(x >> 1) : -1;
                if (t >= n_tiles) t = -1;
                tq_tile_ptr[q] = t;
                st_shared_cluster_u32(peer_tile + 4 * q, (uint32_t)t);
                mbar_arrive_cluster(own_full + 8 * q);
                mbar_arrive_cluster(peer_full + 8 * q);
                if (t < 0) break;  // no cluster left: try_cancel is not issued again
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader only)
        // One thread issues every tcgen05 op of the pair, so its instruction count per
        // slot bounds the tensor rate: descriptors advance by constant strides, scale
        // columns rotate through kSfSets sets, and a slot's scale copies go out before
        // its MMAs.
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc = idesc_mxf4nvf4(256, BN);
            const uint32_t empty0 = map_to_cta(bar_empty, 0), empty1 = map_to_cta(bar_empty, 1);
            const uint32_t accf0 = map_to_cta(bar_acc_full, 0), accf1 = map_to_cta(bar_acc_full, 1);
            const uint64_t a_desc0 = smem_desc(sA, 16, L::kSbo, L::kLayout);
            const uint64_t b_desc0 = smem_desc(sB, 16, L::kSbo, L::kLayout);
            const uint64_t sfa_desc0 = smem_desc(sSfa, 16, 128, 0), sfb_desc0 = smem_desc(sSfb, 16, 128, 0);
            const uint32_t sf_col0 = tmem_base + L::kSfBase;
            uint32_t stage = 0, phase = 0, sf_set = 0;
            uint64_t a_d = a_desc0, b_d = b_desc0, sfa_d = sfa_desc0, sfb_d = sfb_desc0;
            uint32_t sf_col = sf_col0, full_bar = bar_full, e0 = empty0, e1 = empty1;
            int local = 0;
            bool ok = true, any_issued = false;
            long long t_full = 0, t_acc = 0, t_first = 0;
            uint64_t ns_first = 0, ns_landed3 = 0, ns_resume3 = 0;  // hand-off sample (kept in registers)
            for (int k = 0; ok; k++, local++) {
                const int t = tile_at(k, ok);
                if (t < 0) break;
                const int tn = tile_info(t).tn;
                // accumulator buffer and its use count; B-scale column shift of this tile
                const uint32_t buf = L::kAccBufs == 2 ? (uint32_t)(local & 1) : 0u;
                const uint32_t use = L::kAccBufs == 2 ? (uint32_t)(local >> 1) : (uint32_t)local;
                const uint32_t d_tmem = tmem_base + buf * BN;
                const uint32_t sfb_shift = (uint32_t)(((tn * BN) & 127) >> 5);
                long long c0 = 0;
                // The accumulator is waited for just before the tile's first MMA: the first
                // slot's scale copies (other tensor-memory columns) go out before, so they
                // run while the epilogue is still reading the previous tile out.
                auto wait_acc = [&]() -> bool {
                    if (TRACE) c0 = clock64();
                    if (!(p.spin ? spin_parity(bar_acc_empty + 8 * buf, (use & 1) ^ 1, tmo, abort_flag)
                                 : wait_parity(bar_acc_empty + 8 * buf, (use & 1) ^ 1, tmo, abort_flag))) {
                        report_timeout(abort_flag, p.ctl.status);
                        return false;
                    }
                    if (TRACE) {
                        const long long c1 = clock64();
                        t_acc += c1 - c0;
                        if (local == 3) ns_resume3 = global_timer_ns();  // hand-off sample: MMA resumes
                        if (!t_first) {
                            t_first = c1;
                            ns_first = global_timer_ns();
                        }
                    }
                    tc_fence_after();
                    return true;
                };
                for (int kb = 0; kb < p.num_kb; kb++) {
                    if (TRACE) c0 = clock64();
                    if (!(p.spin ? spin_parity(full_bar, phase, tmo, abort_flag)
                                 : (mbar_try_wait(full_bar, phase) || wait_parity(full_bar, phase, tmo, abort_flag)))) {
                        report_timeout(abort_flag, p.ctl.status);
                        ok = false;
                        break;
                    }
                    if (TRACE) t_full += clock64() - c0;
                    if (TRACE && local == 3 && kb == 0) ns_landed3 = global_timer_ns();  // tile 3's first slot landed
                    tc_fence_after();
                    const uint32_t acc0 = kb != 0;
                    if ((kb + 1) * KG <= p.k_groups) {
                        // full slot: descriptor offsets are immediates (addr >> 4 units)
                        any_issued = true;  // an abort after these copies drains them
#pragma unroll
                        for (int j = 0; j < KG; j++) {
                            const uint32_t col = sf_col + j * L::kSfColsPerGroup;
                            tmem_cp_32x128_x4_pair(col, sfa_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 4, sfb_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 8, sfb_d + (KG + j) * 32);
                        }
                        if (kb == 0 && !wait_acc()) {
                            ok = false;
                            break;
                        }
#pragma unroll
                        for (int j = 0; j < KG; j++) {
                            const uint32_t col = sf_col + j * L::kSfColsPerGroup;
                            mma_mxf4nvf4_pair(d_tmem, a_d + j * 2, b_d + j * 2, idesc, col, col + 4 + sfb_shift,
                                              j == 0 ? acc0 : 1u);
                        }
                    } else {
                        const int kg = p.k_groups - kb * KG;  // last, partial slot
                        if (kb == 0 && !wait_acc()) {
                            ok = false;
                            break;
                        }
                        for (int j = 0; j < kg; j++) {
                            const uint32_t col = sf_col + j * L::kSfColsPerGroup;
                            tmem_cp_32x128_x4_pair(col, sfa_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 4, sfb_d + j * 32);
                            tmem_cp_32x128_x4_pair(col + 8, sfb_d + (KG + j) * 32);
                            mma_mxf4nvf4_pair(d_tmem, a_d + j * 2, b_d + j * 2, idesc, col, col + 4 + sfb_shift,
                                              j == 0 ? acc0 : 1u);
                        }
                    }
                    any_issued = true;
                    mma_commit_pair(e0);  // frees the slot in both CTAs once these MMAs finish
                    mma_commit_pair(e1);
                    if (++sf_set == L::kSfSets) {
                        sf_set = 0;
                        sf_col = sf_col0;
                    } else {
                        sf_col += L::kSfCols;
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                        a_d = a_desc0;
                        b_d = b_desc0;
                        sfa_d = sfa_desc0;
                        sfb_d = sfb_desc0;
                        full_bar = bar_full;
                        e0 = empty0;
                        e1 = empty1;
                    } else {
                        a_d += L::kA >> 4;
                        b_d += L::kB >> 4;
                        sfa_d += L::kSfa >> 4;
                        sfb_d += L::kSfb >> 4;
                        full_bar += 8;
                        e0 += 8;
                        e1 += 8;
                    }
                }
                if (!ok) break;
                mma_commit_pair(accf0 + 8 * buf);
                mma_commit_pair(accf1 + 8 * buf);
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
                const uint64_t ns_last = global_timer_ns();
                tr[7] = ns_last - ns_first;
                tr[10] = ns_first;
                tr[11] = ns_last;
                tr[12] = ns_landed3;
                tr[13] = ns_resume3;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        constexpr int kCols = BN / 2;
        const uint32_t lead_acc_empty = map_to_cta(bar_acc_empty, 0);
        // NVFP4 output: the scale-code tables of this launch's global scale, built once
        // by the epilogue warps while the first tile's MMAs run
        ScaleTables *tab = reinterpret_cast<ScaleTables *>(base_ptr + L::kOffTable);
        ScaleGuess guess{0.0f, 1.0f};
        bool gs_ok = false;
        if constexpr (!F16) {
            if (p.epi.q) {
                const float gs = *p.epi.gs;
                gs_ok = gs_usable(gs);
                guess = scale_guess_factor(gs);
                build_scale_tables(tab, gs, (int)threadIdx.x - 64, 32 * kEpiWarps);
                named_barrier(1, 32 * kEpiWarps);
            }
        }
        const uint64_t pol_d = policy_evict_first();  // D stores leave L2 first (l2hint >= 1)
        const bool d_hint = p.l2hint >= 1;
        int local = 0;
        uint32_t chunk = 0;  // TMA-store boxes issued by this warp (two staging boxes alternate)
        long long t_accw = 0, t_store = 0, c_ready = 0;
        uint64_t ns_wake2 = 0, ns_read2 = 0;  // hand-off sample (kept in registers)
        for (int k = 0;; k++, local++) {
            bool okq = true;
            int t = 0;
            if (lane == 0) t = tile_at(k, okq);
            t = __shfl_sync(0xffffffffu, t, 0);
            if (t < 0) break;
            const TileInfo ti = tile_info(t);
            const uint32_t buf = L::kAccBufs == 2 ? (uint32_t)(local & 1) : 0u;
            const uint32_t use = L::kAccBufs == 2 ? (uint32_t)(local >> 1) : (uint32_t)local;
            bool ok = true;
            const long long c0 = TRACE ? clock64() : 0;
            if (lane == 0)
                ok = p.spin ? spin_parity(bar_acc_full + 8 * buf, use & 1, tmo, abort_flag)
                            : wait_parity(bar_acc_full + 8 * buf, use & 1, tmo, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            uint64_t ns_ready = 0;
            if (TRACE) {
                c_ready = clock64();
                t_accw += c_ready - c0;
                ns_ready = global_timer_ns();
            }
            if (!ok) {
                if (lane == 0) report_timeout(abort_flag, p.ctl.status);
                break;
            }
            tc_fence_after();
            uint32_t acc[kCols];
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN + half * kCols;
#pragma unroll
            for (int c = 0; c < kCols / 32; c++)
                tmem_ld_32x32b_x32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&acc[c * 32]));
            tmem_ld_wait();
            if (TRACE && local == 2) {  // hand-off sample: tile 2 woken, read out (no memory access here)
                ns_wake2 = ns_ready;
                ns_read2 = global_timer_ns();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_cta_release(lead_acc_empty + 8 * buf);
            const int row = ti.a_row0 + (int)rank * 128 + quarter * 32 + lane, col0 = ti.tn * BN + half * kCols;
            if (p.gather.n_dst > 0) {
                if constexpr (L::kHasStage && kCols % 64 == 0)
                    store_rows_gather_staged<kCols>(acc, p, ti.a_row0 + (int)rank * 128 + quarter * 32, col0,
                                                    ti.row_end, ti.alpha,
                                                    base + L::kOffStage + (uint32_t)(warp - 2) * L::kStageWarp, lane);
                else
                    store_row_gather<kCols>(acc, p, row, col0, ti.row_end, ti.alpha);
            } else if constexpr (L::kHasStage) {
                if (p.tma_store) {
                    // 16 columns at a time: convert, write this lane's row of the warp's
                    // staging box (32-byte swizzle: the 16-byte halves of rows 4-7 of
                    // each group of 8 swap places, so a warp's writes hit every bank
                    // once), then one TMA store of the 32 x 16 box; the box rows and
                    // columns outside D are clipped by the tensor map
                    const uint32_t my_stage = base + L::kOffStage + (uint32_t)(warp - 2) * L::kStageWarp;
                    const int row0 = ti.a_row0 + (int)rank * 128 + quarter * 32;
                    const uint32_t sw = ((uint32_t)lane >> 2) & 1u;
#pragma unroll
                    for (int c = 0; c < kCols / 16; c++, chunk++) {
                        const uint32_t box = my_stage + (chunk & 1u) * L::kStageBox;
                        if (chunk >= 2) {  // this box's previous store has finished reading it
                            if (lane == 0) bulk_wait_group_read<1>();
                            __syncwarp();
                        }
                        uint32_t w[8];
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            w[i] = pack2(__uint_as_float(acc[c * 16 + 2 * i]) * ti.alpha,
                                         __uint_as_float(acc[c * 16 + 2 * i + 1]) * ti.alpha, F16);
                        const uint32_t rowaddr = box + (uint32_t)lane * 32u;
                        st_shared_v4(rowaddr + 16u * sw, w[0], w[1], w[2], w[3]);
                        st_shared_v4(rowaddr + 16u * (sw ^ 1u), w[4], w[5], w[6], w[7]);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmap_d, box, col0 + c * 16, row0);
                            bulk_commit_group();
                        }
                    }
                } else if (p.epi.plain()) {
                    store_row<kCols, F16>(acc, p, row, col0, ti.row_end, ti.alpha, d_hint, pol_d);
                } else if constexpr (!F16) {
                    store_row_epi_fast<kCols>(acc, p, row, col0, ti.row_end, ti.alpha,
                                              p.epi.bias ? p.epi.bias + (int64_t)ti.group * p.N : nullptr,
                                              row + ti.sf_row_off, tab, guess, gs_ok);
                }
            } else {
                if (p.epi.plain())
                    store_row<kCols, F16>(acc, p, row, col0, ti.row_end, ti.alpha, d_hint, pol_d);
                else if constexpr (!F16)
                    store_row_epi_fast<kCols>(acc, p, row, col0, ti.row_end, ti.alpha,
                                              p.epi.bias ? p.epi.bias + (int64_t)ti.group * p.N : nullptr,
                                              row + ti.sf_row_off, tab, guess, gs_ok);
            }
            if (TRACE && warp == 2 && lane == 0) t_store += clock64() - c_ready;
        }
        if (TRACE && lane == 0 && ns_read2) {  // the last epilogue warp's read-out time of tile 2
            atomicMax(p.trace + blockIdx.x * kTraceSlots + 15, (unsigned long long)ns_read2);
            if (warp == 2) p.trace[blockIdx.x * kTraceSlots + 14] = ns_wake2;
        }
        if (TRACE && warp == 2 && lane == 0) {
            p.trace[blockIdx.x * kTraceSlots + 3] = t_accw;
            p.trace[blockIdx.x * kTraceSlots + 4] = t_store;
        }
        if (p.tma_store && lane == 0) bulk_wait_group<0>();  // stores done before the staging memory goes
        // the peer / multicast stores of this thread are ordered before whatever follows
        // the kernel (the cross-rank barrier that publishes the gathered output)
        if (p.gather.n_dst > 0) __threadfence_system();
        __syncwarp();
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, L::kTmemCols);
    }
    if (TRACE && threadIdx.x == 0) p.trace[blockIdx.x * kTraceSlots + 9] = global_timer_ns();
}

// L2 eviction hints of the pair kernel: 0 none, 1 D stores evict-first, 2 also the A
// and B tile loads evict-last; env NVFP4_PAIR_L2HINT.
static int pair_l2hint() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_PAIR_L2HINT");
        return e ? std::atoi(e) : 0;
    }();
    return v;
}

// Epilogue stores of the pair kernel: through shared memory with TMA (1) or direct
// 32-byte stores from registers (0, the default); env NVFP4_PAIR_TMA_STORE=0|1
// overrides.  Measured at M=N=K=8192: TMA stores 199.5 us, direct stores 198.3 us —
// the epilogue runs in the shadow of the next tile's MMAs either way, and the box
// stores add a shared-memory round trip per 16 columns.
static int pair_tma_store() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_PAIR_TMA_STORE");
        return e ? (std::atoi(e) ? 1 : 0) : 0;
    }();
    return v;
}

// Barrier waits: 0 the suspending try_wait everywhere, 1 polling (test_wait) in the
// MMA thread and the epilogue, 2 also in the producers; env NVFP4_PAIR_SPIN overrides.
static int pair_spin() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_PAIR_SPIN");
        const int x = e ? std::atoi(e) : 1;
        return x < 0 ? 0 : (x > 2 ? 2 : x);
    }();
    return v;
}

// Programmatic dependent launch of the pair kernel (1, the default): its set-up runs
// while the previous kernel in the stream finishes, every global access waits for
// it (griddepcontrol.wait); env NVFP4_PAIR_PDL=0 launches it in plain stream order.
static int pair_pdl() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_PAIR_PDL");
        return e ? (std::atoi(e) ? 1 : 0) : 1;
    }();
    return v;
}

// Tile scheduler of the pair kernel: static persistent (0) or cluster launch control
// (1); env NVFP4_PAIR_SCHED=static|clc overrides.  Measured at M=N=K=8192 on one box:
// static 203.2 us, cluster launch control 208.2 us (MoE grouped: 232 vs 242 us) —
// with uniform tiles the static schedule already balances, and every tile then costs
// the queue hand-off; cluster launch control is kept for uneven or shared-GPU loads.
static int pair_clc() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_PAIR_SCHED");
        if (e && !std::strcmp(e, "clc")) return 1;
        return 0;
    }();
    return v;
}

// Raster group (256-row tile rows sharing a sweep over N); env NVFP4_GROUP_M overrides.
static int pair_group_m() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_GROUP_M");
        int x = e ? std::atoi(e) : 32;
        return x < 1 ? 1 : (x > 1024 ? 1024 : x);
    }();
    return v;
}

// Grouped launches (grp.groups > 0) take M = grp.m_total; A's scale tensor then
// holds ceil(m_total / 128) + groups blocks (every group's scales start on a block),
// B and its scales groups x N rows.
template <int STAGES, int BKB, int BN, bool F16>
static int launch_pair(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                       void *D, int M, int N, int K, cudaStream_t stream, const DeviceInfo &di,
                       unsigned long long *trace, const Epi &epi, const Grouped &grp = Grouped(),
                       const Gather &gat = Gather()) {
    if (epi.q && BN % 128 != 0) return NVFP4_ERR_UNSUPPORTED;  // NVFP4 output wants 64-column aligned halves
    if (F16 && !epi.plain()) return NVFP4_ERR_UNSUPPORTED;     // the fused epilogue writes bf16 / NVFP4
    if (epi.act == kActSwiglu && BN % 256 != 0) return NVFP4_ERR_UNSUPPORTED;  // 128-column halves
    using L = PairLayout<STAGES, BKB, BN>;
#ifdef NVFP4_DIAG
    // the per-CTA cycle trace exists only in the diagnostic library (nvfp4_diag)
    auto kern = trace ? nvfp4_gemm_pair_kernel<STAGES, BKB, BN, F16, true>
                      : nvfp4_gemm_pair_kernel<STAGES, BKB, BN, F16, false>;
#else
    if (trace) return NVFP4_ERR_UNSUPPORTED;
    auto kern = nvfp4_gemm_pair_kernel<STAGES, BKB, BN, F16, false>;
#endif
    static int configured[2][64] = {};
    if (!configured[trace != nullptr][di.device]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDynamicSmem) != cudaSuccess)
            return NVFP4_ERR_CUDA;
        configured[trace != nullptr][di.device] = 1;
    }
    const int G = grp.groups;
    const int64_t b_rows = G > 0 ? (int64_t)G * N : N;
    CUtensorMap ta, tb, tsa, tsb, td;
    std::memset(&td, 0, sizeof(td));
    int st = operand_map(A, M, K, 128, BKB, &ta);
    if (!st) st = operand_map(B, b_rows, K, L::kBRows, BKB, &tb);
    // scale tensors as [bytes/256, 256]: one (128-row block, 64-K group) chunk is two rows
    const uint64_t sfa_blocks = (uint64_t)((M + 127) / 128) + (uint64_t)G;
    const uint64_t sfb_blocks = (uint64_t)((b_rows + 127) / 128);
    const uint64_t sfa_rows = sfa_blocks * (K / 64) * 2;
    const uint64_t sfb_rows = sfb_blocks * (K / 64) * 2;
    if (!st) st = encode_tiled_2d(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, SFA, 256, sfa_rows, 256, 256, 2 * L::kKG,
                                  CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!st) st = encode_tiled_2d(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, SFB, 256, sfb_rows, 256, 256, 2 * L::kKG,
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
    p.num_m_tiles = (M + 255) / 256 + G;  // grouped: an upper bound (group sizes live on the device)
    p.num_n_tiles = (N + BN - 1) / BN;
    p.num_tiles = p.num_m_tiles * p.num_n_tiles;
    p.num_kb = (K + 2 * BKB - 1) / (2 * BKB);
    p.k_groups = K / 64;
    p.vec32_store = ((reinterpret_cast<uintptr_t>(D) & 31u) == 0) && (N % 16 == 0);
    p.trace = trace;
    p.group_m = pair_group_m();
    p.clc = pair_clc();
    p.epi = epi;
    p.grouped = grp;
    // TMA stores of D only for a plain output whose tiles lie inside one matrix (a
    // grouped tile can reach into the next group's rows, which a box store would clip
    // to D's extent but not to the group)
    p.gather = gat;
    p.tma_store = (L::kHasStage && epi.plain() && G == 0 && gat.n_dst == 0 && pair_tma_store()) ? 1 : 0;
    p.l2hint = pair_l2hint();
    p.spin = pair_spin();
    if (p.tma_store && (st = output_map(D, M, N, 32, &td))) return st;
    if ((st = kernel_ctl(&p.ctl))) return st;
    // static: one persistent cluster per SM pair; cluster launch control: one cluster
    // per tile, the running ones cancelling the rest as they finish
    const int pairs = p.clc ? p.num_tiles : std::min(p.num_tiles, di.sm_count / 2);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kPairThreads);
    cfg.dynamicSmemBytes = L::kDynamicSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pair_pdl() ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, ta, tb, tsa, tsb, td, p) != cudaSuccess) return NVFP4_ERR_CUDA;
    count_launch();
    return cuda_status(cudaGetLastError());
}

// Tile and ring shape of the pair kernel (env NVFP4_PAIR_RING overrides):
//   "6x128n192"  256x192 tiles, two TMEM accumulators, 6 slots of 128 bytes of K
//   "5x128"      256x256 tiles, one accumulator, 5 slots of 128 bytes of K
//   "11x64"      256x256 tiles, one accumulator, 11 slots of 64 bytes of K
// Measured at M=N=K=8192: 5x128 spends 268K MMA-thread cycles per CTA pair, 11x64
// 405K — the single issuing thread's fixed cost per slot (wait, fence, two commits)
// outweighs the deeper ring.  6x128n192 (trace: 0.4 % waiting for an accumulator)
// runs 213 us against 5x128's 200 us: the MMA thread spends ~455 cycles per slot
// whatever the tile width, more than a 192-wide slot's 384 cycles of MMA work.  Not
// instruction issue (probe: a scale copy issues in 8 cycles, commits are free);
// the shared-memory traffic per slot (MMA operand reads plus TMA fills, per FLOP
// higher for 192-wide tiles) is the likely limit.
// Writing the scales into TMEM from other warps (tcgen05.st) instead of tcgen05.cp
// was measured 2.4-3x slower: those stores complete only behind the MMAs already
// queued, so the scale path serialises with the tensor pipe.  An L2 prefetch of the
// A/B tiles 4-24 slots ahead of the loads made the GEMM 10 % slower (200 -> 220 us):
// the ring does not stall on L2 misses.
enum PairCfg {
    kCfg5x128 = 0,
    kCfg11x64 = 1,
    kCfg6x128n192 = 2,
    kCfgDefault = kCfg5x128
};
static int pair_cfg() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_PAIR_RING");
        if (e && !std::strcmp(e, "11x64")) return (int)kCfg11x64;
        if (e && !std::strcmp(e, "5x128")) return (int)kCfg5x128;
        if (e && !std::strcmp(e, "6x128n192")) return (int)kCfg6x128n192;
        return (int)kCfgDefault;
    }();
    return v;
}

template <bool F16>
static int launch_pair_cfg(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                           void *D, int M, int N, int K, cudaStream_t stream, const DeviceInfo &di,
                           unsigned long long *trace, const Epi &epi) {
    switch (pair_cfg()) {
        case kCfg11x64:
            return launch_pair<11, 64, 256, F16>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, trace, epi);
        case kCfg6x128n192:
            return launch_pair<6, 128, 192, F16>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, trace, epi);
        default: return launch_pair<5, 128, 256, F16>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, trace, epi);
    }
}

}  // namespace gemm

int gemm_validate(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const void *D, int M,
                  int N, int K);

int pair_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16, const DeviceInfo &di, const Epi &epi) {
    if (f16) return gemm::launch_pair_cfg<true>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, nullptr, epi);
    return gemm::launch_pair_cfg<false>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, nullptr, epi);
}

// Grouped (mixture-of-experts) GEMM on the CTA-pair kernel, bf16 output.
int grouped_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const float *alphas,
                     uint16_t *D, const int *m_offsets, int groups, int m_total, int N, int K, cudaStream_t stream,
                     const Epi &epi) {
    if (!A || !SFA || !B || !SFB || !alphas || (!D && !epi.q) || !m_offsets) return NVFP4_ERR_INVALID;
    if (groups < 1 || groups > gemm::kMaxGroups || m_total < 1 || N < 128 || N % 128 || K < 64 || K % 64)
        return NVFP4_ERR_SHAPE;
    if (!aligned16(A) || !aligned16(SFA) || !aligned16(B) || !aligned16(SFB) || (D && !aligned16(D)) ||
        (reinterpret_cast<uintptr_t>(alphas) & 3u) || (reinterpret_cast<uintptr_t>(m_offsets) & 3u))
        return NVFP4_ERR_ALIGN;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    gemm::Grouped grp;
    grp.m_offsets = m_offsets;
    grp.alphas = alphas;
    grp.groups = groups;
    grp.m_total = m_total;
    return gemm::launch_pair<5, 128, 256, false>(A, SFA, B, SFB, 1.0f, epi.q ? static_cast<void *>(epi.q) : D,
                                                 m_total, N, K, stream, di, nullptr, epi, grp);
}

// Column-parallel GEMM with the all-gather fused into the epilogue (bf16 output):
// D_shard = alpha * A . B_shard^T is stored into the full [M, ld] output of every rank
// at column col_off, through each rank's buffer (dst[0..n_dst)) or one multicast
// address (dst[0], multicast != 0).  The caller orders the ranks afterwards.
int gather_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, int M,
                    int N, int K, const uint64_t *dst, int n_dst, int multicast, int64_t ld, int col_off,
                    cudaStream_t stream) {
    if (!A || !SFA || !B || !SFB || !dst) return NVFP4_ERR_INVALID;
    if (M < 1 || N < 16 || N % 16 || K < 64 || K % 64 || n_dst < 1 || n_dst > gemm::kMaxGatherRanks ||
        (multicast && n_dst != 1) || col_off < 0 || col_off % 16 || ld % 16 || ld < (int64_t)col_off + N)
        return NVFP4_ERR_SHAPE;
    if (!aligned16(A) || !aligned16(SFA) || !aligned16(B) || !aligned16(SFB)) return NVFP4_ERR_ALIGN;
    gemm::Gather g;
    for (int d = 0; d < n_dst; d++) {
        if (!dst[d]) return NVFP4_ERR_INVALID;
        if (dst[d] & 31u) return NVFP4_ERR_ALIGN;
        g.dst[d] = dst[d];
    }
    g.n_dst = n_dst;
    g.multicast = multicast ? 1 : 0;
    g.ld = ld;
    g.col_off = col_off;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    // D is never written through the shard pointer: dst[0] stands in for validation only
    return gemm::launch_pair<5, 128, 256, false>(A, SFA, B, SFB, alpha, reinterpret_cast<void *>(dst[0]), M, N, K,
                                                 stream, di, nullptr, Epi(), gemm::Grouped(), g);
}

#ifdef NVFP4_DIAG
// Pair kernel with the per-CTA cycle trace on (trace: 148 x kTraceSlots u64 on the
// device); diagnostic library only.
int gemm_trace(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D, int M,
               int N, int K, unsigned long long *trace, cudaStream_t stream, const Epi &epi) {
    int st = gemm_validate(A, SFA, B, SFB, D, M, N, K);
    if (st) return st;
    if (!trace) return NVFP4_ERR_INVALID;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    return gemm::launch_pair_cfg<false>(A, SFA, B, SFB, alpha, D, M, N, K, stream, di, trace, epi);
}
#endif

}  // namespace nvfp4
