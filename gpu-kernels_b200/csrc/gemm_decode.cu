// gemm_decode.cu — stream-K, swap-AB NVFP4 GEMM for skinny M (decode shapes).
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
//
// This file holds the host-side dispatch; the kernel is in gemm_decode.cuh and its
// instantiations in decode_inst.cu.
#include <mutex>

#include "gemm_decode.cuh"

namespace nvfp4 {
namespace decode {

int launch_for(int rows, bool grouped, const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
               float alpha, uint16_t *D, int M, int N, int K, void *ws, cudaStream_t stream, const DeviceInfo &di,
               const Epi &epi, unsigned long long *trace, const int *m_offsets, const float *alphas, int groups) {
#define NVFP4_DECODE_CASE(MP)                                                                                      \
    case MP:                                                                                                       \
        return grouped ? launch_mpad<MP, true>(A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, epi, trace,     \
                                               m_offsets, alphas, groups)                                         \
                       : launch_mpad<MP, false>(A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, epi, trace,    \
                                                m_offsets, alphas, groups);
    switch (mpad_for(rows)) {
        NVFP4_DECODE_CASE(8)
        NVFP4_DECODE_CASE(16)
        NVFP4_DECODE_CASE(32)
        NVFP4_DECODE_CASE(64)
        NVFP4_DECODE_CASE(128)
        default: return NVFP4_ERR_SHAPE;
    }
#undef NVFP4_DECODE_CASE
}

}  // namespace decode

int gemm_validate(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const void *D, int M,
                  int N, int K);

bool decode_tiles_fit(int N, int groups) { return decode::tiles_fit(N, groups); }

size_t decode_workspace_bytes(int M, int N) {
    DeviceInfo di;
    if (device_info(&di)) return 0;
    return decode::workspace_bytes(M, N, di.sm_count);
}

// Decode GEMM with an optional fused epilogue; with NVFP4 output (epi.q) D is not
// written and may be null.
int decode_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                    uint16_t *D, int M, int N, int K, void *ws, size_t ws_bytes, cudaStream_t stream,
                    const Epi &epi) {
    int st = gemm_validate(A, SFA, B, SFB, epi.q ? static_cast<const void *>(epi.q) : D, M, N, K);
    if (st) return st;
    if (M > 128 || !decode::tiles_fit(N)) return NVFP4_ERR_SHAPE;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    if (!ws || ws_bytes < decode::workspace_bytes(M, N, di.sm_count) ||
        (reinterpret_cast<uintptr_t>(ws) & 255u))
        return NVFP4_ERR_WORKSPACE;
    return decode::launch_for(M, false, A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, epi, nullptr, nullptr,
                              nullptr, 0);
}

size_t decode_grouped_workspace_bytes(int m_total, int N, int groups) {
    DeviceInfo di;
    if (device_info(&di)) return 0;
    return decode::workspace_bytes(m_total, N, di.sm_count, groups);
}

// Grouped (mixture-of-experts) GEMM for m_total <= 128 rows in all: the swap-AB
// stream-K kernel over (active expert, 128-row weight tile) tiles, reading only the
// weights of experts that have rows.  Same arguments as the CTA-pair grouped GEMM plus
// the split-K workspace (decode_grouped_workspace_bytes, zero-filled once).
int decode_grouped_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                            const float *alphas, uint16_t *D, const int *m_offsets, int groups, int m_total, int N,
                            int K, void *ws, size_t ws_bytes, cudaStream_t stream, const Epi &epi) {
    if (!A || !SFA || !B || !SFB || !alphas || (!D && !epi.q) || !m_offsets) return NVFP4_ERR_INVALID;
    if (groups < 1 || groups > gemm::kMaxGroups || m_total < 1 || m_total > 128 || N < 128 || N % 128 || K < 64 ||
        K % 64 || !decode::tiles_fit(N, groups))
        return NVFP4_ERR_SHAPE;
    if (!aligned16(A) || !aligned16(SFA) || !aligned16(B) || !aligned16(SFB) || (D && !aligned16(D)) ||
        (reinterpret_cast<uintptr_t>(alphas) & 3u) || (reinterpret_cast<uintptr_t>(m_offsets) & 3u))
        return NVFP4_ERR_ALIGN;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    if (!ws || ws_bytes < decode::workspace_bytes(m_total, N, di.sm_count, groups) ||
        (reinterpret_cast<uintptr_t>(ws) & 255u))
        return NVFP4_ERR_WORKSPACE;
    return decode::launch_for(m_total, true, A, SFA, B, SFB, 1.0f, D, m_total, N, K, ws, stream, di, epi, nullptr,
                              m_offsets, alphas, groups);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the decode GEMM.
//
// Some callers cannot let a kernel library allocate device memory: hosts that own
// all device memory themselves (memory-budgeted inference servers, plugin
// interfaces of other frameworks that hand a library only its inputs and outputs),
// and latency-critical loops in which a cudaMalloc — which may synchronise the
// whole device — is not acceptable.  For them the split-K scratch (per-tile arrival
// counters and fp32 partial tiles) lives in this fixed, file-scope device array
// instead of a caller- or library-allocated workspace.  Every GPU that loads the
// library holds these kNoAllocScratchBytes until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB: M <= 16 on a 148-SM B200
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

// Device address of g_decode_scratch on the current device, looked up once per
// device (host code must not use the symbol itself as a device pointer).  The
// arrival counters must read zero when a call starts: the array starts zeroed and
// every call that completes leaves its counters at zero, so they are cleared (a
// memset on `stream`, not an allocation) only when the address is first looked up
// and again after nvfp4_device_status has reported a device-side timeout, which can
// leave counters set.
static int noalloc_scratch(void **out, cudaStream_t stream) {
    static std::mutex mu;
    static void *addr[64] = {};
    static uint64_t cleared_at[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4_ERR_CUDA;
    std::lock_guard<std::mutex> lock(mu);
    const uint64_t epoch = timeout_epoch(dev);
    if (!addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) return NVFP4_ERR_CUDA;
        if (cudaMemsetAsync(p, 0, decode::kCounterBytes, stream) != cudaSuccess) return NVFP4_ERR_CUDA;
        addr[dev] = p;
        cleared_at[dev] = epoch;
    } else if (cleared_at[dev] != epoch) {
        if (cudaMemsetAsync(addr[dev], 0, decode::kCounterBytes, stream) != cudaSuccess) return NVFP4_ERR_CUDA;
        cleared_at[dev] = epoch;
    }
    *out = addr[dev];
    return NVFP4_OK;
}

int decode_noalloc_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                            uint16_t *D, int M, int N, int K, cudaStream_t stream) {
    int st = gemm_validate(A, SFA, B, SFB, D, M, N, K);
    if (st) return st;
    if (M > 128 || !decode::tiles_fit(N)) return NVFP4_ERR_SHAPE;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const size_t need = decode::workspace_bytes(M, N, di.sm_count);
    if (need > kNoAllocScratchBytes) return NVFP4_ERR_WORKSPACE;  // problem too large for the fixed scratch
    void *ws = nullptr;
    if ((st = noalloc_scratch(&ws, stream))) return st;
    return decode::launch_for(M, false, A, SFA, B, SFB, alpha, D, M, N, K, ws, stream, di, Epi(), nullptr, nullptr,
                              nullptr, 0);
}

}  // namespace nvfp4
