// capi.cu — the extern "C" GEMM entry points of libnvfp4_b200 (declared in
// include/nvfp4_b200.h).  Argument checking lives in gemm_validate; kernels in
// gemm.cu, quantize.cu; shared plumbing in runtime.cu.
#include <atomic>
#include <cstdlib>
#include <map>
#include <tuple>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "epilogue.cuh"

namespace nvfp4 {
int gemm_dispatch_epi(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                      int M, int N, int K, cudaStream_t stream, bool f16, const Epi &epi);
int sf_pad_zero(uint8_t *SF, int M, int K, cudaStream_t s, const DeviceInfo &di);
int gather_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, int M,
                    int N, int K, const uint64_t *dst, int n_dst, int multicast, int64_t ld, int col_off,
                    cudaStream_t stream);
size_t decode_grouped_workspace_bytes(int m_total, int N, int groups);
int decode_grouped_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                            const float *alphas, uint16_t *D, const int *m_offsets, int groups, int m_total, int N,
                            int K, void *ws, size_t ws_bytes, cudaStream_t stream, const Epi &epi);
int grouped_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const float *alphas,
                     uint16_t *D, const int *m_offsets, int groups, int m_total, int N, int K, cudaStream_t stream,
                     const Epi &epi);
int grouped_sf_pad_zero(uint8_t *SF, const int *m_offsets, int groups, int m_total, int K, cudaStream_t s);
size_t quantize_dynamic_workspace_bytes();
int quantize_dynamic_check(const uint16_t *X, const uint8_t *Q, const uint8_t *SF, const float *amax_out,
                           const float *gs_out, int M, int K);
int quantize_dynamic_dispatch(const uint16_t *X, uint8_t *Q, uint8_t *SF, float *amax_out, float *gs_out, int M,
                              int K, void *ws, size_t ws_bytes, cudaStream_t s);
int gemm_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16);
size_t decode_workspace_bytes(int M, int N);
bool decode_tiles_fit(int N, int groups);
int decode_noalloc_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                            uint16_t *D, int M, int N, int K, cudaStream_t stream);
int gemm_host(const uint8_t *hA, const uint8_t *hSFA, const uint8_t *hB, const uint8_t *hSFB, float alpha,
              uint16_t *hD, int M, int N, int K, cudaStream_t stream);
int gemm_validate(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const void *D, int M,
                  int N, int K);
int decode_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                    uint16_t *D, int M, int N, int K, void *ws, size_t ws_bytes, cudaStream_t stream,
                    const Epi &epi = Epi());
}  // namespace nvfp4

using namespace nvfp4;

static std::atomic<int> g_last_status{NVFP4_OK};

// Largest M routed to the split-K decode kernel by nvfp4_gemm (env override
// NVFP4_DECODE_MAX_M, 0 disables the decode path).
static int decode_max_m() {
    static int v = [] {
        const char *e = std::getenv("NVFP4_DECODE_MAX_M");
        int x = e ? std::atoi(e) : 128;
        return x < 0 ? 0 : (x > 128 ? 128 : x);
    }();
    return v;
}

// nvfp4_gemm's kernel for M <= decode_max_m(): the split-K decode kernel (128-row
// weight tiles spread over every SM), or the persistent single-CTA kernel (one 128 x
// 256 tile per 256 weight rows: the activations are read once per 256 weight rows
// instead of once per 128, and no split-K partials are written).  The second wins
// once the activations are a sizeable share of each k-block and there are enough
// 256-row tiles to keep most SMs streaming.  Measured (CUDA-graph replay, us, decode
// against persistent): N=28672 K=8192 (112 tiles) M=32 26.1/25.5, M=64 28.6/26.0,
// M=128 31.1/26.8, M=16 25.5/29.6; N=57344 K=4096 (224) M=32 29.6/28.6, M=128 50.1/29.5;
// N=20480 K=8192 (80) M=32 20.0/21.2, M=64 23.7/21.6; N=14336 K=4096 (56) M=32
// 13.3/11.6; N=8192 (32 tiles) decode always, 26.8-36.8 against 49.7-50.8.
static bool use_decode(int M, int N, int K, const Epi &e) {
    if (M > decode_max_m() || !decode_tiles_fit(N, 1)) return false;
    if (e.act == kActSwiglu) return true;  // the single-CTA epilogue has no SwiGLU
    const int tiles = (N + 255) / 256;
    if (tiles >= 48 && (M >= 64 || (M >= 32 && (tiles >= 100 || K <= 4096)))) return false;
    return true;
}

// nvfp4_gemm's own decode workspace: one zero-initialised buffer per (device,
// stream), grown on demand and kept for the life of the process.  Calls on the
// same stream are ordered, so they may share it.  Kernels leave its counters at
// zero, except one that timed out: after nvfp4_device_status has reported a timeout
// on the device the buffer is cleared again before its next use.
// kind separates users whose workspace contents must not meet (0: decode split-K
// counters and partials, 1: the dynamic quantizer's barrier and amax partials).
struct Workspace {
    void *ptr = nullptr;
    size_t bytes = 0;
    uint64_t epoch = 0;  // timeout_epoch() when it was last cleared
};

static int internal_workspace(size_t need, cudaStream_t stream, void **ws, size_t *bytes, int kind = 0) {
    static std::mutex mu;
    static std::map<std::tuple<int, cudaStream_t, int>, Workspace> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NVFP4_ERR_CUDA;
    if (!need) return NVFP4_ERR_CUDA;
    std::lock_guard<std::mutex> lock(mu);
    Workspace &slot = cache[{dev, stream, kind}];
    const uint64_t epoch = timeout_epoch(dev);
    if (slot.bytes < need) {
        if (slot.ptr) {
            cudaStreamSynchronize(stream);
            cudaFree(slot.ptr);
            slot = Workspace();
        }
        void *p = nullptr;
        if (cudaMalloc(&p, need) != cudaSuccess) return NVFP4_ERR_CUDA;
        if (cudaMemsetAsync(p, 0, need, stream) != cudaSuccess) {
            cudaFree(p);
            return NVFP4_ERR_CUDA;
        }
        slot.ptr = p;
        slot.bytes = need;
        slot.epoch = epoch;
    } else if (slot.epoch != epoch) {  // a timeout since the last clear: counters may be left set
        if (cudaMemsetAsync(slot.ptr, 0, slot.bytes, stream) != cudaSuccess) return NVFP4_ERR_CUDA;
        slot.epoch = epoch;
    }
    *ws = slot.ptr;
    *bytes = slot.bytes;
    return NVFP4_OK;
}

extern "C" {

int nvfp4_gemm(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, uint16_t *D,
               int M, int N, int K, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = gemm_validate(A, SFA, B, SFB, D, M, N, K);
    if (st) return st;
    if (use_decode(M, N, K, Epi())) {
        void *ws = nullptr;
        size_t bytes = 0;
        st = internal_workspace(decode_workspace_bytes(M, N), s, &ws, &bytes);
        if (st) return st;
        return decode_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, ws, bytes, s);
    }
    return gemm_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, s, false);
}

}  // extern "C"

// Columns of the epilogue's output for a GEMM of N columns (SwiGLU halves them).
static int epi_out_cols(const Epi &e, int N) { return e.act == NVFP4_ACT_SWIGLU ? N / 2 : N; }

// The C epilogue description as the kernels' Epi, with its argument checks.
int epilogue_from(const nvfp4_epilogue *epi, int N, Epi *out) {
    Epi e;
    e.bias = epi->bias;
    e.act = epi->activation;
    e.q = epi->q_out;
    e.sf = epi->sf_out;
    e.gs = epi->out_global_scale;
    if (e.act < NVFP4_ACT_NONE || e.act > NVFP4_ACT_SWIGLU) return NVFP4_ERR_INVALID;
    if (e.act == NVFP4_ACT_SWIGLU && N % 128) return NVFP4_ERR_SHAPE;  // whole 32-column gate / up blocks per warp
    if (e.bias && !aligned16(e.bias)) return NVFP4_ERR_ALIGN;
    if (e.q) {
        if (!e.sf || !e.gs) return NVFP4_ERR_INVALID;
        if (N % 64) return NVFP4_ERR_SHAPE;
        if ((reinterpret_cast<uintptr_t>(e.q) & 31u) || (reinterpret_cast<uintptr_t>(e.sf) & 3u) ||
            (reinterpret_cast<uintptr_t>(e.gs) & 3u))
            return NVFP4_ERR_ALIGN;
    }
    *out = e;
    return NVFP4_OK;
}

extern "C" {

int nvfp4_gemm_epilogue(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                        uint16_t *D, int M, int N, int K, const nvfp4_epilogue *epi, void *stream) {
    if (!epi) return nvfp4_gemm(A, SFA, B, SFB, alpha, D, M, N, K, stream);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Epi e;
    int st = epilogue_from(epi, N, &e);
    if (st) return st;
    st = gemm_validate(A, SFA, B, SFB, e.q ? static_cast<const void *>(e.q) : D, M, N, K);
    if (st) return st;
    if (use_decode(M, N, K, e)) {
        void *ws = nullptr;
        size_t bytes = 0;
        if ((st = internal_workspace(decode_workspace_bytes(M, N), s, &ws, &bytes))) return st;
        st = decode_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, ws, bytes, s, e);
    } else {
        st = gemm_dispatch_epi(A, SFA, B, SFB, alpha, D, M, N, K, s, false, e);
    }
    if (st || !e.q) return st;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    return sf_pad_zero(e.sf, M, epi_out_cols(e, N), s, di);  // the output's scale padding rows
}

}  // extern "C"

// Grouped GEMM with an optional fused epilogue (bias rows per group).  At most 128
// rows in all (decode): the stream-K kernel that reads only the active experts'
// weights; otherwise the CTA-pair kernel's grouped scheduler.
static int gemm_grouped_epi(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                            const float *alpha, uint16_t *D, const int32_t *m_offsets, int groups, int m_total, int N,
                            int K, cudaStream_t s, const Epi &e) {
    if (m_total >= 1 && m_total <= decode_max_m() && groups >= 1 && groups <= 256 && N >= 128 && N % 128 == 0 &&
        decode_tiles_fit(N, groups)) {
        void *ws = nullptr;
        size_t bytes = 0;
        int st = internal_workspace(decode_grouped_workspace_bytes(m_total, N, groups), s, &ws, &bytes);
        if (st) return st;
        return decode_grouped_dispatch(A, SFA, B, SFB, alpha, D, m_offsets, groups, m_total, N, K, ws, bytes, s, e);
    }
    return grouped_dispatch(A, SFA, B, SFB, alpha, D, m_offsets, groups, m_total, N, K, s, e);
}

extern "C" {

int nvfp4_quantize_dynamic(const uint16_t *X, uint8_t *Q, uint8_t *SF, float *amax_out, float *gs_out, int M, int K,
                           void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = quantize_dynamic_check(X, Q, SF, amax_out, gs_out, M, K);
    if (st) return st;
    void *ws = nullptr;
    size_t bytes = 0;
    st = internal_workspace(quantize_dynamic_workspace_bytes(), s, &ws, &bytes, 1);
    if (st) return st;
    return quantize_dynamic_dispatch(X, Q, SF, amax_out, gs_out, M, K, ws, bytes, s);
}

int nvfp4_gemm_grouped(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, const float *alpha,
                       uint16_t *D, const int32_t *m_offsets, int groups, int m_total, int N, int K, void *stream) {
    return gemm_grouped_epi(A, SFA, B, SFB, alpha, D, m_offsets, groups, m_total, N, K,
                            static_cast<cudaStream_t>(stream), Epi());
}

int nvfp4_gemm_grouped_epilogue(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                                const float *alpha, uint16_t *D, const int32_t *m_offsets, int groups, int m_total,
                                int N, int K, const nvfp4_epilogue *epi, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Epi e;
    if (epi) {
        int st = epilogue_from(epi, N, &e);
        if (st) return st;
    }
    int st = gemm_grouped_epi(A, SFA, B, SFB, alpha, D, m_offsets, groups, m_total, N, K, s, e);
    if (st || !e.q) return st;
    return grouped_sf_pad_zero(e.sf, m_offsets, groups, m_total, epi_out_cols(e, N), s);  // padding rows
}

int nvfp4_gemm_gather(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, int M,
                      int N, int K, const uint64_t *dst, int n_dst, int multicast, int64_t ld, int col_off,
                      void *stream) {
    return gather_dispatch(A, SFA, B, SFB, alpha, M, N, K, dst, n_dst, multicast, ld, col_off,
                           static_cast<cudaStream_t>(stream));
}

int nvfp4_gemm_persistent(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                          uint16_t *D, int M, int N, int K, void *stream) {
    return gemm_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, static_cast<cudaStream_t>(stream), false);
}

size_t nvfp4_gemm_decode_workspace_size(int M, int N) {
    if (M < 1 || M > 128 || N < 1 || !decode_tiles_fit(N, 1)) return 0;
    return decode_workspace_bytes(M, N);
}

int nvfp4_gemm_decode(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                      uint16_t *D, int M, int N, int K, void *workspace, size_t workspace_bytes, void *stream) {
    return decode_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

int nvfp4_gemm_f16(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha,
                   uint16_t *D, int M, int N, int K, void *stream) {
    return gemm_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, static_cast<cudaStream_t>(stream), true);
}

// Reference signature (matmul/sm100_nvfp4/block_scaled_nvfp4.cuh:15-16): note the
// argument order c, sfa, sfb, a, b.
void matmul_nvfp4_b200(void *c, const uint8_t *sfa, const uint8_t *sfb, const uint8_t *a, const uint8_t *b, int M,
                       int N, int K) {
    g_last_status.store(gemm_dispatch(a, sfa, b, sfb, 1.0f, c, M, N, K, nullptr, true));
}

int nvfp4_last_status(void) { return g_last_status.load(); }

int nvfp4_gemm_decode_noalloc(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                              float alpha, uint16_t *D, int M, int N, int K, void *stream) {
    return decode_noalloc_dispatch(A, SFA, B, SFB, alpha, D, M, N, K, static_cast<cudaStream_t>(stream));
}

int nvfp4_gemm_host(const uint8_t *hA, const uint8_t *hSFA, const uint8_t *hB, const uint8_t *hSFB, float alpha,
                    uint16_t *hD, int M, int N, int K, void *stream) {
    return gemm_host(hA, hSFA, hB, hSFB, alpha, hD, M, N, K, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
