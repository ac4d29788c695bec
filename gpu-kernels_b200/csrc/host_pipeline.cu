// host_pipeline.cu — nvfp4_gemm_host: the GEMM on HOST buffers, with the PCIe
// copies overlapped with the tensor-core work.
//
// The reference's runner (matmul/sm100_nvfp4/runner.cu:45-59, 78-90) copies all
// operands to the device, runs the GEMM and copies D back, one after the other.
// At M=N=K=8192 the copies (75.5 MB in, 134 MB of bf16 out) take ~20x the GEMM, so
// this entry point cuts D into row strips of up to 1024 rows and pipelines three
// streams:
//   copy-in : A strip 0, the B blocks (2048 rows each), then the other A strips,
//   compute : strip 0 as one GEMM per 2048-column block, as each B block lands (so
//             the download starts after ~14 MB of uploads, not after all of B);
//             every later strip as one full-width GEMM,
//   copy-out: strip 0's blocks as 2-D copies (rows of 4 KB copy at the contiguous
//             rate; 2 KB rows are ~18 % slower), the later strips as contiguous
//             copies of their rows of the row-major result.
// H2D and D2H run on separate copy engines.  Consecutive calls overlap too: a call's
// uploads wait only for the previous call's GEMMs (the operand buffers are free once
// those have run), and D alternates between two device buffers, so the next call's
// uploads and GEMMs proceed while this call's D is still downloading — issued from
// two caller streams in turn, back-to-back calls cost about their download alone.
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace nvfp4 {

int gemm_dispatch(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB, float alpha, void *D,
                  int M, int N, int K, cudaStream_t stream, bool f16);

namespace {

constexpr int kStripRows = 1024;  // rows of a D strip (a multiple of the 256-row tile)
constexpr int kBlockCols = 2048;  // columns of strip 0's blocks (multiple of 256; 4 KB rows of bf16)

struct DeviceBuffers {
    void *mem = nullptr;
    size_t bytes = 0;
    cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
    std::vector<cudaEvent_t> ev;
    cudaEvent_t comp_done = nullptr;     // the previous call's GEMMs have run: operand buffers free
    cudaEvent_t out_done[2] = {};        // each D buffer's last downloads have finished
    int calls = 0;                       // which D buffer the next call uses (calls & 1)
    size_t off_d = 0, d_set = 0;         // the previous call's layout: D buffers' offset and size
    bool ready = false;
};

int setup(DeviceBuffers &b, size_t need, size_t events) {
    if (!b.ready) {
        if (cudaStreamCreateWithFlags(&b.s_in, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&b.s_comp, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&b.s_out, cudaStreamNonBlocking) != cudaSuccess)
            return NVFP4_ERR_CUDA;
        for (cudaEvent_t *e : {&b.comp_done, &b.out_done[0], &b.out_done[1]}) {
            if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return NVFP4_ERR_CUDA;
            if (cudaEventRecord(*e, b.s_out) != cudaSuccess) return NVFP4_ERR_CUDA;
        }
        b.ready = true;
    }
    while (b.ev.size() < events) {
        cudaEvent_t e;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return NVFP4_ERR_CUDA;
        b.ev.push_back(e);
    }
    if (b.bytes < need) {
        if (b.mem) {
            cudaDeviceSynchronize();
            cudaFree(b.mem);
            b.mem = nullptr;
            b.bytes = 0;
        }
        if (cudaMalloc(&b.mem, need) != cudaSuccess) return NVFP4_ERR_CUDA;
        b.bytes = need;
    }
    return NVFP4_OK;
}

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

int gemm_host(const uint8_t *hA, const uint8_t *hSFA, const uint8_t *hB, const uint8_t *hSFB, float alpha,
              uint16_t *hD, int M, int N, int K, cudaStream_t stream) {
    if (!hA || !hSFA || !hB || !hSFB || !hD) return NVFP4_ERR_INVALID;
    if (M < 1 || N < 8 || N % 8 || K < 64 || K % 64) return NVFP4_ERR_SHAPE;
    static std::mutex mu;
    static DeviceBuffers bufs[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4_ERR_CUDA;
    std::lock_guard<std::mutex> lock(mu);  // one pipeline per device at a time
    DeviceBuffers &b = bufs[dev];

    // strips of mb rows, strip 0 in blocks of nb columns: multiples of 256 (CTA-pair
    // tiles, 128-row scale blocks)
    const int mb = std::min(kStripRows, (M + 255) / 256 * 256), nb = std::min(kBlockCols, (N + 255) / 256 * 256);
    const int gm = (M + mb - 1) / mb, gn = (N + nb - 1) / nb;
    const size_t kb2 = (size_t)K / 2, sf_row = (size_t)K / 16;
    const size_t m_pad = (size_t)((M + 127) / 128) * 128, n_pad = (size_t)((N + 127) / 128) * 128;
    const size_t off_a = 0, off_sfa = align256(off_a + (size_t)M * kb2);
    const size_t off_b = align256(off_sfa + m_pad * sf_row), off_sfb = align256(off_b + (size_t)N * kb2);
    const size_t off_d = align256(off_sfb + n_pad * sf_row);
    // one D buffer: strip 0's blocks (each mb x nb, compact), then the row-major rest
    const size_t d_block = align256((size_t)mb * nb * 2);
    const size_t d_set = d_block * gn + align256((size_t)(M - std::min(M, mb)) * N * 2);
    int st = setup(b, off_d + 2 * d_set, 2 * ((size_t)gm + gn) + 2);
    if (st) return st;
    const int set = b.calls & 1;
    uint8_t *base = static_cast<uint8_t *>(b.mem);
    uint8_t *dA = base + off_a, *dSFA = base + off_sfa, *dB = base + off_b, *dSFB = base + off_sfb;
    uint8_t *dD0 = base + off_d + set * d_set;               // strip 0's blocks
    uint8_t *dDr = dD0 + d_block * gn;                       // rows mb..M, row-major

    size_t ev_i = 0;
    cudaEvent_t start = b.ev[ev_i++];
    if ((st = cuda_status(cudaEventRecord(start, stream)))) return st;
    cudaStreamWaitEvent(b.s_in, start, 0);
    cudaStreamWaitEvent(b.s_in, b.comp_done, 0);       // the previous call's GEMMs no longer read A, B
    cudaStreamWaitEvent(b.s_comp, start, 0);
    cudaStreamWaitEvent(b.s_comp, b.out_done[set], 0);  // this D buffer's earlier downloads are done
    if (b.off_d != off_d || b.d_set != d_set) {
        // a new layout: this call's operands or D may cover memory that an earlier
        // call's D still occupies, so its uploads and GEMMs wait for every download
        for (int k = 0; k < 2; k++) {
            cudaStreamWaitEvent(b.s_in, b.out_done[k], 0);
            cudaStreamWaitEvent(b.s_comp, b.out_done[k], 0);
        }
    }
    b.off_d = off_d;
    b.d_set = d_set;
    cudaStreamWaitEvent(b.s_out, start, 0);

    auto upload = [&](uint8_t *d, const uint8_t *h, uint8_t *dsf, const uint8_t *hsf, int r0, int rows, int span,
                      size_t pad) {
        const size_t sf_rows = std::min((size_t)span, pad - (size_t)r0);
        cudaMemcpyAsync(d + (size_t)r0 * kb2, h + (size_t)r0 * kb2, (size_t)rows * kb2, cudaMemcpyHostToDevice,
                        b.s_in);
        cudaMemcpyAsync(dsf + (size_t)r0 * sf_row, hsf + (size_t)r0 * sf_row, sf_rows * sf_row,
                        cudaMemcpyHostToDevice, b.s_in);
        cudaEvent_t e = b.ev[ev_i++];
        cudaEventRecord(e, b.s_in);
        return e;
    };
    auto ready = [&](cudaEvent_t e) { cudaStreamWaitEvent(b.s_comp, e, 0); };
    auto computed = [&]() {
        cudaEvent_t e = b.ev[ev_i++];
        cudaEventRecord(e, b.s_comp);
        cudaStreamWaitEvent(b.s_out, e, 0);
    };

    // strip 0, block by block as the B blocks land
    const int rows0 = std::min(mb, M);
    ready(upload(dA, hA, dSFA, hSFA, 0, rows0, mb, m_pad));
    for (int j = 0; j < gn; j++) {
        const int c0 = j * nb, cols = std::min(nb, N - c0);
        ready(upload(dB, hB, dSFB, hSFB, c0, cols, nb, n_pad));
        uint8_t *dDb = dD0 + d_block * (size_t)j;
        if ((st = gemm_dispatch(dA, dSFA, dB + (size_t)c0 * kb2, dSFB + (size_t)c0 * sf_row, alpha, dDb, rows0, cols,
                                K, b.s_comp, false)))
            return st;
        computed();
        cudaMemcpy2DAsync(reinterpret_cast<uint8_t *>(hD) + (size_t)c0 * 2, (size_t)N * 2, dDb, (size_t)cols * 2,
                          (size_t)cols * 2, rows0, cudaMemcpyDeviceToHost, b.s_out);
    }
    // the other strips, full width: one GEMM and one contiguous download each
    for (int i = 1; i < gm; i++) {
        const int r0 = i * mb, rows = std::min(mb, M - r0);
        ready(upload(dA, hA, dSFA, hSFA, r0, rows, mb, m_pad));
        uint8_t *dDs = dDr + (size_t)(r0 - mb) * N * 2;
        if ((st = gemm_dispatch(dA + (size_t)r0 * kb2, dSFA + (size_t)r0 * sf_row, dB, dSFB, alpha, dDs, rows, N, K,
                                b.s_comp, false)))
            return st;
        computed();
        cudaMemcpyAsync(reinterpret_cast<uint8_t *>(hD) + (size_t)r0 * N * 2, dDs, (size_t)rows * N * 2,
                        cudaMemcpyDeviceToHost, b.s_out);
    }
    cudaEventRecord(b.comp_done, b.s_comp);
    cudaEventRecord(b.out_done[set], b.s_out);
    b.calls++;
    cudaStreamWaitEvent(stream, b.out_done[set], 0);  // the caller's stream now orders after D is on the host
    return cuda_status(cudaGetLastError());
}

}  // namespace nvfp4
