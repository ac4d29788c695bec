// probe.cu — measured tensor-core ceiling for kind::mxf4nvf4 on this GPU.
//
// No FP4 peak is published for this pool's B200s, so the roofline denominator is
// measured here: every SM issues back-to-back tcgen05.mma kind::mxf4nvf4 MMAs on
// operands already resident in shared memory (no HBM/L2 traffic), optionally with
// the per-MMA scale-factor copies (tcgen05.cp) the GEMM kernels issue.  The result
// (FLOP / elapsed device time) is the ceiling the GEMM's roofline.frac is taken
// against, at whatever clock the GPU runs under this load.
//
// modes: 0 single-CTA M=128 N=256, MMA only
//        1 single-CTA, 3 scale copies before each MMA (the GEMM kernels' order)
//        2 CTA pair M=256 N=256, MMA only
//        3 CTA pair, 3 scale copies before each MMA
//        4 CTA pair, the 12 scale copies of a 4-MMA stage issued first, then 4 MMAs
//        5 CTA pair M=256 N=192, 3 scale copies before each MMA
// Issue-cost modes (the iteration is shorter than its tensor work would allow, so
// cycles per iteration measure the issuing thread):
//        6 CTA pair, 3 scale copies per iteration, no MMA
//        7 CTA pair M=256 N=64 MMA only (32 cycles of tensor work each)
//        8 CTA pair N=64 MMA + 2 commits (one per CTA's barrier) per iteration
//        9 CTA pair, 3 scale copies + N=64 MMA + 2 commits per iteration
// Operand-value modes (pseudo-random e2m1 codes and scale codes 0x30..0x3f instead
// of zeros, to see whether the rate depends on the data):
//       10 as 4 (CTA pair, 12 scale copies per 4-MMA stage, then 4 MMAs)
//       11 as 2 (CTA pair, MMA only)
#include "common.cuh"
#include "ptx.cuh"

namespace nvfp4 {

constexpr int kProbeSmem = 64 * 1024;

template <int MODE>
__global__ void __launch_bounds__(128, 1) mma_probe_kernel(int iters, unsigned long long *cycles) {
    constexpr bool kPair = MODE >= 2;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    __shared__ uint32_t tmem_slot;
    __shared__ __align__(8) uint64_t bar;
    __shared__ __align__(8) uint64_t bar2;  // per-iteration commits of modes 8 and 9 (never waited on)
    const int warp = threadIdx.x >> 5;
    // zero operands and scales (modes 0-9), or pseudo-random ones (10, 11)
    constexpr bool kRandom = MODE >= 10;
    for (int i = threadIdx.x * 16; i < kProbeSmem - 1024; i += blockDim.x * 16) {
        uint32_t w[4] = {0, 0, 0, 0};
        if (kRandom) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t h = (uint32_t)(i + 4 * q) * 2654435761u + blockIdx.x * 40503u;
                h ^= h >> 15;
                h *= 2246822519u;
                h ^= h >> 13;
                // scale region (from 48 KB): e4m3 codes 0x30..0x3f; operands: any e2m1 nibbles
                w[q] = i >= 49152 ? (h & 0x0f0f0f0fu) | 0x30303030u : h;
            }
        }
        st_shared_v4(base + i, w[0], w[1], w[2], w[3]);
    }
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        mbar_init(smem_u32(&bar2), 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        if (kPair) {
            tmem_alloc_pair(smem_u32(&tmem_slot), 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(&tmem_slot), 512);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if (kPair) cluster_sync(); else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t sA = base, sB = base + 16384, sSf = base + 49152;
    const bool issuer = kPair ? (cluster_ctarank() == 0) : true;
    if (warp == 0 && issuer && elect_one()) {
        constexpr uint32_t idesc = idesc_mxf4nvf4(kPair ? 256 : 128, MODE == 5 ? 192 : ((MODE >= 7 && MODE <= 9) ? 64 : 256));
        const uint32_t c0 = map_to_cta(smem_u32(&bar2), 0), c1 = map_to_cta(smem_u32(&bar2), 1);
        const unsigned long long t0 = clock64();
        for (int i = 0; i < iters; i++) {
            const int j = i & 3;
            const uint32_t col = tmem + 256 + j * 12;
            const uint64_t ad = smem_desc(sA + j * 32, 16, 1024, 2), bd = smem_desc(sB + j * 32, 16, 1024, 2);
            if constexpr (MODE == 0) {
                mma_mxf4nvf4(tmem, ad, bd, idesc, col, col + 4, i != 0);
            } else if constexpr (MODE == 1) {
                tmem_cp_32x128_x4(col, smem_desc(sSf + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4(col + 4, smem_desc(sSf + 2048 + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4(col + 8, smem_desc(sSf + 4096 + j * 512, 16, 128, 0));
                mma_mxf4nvf4(tmem, ad, bd, idesc, col, col + 4, i != 0);
            } else if constexpr (MODE == 2 || MODE == 11) {
                mma_mxf4nvf4_pair(tmem, ad, bd, idesc, col, col + 4, i != 0);
            } else if constexpr (MODE == 3 || MODE == 5) {
                tmem_cp_32x128_x4_pair(col, smem_desc(sSf + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4_pair(col + 4, smem_desc(sSf + 2048 + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4_pair(col + 8, smem_desc(sSf + 4096 + j * 512, 16, 128, 0));
                mma_mxf4nvf4_pair(tmem, ad, bd, idesc, col, col + 4, i != 0);
            } else if constexpr (MODE == 6) {
                tmem_cp_32x128_x4_pair(col, smem_desc(sSf + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4_pair(col + 4, smem_desc(sSf + 2048 + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4_pair(col + 8, smem_desc(sSf + 4096 + j * 512, 16, 128, 0));
            } else if constexpr (MODE == 7) {
                mma_mxf4nvf4_pair(tmem, ad, bd, idesc, col, col + 4, i != 0);
            } else if constexpr (MODE == 8) {
                mma_mxf4nvf4_pair(tmem, ad, bd, idesc, col, col + 4, i != 0);
                mma_commit_pair(c0);
                mma_commit_pair(c1);
            } else if constexpr (MODE == 9) {
                tmem_cp_32x128_x4_pair(col, smem_desc(sSf + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4_pair(col + 4, smem_desc(sSf + 2048 + j * 512, 16, 128, 0));
                tmem_cp_32x128_x4_pair(col + 8, smem_desc(sSf + 4096 + j * 512, 16, 128, 0));
                mma_mxf4nvf4_pair(tmem, ad, bd, idesc, col, col + 4, i != 0);
                mma_commit_pair(c0);
                mma_commit_pair(c1);
            } else {
                if (j == 0) {
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const uint32_t c = tmem + 256 + q * 12;
                        tmem_cp_32x128_x4_pair(c, smem_desc(sSf + q * 512, 16, 128, 0));
                        tmem_cp_32x128_x4_pair(c + 4, smem_desc(sSf + 2048 + q * 512, 16, 128, 0));
                        tmem_cp_32x128_x4_pair(c + 8, smem_desc(sSf + 4096 + q * 512, 16, 128, 0));
                    }
                }
                mma_mxf4nvf4_pair(tmem, ad, bd, idesc, col, col + 4, i != 0);
            }
        }
        if (kPair) mma_commit_pair(smem_u32(&bar)); else mma_commit(smem_u32(&bar));
        volatile int never = 0;
        wait_parity(smem_u32(&bar), 0, 2000000000ull, &never);
        const unsigned long long t1 = clock64();
        atomicMax(cycles, t1 - t0);
    }
    __syncwarp();
    tc_fence_before();
    if (kPair) cluster_sync(); else __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        if (kPair) tmem_dealloc_pair(tmem, 512); else tmem_dealloc(tmem, 512);
    }
}

template <int MODE>
static int run_probe(int iters, int sms, cudaStream_t s, unsigned long long *cycles) {
    auto kern = mma_probe_kernel<MODE>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem) != cudaSuccess)
        return NVFP4_ERR_CUDA;
    if (MODE >= 2) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(sms / 2 * 2);
        cfg.blockDim = dim3(128);
        cfg.dynamicSmemBytes = kProbeSmem;
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, kern, iters, cycles) != cudaSuccess) return NVFP4_ERR_CUDA;
    } else {
        kern<<<sms, 128, kProbeSmem, s>>>(iters, cycles);
    }
    count_launch();
    return cuda_status(cudaGetLastError());
}

}  // namespace nvfp4

using namespace nvfp4;

// Runs the probe on every SM and returns the achieved dense FP4 rate in TFLOP/s
// (FLOP of all MMAs / elapsed device time measured with CUDA events) and the
// longest per-SM MMA-issue time in cycles.  Synchronous; allocates a few bytes.
extern "C" NVFP4_API int nvfp4_probe_mma_rate(int mode, int iters, double *tflops, double *cycles_per_mma) {
    if (mode < 0 || mode > 11 || iters < 16 || !tflops) return NVFP4_ERR_INVALID;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    unsigned long long *dcyc = nullptr;
    if (cudaMalloc(&dcyc, sizeof(*dcyc)) != cudaSuccess) return NVFP4_ERR_CUDA;
    cudaMemset(dcyc, 0, sizeof(*dcyc));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    auto go = [&](int it) {
        switch (mode) {
            case 0: return run_probe<0>(it, di.sm_count, nullptr, dcyc);
            case 1: return run_probe<1>(it, di.sm_count, nullptr, dcyc);
            case 2: return run_probe<2>(it, di.sm_count, nullptr, dcyc);
            case 3: return run_probe<3>(it, di.sm_count, nullptr, dcyc);
            case 4: return run_probe<4>(it, di.sm_count, nullptr, dcyc);
            case 5: return run_probe<5>(it, di.sm_count, nullptr, dcyc);
            case 6: return run_probe<6>(it, di.sm_count, nullptr, dcyc);
            case 7: return run_probe<7>(it, di.sm_count, nullptr, dcyc);
            case 8: return run_probe<8>(it, di.sm_count, nullptr, dcyc);
            case 9: return run_probe<9>(it, di.sm_count, nullptr, dcyc);
            case 10: return run_probe<10>(it, di.sm_count, nullptr, dcyc);
            default: return run_probe<11>(it, di.sm_count, nullptr, dcyc);
        }
    };
    st = go(iters);  // warm-up (clocks ramp)
    if (!st) {
        cudaMemset(dcyc, 0, sizeof(*dcyc));
        cudaEventRecord(e0);
        st = go(iters);
        cudaEventRecord(e1);
    }
    if (!st && cudaEventSynchronize(e1) != cudaSuccess) st = NVFP4_ERR_CUDA;
    if (!st) {
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        const bool pair = mode >= 2;
        const int ctas = pair ? di.sm_count / 2 * 2 : di.sm_count;
        // per MMA: 2 * M * N * K with M = 256 over a pair (128 per CTA), N = 256 (192 in
        // mode 5, 64 in modes 7-9, no MMA in mode 6), K = 64
        const int n = mode == 5 ? 192 : ((mode >= 7 && mode <= 9) ? 64 : (mode == 6 ? 0 : 256));
        const double flop = (double)ctas * iters * 2.0 * 128 * n * 64;
        *tflops = flop / (ms * 1e-3) / 1e12;
        unsigned long long cyc = 0;
        cudaMemcpy(&cyc, dcyc, sizeof(cyc), cudaMemcpyDeviceToHost);
        if (cycles_per_mma) *cycles_per_mma = (double)cyc / iters;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(dcyc);
    return st;
}
