// quantize.cu — bf16 -> NVFP4 quantizer and tensor amax (HBM-bound streaming kernels).
//
// The reference has no quantizer (its operands are random codes,
// matmul/sm100_nvfp4/main.py:9-23); the specification it must meet bit-for-bit
// is the CPU oracle's (oracle/nvfp4_oracle.c, nvfp4o_quantize):
//   sf = e4m3_rn_sat((amax/6)/gs), inv = 1/(float(sf)*gs) (0 if that is 0),
//   q  = e2m1_rn_sat(x*inv), each fp32 step one IEEE round-to-nearest op
//   (a gs outside [2^-100, FLT_MAX] gives sf = 0, inv = 0).
//
// Work split: a lane owns one 16-element scale block (one 32-byte load, 8 bytes of
// codes out); four lanes form one 64-element k-group of one row, whose 4 scale
// bytes are contiguous in the blocked layout and leave as one 32-bit store.  A warp
// reads 1 KB contiguous and writes 256 contiguous bytes of codes per step.  The
// kernel is instruction-bound before it is HBM-bound (IEEE divisions), so the
// per-block reciprocal comes from a 256-entry table.
#include "common.cuh"
#include "grouped.cuh"
#include "ptx.cuh"
#include "quant_common.cuh"

namespace nvfp4 {

__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

constexpr int kQuantUnroll = 2;

__device__ __forceinline__ void ld_stream_v8(const void *p, uint32_t (&w)[8]) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
                 : "l"(p));
}

// X: [M, K] bf16, Q: [M, K/2], SF: blocked [pad128(M), K/16].  n_blocks = M*K/16.
// A lane owns one 16-element scale block (one 32-byte load, one 8-byte store of
// codes); four consecutive lanes own one 64-element k-group, whose 4 scale bytes
// are contiguous in the blocked layout and leave as one 32-bit store.  The
// reciprocal 1/(float(sf)*gs) takes only 256 values per launch, so each CTA
// tabulates it once in shared memory with the same IEEE operations.
// The per-block loop shared by quantize_kernel and quantize_dynamic_kernel: blocks
// g, g + stride, ... of X (one per lane), inv_table the 256 reciprocals of gs.
__device__ __forceinline__ void quantize_blocks(const __nv_bfloat16 *__restrict__ X, uint8_t *__restrict__ Q,
                                                uint8_t *__restrict__ SF, float gs, bool gs_ok,
                                                const float *inv_table, int64_t n_blocks, int64_t K) {
    const int lane = threadIdx.x & 31;
    const int64_t rest_k = K >> 6;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // Row and block-in-row of each of this lane's blocks, kept as running values: the
    // lane's blocks advance by a fixed step, so a division happens once per lane, not
    // once per block (a 64-bit division was a large share of the loop's instructions).
    const int per_row = (int)(K >> 4);
    const int64_t step = stride * kQuantUnroll;
    const int step_rows = (int)(step / per_row), step_rem = (int)(step % per_row);
    int row[kQuantUnroll], col[kQuantUnroll];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; u++) {
        const int64_t gi = g + u * stride;
        row[u] = (int)(gi / per_row);
        col[u] = (int)(gi - (int64_t)row[u] * per_row);
    }
    // The trip count is warp-uniform: every warp covers 32 consecutive blocks and
    // n_blocks % 4 == 0 (K % 64 == 0), so whole 4-lane k-groups are active or not.
    for (; g - lane < n_blocks; g += step) {
        uint32_t raw[kQuantUnroll][8];
#pragma unroll
        for (int u = 0; u < kQuantUnroll; u++) {
            const int64_t gi = g + u * stride;
            if (gi < n_blocks) {
                ld_stream_v8(X + gi * 16, raw[u]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) raw[u][i] = 0;
            }
        }
#pragma unroll
        for (int u = 0; u < kQuantUnroll; u++) {
            const int64_t gi = g + u * stride;
            float v[16];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                v[2 * i] = __uint_as_float(raw[u][i] << 16);
                v[2 * i + 1] = __uint_as_float(raw[u][i] & 0xFFFF0000u);
            }
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(v[i]));
            const uint32_t code = block_scale_code(amax, gs, gs_ok);
            uint32_t lo, hi;
            block_codes(v, inv_table[code], lo, hi);
            // gather the 4 scale codes of this lane's k-group into its first lane
            const uint32_t c1 = __shfl_down_sync(0xffffffffu, code, 1);
            const uint32_t c2 = __shfl_down_sync(0xffffffffu, code, 2);
            const uint32_t c3 = __shfl_down_sync(0xffffffffu, code, 3);
            if (gi < n_blocks) {
                *reinterpret_cast<uint2 *>(Q + gi * 8) = make_uint2(lo, hi);
                if ((lane & 3) == 0)  // first block of the k-group
                    *reinterpret_cast<uint32_t *>(SF + sf_group_offset(row[u], col[u] >> 2, rest_k)) =
                        code | (c1 << 8) | (c2 << 16) | (c3 << 24);
            }
        }
#pragma unroll
        for (int u = 0; u < kQuantUnroll; u++) {
            row[u] += step_rows;
            col[u] += step_rem;
            if (col[u] >= per_row) {
                col[u] -= per_row;
                row[u]++;
            }
        }
    }
}

// 5 CTAs (40 warps) per SM: the register bound keeps the loop at 48 registers.
__global__ void __launch_bounds__(256, 5)
    quantize_kernel(const __nv_bfloat16 *__restrict__ X, uint8_t *__restrict__ Q, uint8_t *__restrict__ SF,
                    const float *__restrict__ gs_ptr, int64_t n_blocks, int64_t K) {
    __shared__ float inv_table[256];
    grid_dependency_wait();    // X and gs may come from the previous kernel in the stream
    grid_launch_dependents();  // the next kernel may be placed as this one's CTAs finish
    const float gs = *gs_ptr;
    const bool gs_ok = gs_usable(gs);
    inv_table[threadIdx.x] = block_inverse(threadIdx.x, gs, gs_ok);  // blockDim.x == 256
    __syncthreads();
    quantize_blocks(X, Q, SF, gs, gs_ok, inv_table, n_blocks, K);
}

// amax, global scale and quantization in one cooperative launch (every CTA resident):
// each CTA's amax of its blocks goes to partials[blockIdx.x]; a grid barrier (arrival
// counter bar[0], exit counter bar[1], both back at zero when the kernel ends) orders
// them before every CTA reduces all partials to the same amax and gs = amax / 2688
// (the global_scale_kernel's operation), then quantizes its blocks — X, read once
// from HBM in the first pass, is now mostly in L2.  Same outputs as
// nvfp4_global_scale followed by nvfp4_quantize.  A barrier wait that outlasts the
// timeout records it in the status word and the CTA returns.
__global__ void __launch_bounds__(256) quantize_dynamic_kernel(const __nv_bfloat16 *__restrict__ X,
                                                               uint8_t *__restrict__ Q, uint8_t *__restrict__ SF,
                                                               float *amax_out, float *gs_out, unsigned int *bar,
                                                               float *partials, int64_t n_blocks, int64_t K,
                                                               KernelCtl ctl) {
    __shared__ float inv_table[256];
    __shared__ float wmax[8];
    __shared__ int abort_cta;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    float m = 0.0f;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n_blocks; g += stride) {
        uint32_t w[8];
        ld_stream_v8(X + g * 16, w);
#pragma unroll
        for (int i = 0; i < 8; i++)
            m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[i] << 16)), fabsf(__uint_as_float(w[i] & 0xFFFF0000u))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, wmax[i]);
        __stcg(partials + blockIdx.x, m);
        __threadfence();
        atomicAdd(bar, 1u);
        // every CTA is resident (cooperative launch), so the count reaches the grid soon
        const uint64_t t0 = global_timer_ns();
        int ok = 1;
        while (ld_acquire_gpu_u32(bar) < gridDim.x) {
            if (global_timer_ns() - t0 > ctl.wait_timeout_ns) {
                atomicOr(ctl.status, kDevTimeout);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
        abort_cta = !ok;
        if (ok && atomicAdd(bar + 1, 1u) == gridDim.x - 1) {  // the last CTA past the barrier resets it
            bar[0] = 0;
            bar[1] = 0;
        }
    }
    __syncthreads();
    if (abort_cta) return;
    m = 0.0f;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) m = fmaxf(m, __ldcg(partials + i));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();  // wmax is reused
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    m = wmax[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, wmax[i]);
    const float gs = __fdiv_rn(m, 2688.0f);  // amax / (6 * 448), as global_scale_kernel
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (amax_out) *amax_out = m;
        if (gs_out) *gs_out = gs;
    }
    const bool gs_ok = gs_usable(gs);
    inv_table[threadIdx.x] = block_inverse(threadIdx.x, gs, gs_ok);  // blockDim.x == 256
    __syncthreads();
    quantize_blocks(X, Q, SF, gs, gs_ok, inv_table, n_blocks, K);
}

// Grouped quantizer: the same per-block arithmetic over a stacked [m_total, K]
// matrix whose row groups (grouped.cuh) each get their own blocked scale tensor.
// Codes keep the stacked row order; rows outside every group get codes but no
// scales.  Group tables are built per CTA in shared memory (G <= 256).
constexpr int kQuantMaxGroups = 256;
__global__ void __launch_bounds__(256) quantize_grouped_kernel(const __nv_bfloat16 *__restrict__ X,
                                                               uint8_t *__restrict__ Q, uint8_t *__restrict__ SF,
                                                               const float *__restrict__ gs_ptr,
                                                               const int *__restrict__ m_offsets, int G,
                                                               int m_total, int64_t K) {
    __shared__ float inv_table[256];
    __shared__ int g_r0[kQuantMaxGroups], g_r1[kQuantMaxGroups], g_b0[kQuantMaxGroups + 1];
    const float gs = *gs_ptr;
    const bool gs_ok = gs_usable(gs);
    inv_table[threadIdx.x] = block_inverse(threadIdx.x, gs, gs_ok);  // blockDim.x == 256
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) build_group_tables(m_offsets, G, m_total, 0, lane, g_r0, g_r1, g_b0, nullptr);
    __syncthreads();
    const int64_t rest_k = K >> 6;
    const int64_t n_blocks = (int64_t)m_total * K / 16;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g - lane < n_blocks; g += stride) {
        uint32_t raw[8];
        if (g < n_blocks) {
            ld_stream_v8(X + g * 16, raw);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) raw[i] = 0;
        }
        float v[16];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            v[2 * i] = __uint_as_float(raw[i] << 16);
            v[2 * i + 1] = __uint_as_float(raw[i] & 0xFFFF0000u);
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(v[i]));
        const uint32_t code = block_scale_code(amax, gs, gs_ok);
        uint32_t lo, hi;
        block_codes(v, inv_table[code], lo, hi);
        const uint32_t c1 = __shfl_down_sync(0xffffffffu, code, 1);
        const uint32_t c2 = __shfl_down_sync(0xffffffffu, code, 2);
        const uint32_t c3 = __shfl_down_sync(0xffffffffu, code, 3);
        if (g < n_blocks) {
            *reinterpret_cast<uint2 *>(Q + g * 8) = make_uint2(lo, hi);
            if ((lane & 3) == 0) {
                const int64_t e = g * 16;
                const int r = (int)(e / K);
                const int64_t kg = (e - (int64_t)r * K) >> 6;
                const int gr = last_group_at_or_before(g_r0, G, r);
                if (r >= g_r0[gr] && r < g_r1[gr]) {
                    const int local = r - g_r0[gr];
                    const int64_t off = sf_group_offset((int64_t)g_b0[gr] * 128 + local, kg, rest_k);
                    *reinterpret_cast<uint32_t *>(SF + off) = code | (c1 << 8) | (c2 << 16) | (c3 << 24);
                }
            }
        }
    }
}

// Zero the padding scale rows [M_g, pad128(M_g)) of every group: CTA (g, y) takes pad
// rows y, y + kPadSlices, ... of group g; a row's k-group holds 4 contiguous scale
// bytes, so each thread writes whole 32-bit words (32-bit index arithmetic only).
constexpr int kPadSlices = 16;
__global__ void grouped_sf_pad_zero_kernel(uint8_t *SF, const int *m_offsets, int G, int m_total, int64_t K) {
    __shared__ int g_r0[kQuantMaxGroups], g_r1[kQuantMaxGroups], g_b0[kQuantMaxGroups + 1];
    if (threadIdx.x < 32) build_group_tables(m_offsets, G, m_total, 0, threadIdx.x & 31, g_r0, g_r1, g_b0, nullptr);
    __syncthreads();
    const int gr = blockIdx.x;
    const int mg = g_r1[gr] - g_r0[gr];
    const int pad = (mg + 127) / 128 * 128 - mg;
    const int rest_k = (int)(K >> 6);
    for (int pr = blockIdx.y; pr < pad; pr += gridDim.y) {
        const int64_t r = (int64_t)g_b0[gr] * 128 + mg + pr;
        for (int kg = threadIdx.x; kg < rest_k; kg += blockDim.x)
            *reinterpret_cast<uint32_t *>(SF + sf_group_offset(r, kg, rest_k)) = 0u;
    }
}

// Zero the scale bytes of rows [M, pad128(M)): one CTA per padding row, 32-bit words.
__global__ void sf_pad_zero_kernel(uint8_t *SF, int64_t M, int64_t K) {
    const int64_t r = M + blockIdx.x;
    const int rest_k = (int)(K >> 6);
    for (int kg = threadIdx.x; kg < rest_k; kg += blockDim.x)
        *reinterpret_cast<uint32_t *>(SF + sf_group_offset(r, kg, rest_k)) = 0u;
}

// amax over n bf16 (n % 8 == 0 handled by the vector loop, the rest scalar).
// Non-negative floats order like their bit patterns, so atomicMax on the bits works.
__global__ void __launch_bounds__(256) amax_kernel(const __nv_bfloat16 *__restrict__ X, int64_t n,
                                                   uint32_t *__restrict__ amax_bits) {
    float m = 0.0f;
    const int64_t n8 = n / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += stride) {
        uint4 r = ld_stream_u4(X + i * 8);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            m = fmaxf(m, fabsf(__uint_as_float(w[j] << 16)));
            m = fmaxf(m, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
        }
    }
    for (int64_t i = n8 * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        m = fmaxf(m, fabsf(__bfloat162float(X[i])));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float wmax[8];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, wmax[i]);
        atomicMax(amax_bits, __float_as_uint(m));
    }
}

__global__ void global_scale_kernel(const uint32_t *amax_bits, float *amax_out, float *gs_out) {
    const float a = __uint_as_float(*amax_bits);
    if (amax_out) *amax_out = a;
    if (gs_out) *gs_out = __fdiv_rn(a, 2688.0f);  // amax / (6 * 448)
}

int sf_pad_zero(uint8_t *SF, int M, int K, cudaStream_t s, const DeviceInfo &di);

// Workspace of quantize_dynamic_dispatch: the barrier's two counters (zero between
// calls) and one amax partial per CTA of the largest grid.
static int dynamic_grid(const DeviceInfo &di) {
    static int per_sm[64] = {};
    if (!per_sm[di.device]) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quantize_dynamic_kernel, 256, 0) != cudaSuccess || n < 1)
            return 0;
        per_sm[di.device] = n;
    }
    return per_sm[di.device] * di.sm_count;
}

size_t quantize_dynamic_workspace_bytes() {
    DeviceInfo di;
    if (device_info(&di)) return 0;
    return 256 + (size_t)dynamic_grid(di) * sizeof(float);
}

// Argument checks of quantize_dynamic_dispatch (host only, no device call).
int quantize_dynamic_check(const uint16_t *X, const uint8_t *Q, const uint8_t *SF, const float *amax_out,
                           const float *gs_out, int M, int K) {
    if (!X || !Q || !SF) return NVFP4_ERR_INVALID;
    if (M < 1 || K < 64 || K % 64) return NVFP4_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(X) & 31u) || !aligned16(Q) || (reinterpret_cast<uintptr_t>(SF) & 3u) ||
        (reinterpret_cast<uintptr_t>(amax_out) & 3u) || (reinterpret_cast<uintptr_t>(gs_out) & 3u))
        return NVFP4_ERR_ALIGN;
    return NVFP4_OK;
}

// bf16 X -> amax, global scale, NVFP4 codes and blocked scales in one cooperative
// launch (ws: quantize_dynamic_workspace_bytes(), zero-filled once, one per stream).
int quantize_dynamic_dispatch(const uint16_t *X, uint8_t *Q, uint8_t *SF, float *amax_out, float *gs_out, int M,
                              int K, void *ws, size_t ws_bytes, cudaStream_t s) {
    int st = quantize_dynamic_check(X, Q, SF, amax_out, gs_out, M, K);
    if (st) return st;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const int max_grid = dynamic_grid(di);
    if (!max_grid) return NVFP4_ERR_CUDA;
    if (!ws || ws_bytes < 256 + (size_t)max_grid * sizeof(float) || (reinterpret_cast<uintptr_t>(ws) & 255u))
        return NVFP4_ERR_WORKSPACE;
    KernelCtl ctl;
    if ((st = kernel_ctl(&ctl))) return st;
    const int64_t n_blocks = (int64_t)M * K / 16;
    const unsigned grid = (unsigned)std::min<int64_t>(max_grid, (n_blocks + 255) / 256);
    const __nv_bfloat16 *x = reinterpret_cast<const __nv_bfloat16 *>(X);
    unsigned int *bar = static_cast<unsigned int *>(ws);
    float *partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + 256);
    int64_t nb = n_blocks, kk = K;
    void *args[] = {&x, &Q, &SF, &amax_out, &gs_out, &bar, &partials, &nb, &kk, &ctl};
    if (cudaLaunchCooperativeKernel((void *)quantize_dynamic_kernel, dim3(grid), dim3(256), args, 0, s) !=
        cudaSuccess)
        return NVFP4_ERR_CUDA;
    count_launch();
    if ((st = cuda_status(cudaGetLastError()))) return st;
    return sf_pad_zero(SF, M, K, s, di);
}

// Zero the padding scale rows [M_g, pad128(M_g)) of every group of a grouped scale
// tensor (the layout nvfp4_quantize_grouped writes).
int grouped_sf_pad_zero(uint8_t *SF, const int *m_offsets, int groups, int m_total, int K, cudaStream_t s) {
    grouped_sf_pad_zero_kernel<<<dim3(groups, kPadSlices), 256, 0, s>>>(SF, m_offsets, groups, m_total, K);
    count_launch();
    return cuda_status(cudaGetLastError());
}

// Zero the scale bytes of rows [M, pad128(M)) of a blocked [pad128(M), K/16] tensor.
int sf_pad_zero(uint8_t *SF, int M, int K, cudaStream_t s, const DeviceInfo &di) {
    if (M % 128 == 0) return NVFP4_OK;
    sf_pad_zero_kernel<<<(unsigned)((M + 127) / 128 * 128 - M), 256, 0, s>>>(SF, M, K);
    count_launch();
    return cuda_status(cudaGetLastError());
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" int nvfp4_quantize(const uint16_t *X, uint8_t *Q, uint8_t *SF, const float *global_scale, int M, int K,
                              void *stream) {
    if (!X || !Q || !SF || !global_scale) return NVFP4_ERR_INVALID;
    if (M < 1 || K < 64 || K % 64) return NVFP4_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(X) & 31u) || !aligned16(Q) || (reinterpret_cast<uintptr_t>(SF) & 3u) ||
        (reinterpret_cast<uintptr_t>(global_scale) & 3u))
        return NVFP4_ERR_ALIGN;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t n_blocks = (int64_t)M * K / 16;
    const int threads = 256;
    int64_t blocks = (n_blocks + threads - 1) / threads;
    // at most one wave of resident CTAs (the loop strides over the rest): a grid beyond
    // what fits on the SMs at once leaves a partial second wave
    static int per_sm[64] = {};
    if (!per_sm[di.device]) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quantize_kernel, threads, 0) != cudaSuccess || n < 1)
            n = 1;
        per_sm[di.device] = n;
    }
    const int64_t cap = (int64_t)di.sm_count * per_sm[di.device];
    if (blocks > cap) blocks = cap;
    // a programmatic dependent of the previous kernel in the stream: the CTAs are
    // placed while that kernel finishes, and wait for it before reading anything
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(threads);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, quantize_kernel, reinterpret_cast<const __nv_bfloat16 *>(X), Q, SF, global_scale,
                           n_blocks, (int64_t)K) != cudaSuccess)
        return NVFP4_ERR_CUDA;
    count_launch();
    if ((st = cuda_status(cudaGetLastError()))) return st;
    return sf_pad_zero(SF, M, K, s, di);
}

extern "C" int nvfp4_quantize_grouped(const uint16_t *X, uint8_t *Q, uint8_t *SF, const float *global_scale,
                                      const int32_t *m_offsets, int groups, int m_total, int K, void *stream) {
    if (!X || !Q || !SF || !global_scale || !m_offsets) return NVFP4_ERR_INVALID;
    if (groups < 1 || groups > kQuantMaxGroups || m_total < 1 || K < 64 || K % 64) return NVFP4_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(X) & 31u) || !aligned16(Q) || (reinterpret_cast<uintptr_t>(SF) & 3u) ||
        (reinterpret_cast<uintptr_t>(global_scale) & 3u) || (reinterpret_cast<uintptr_t>(m_offsets) & 3u))
        return NVFP4_ERR_ALIGN;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t n_blocks = (int64_t)m_total * K / 16;
    int64_t blocks = (n_blocks + 255) / 256;
    if (blocks > (int64_t)di.sm_count * 8) blocks = (int64_t)di.sm_count * 8;
    quantize_grouped_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16 *>(X), Q, SF,
                                                             global_scale, m_offsets, groups, m_total, K);
    count_launch();
    if ((st = cuda_status(cudaGetLastError()))) return st;
    return grouped_sf_pad_zero(SF, m_offsets, groups, m_total, K, s);
}

extern "C" int nvfp4_global_scale(const uint16_t *X, int64_t n, float *amax_out, float *gs_out, void *stream) {
    if (!X || n < 1) return NVFP4_ERR_INVALID;
    if (!aligned16(X)) return NVFP4_ERR_ALIGN;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The running max lives in a 4-byte slot of the caller's output when given,
    // otherwise in gs_out; both are fp32 device words of the caller.
    uint32_t *acc = reinterpret_cast<uint32_t *>(amax_out ? amax_out : gs_out);
    if (!acc) return NVFP4_ERR_INVALID;
    if ((st = cuda_status(cudaMemsetAsync(acc, 0, 4, s)))) return st;
    int64_t blocks = (n / 8 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > (int64_t)di.sm_count * 8) blocks = (int64_t)di.sm_count * 8;
    amax_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16 *>(X), n, acc);
    global_scale_kernel<<<1, 1, 0, s>>>(acc, amax_out, gs_out);
    count_launch();
    count_launch();
    return cuda_status(cudaGetLastError());
}
