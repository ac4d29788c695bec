// runtime.cu — host plumbing shared by all entry points: status word, limits,
// device facts, tensor-map encoding, the wait self-test.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"

namespace nvfp4 {

__device__ uint32_t g_device_status = 0;

static std::atomic<uint64_t> g_wait_timeout_ns{2000000000ull};
static std::atomic<uint64_t> g_launches{0};
static std::atomic<uint64_t> g_timeout_epoch[64];

uint64_t timeout_epoch(int dev) {
    return dev >= 0 && dev < 64 ? g_timeout_epoch[dev].load(std::memory_order_acquire) : 0;
}

static uint32_t *status_word_address() {
    static std::mutex mu;
    static uint32_t *addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<uint32_t *>(p);
    }
    return addr[dev];
}

int kernel_ctl(KernelCtl *c) {
    c->wait_timeout_ns = g_wait_timeout_ns.load(std::memory_order_relaxed);
    // Draining after an abort waits only for copies already in flight; they finish
    // in microseconds, so a fixed, independent bound is used.
    c->drain_timeout_ns = 200000000ull;
    c->status = status_word_address();
    return c->status ? NVFP4_OK : NVFP4_ERR_CUDA;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int device_info(DeviceInfo *out) {
    static std::mutex mu;
    static DeviceInfo cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4_ERR_CUDA;
    std::lock_guard<std::mutex> lock(mu);
    DeviceInfo &d = cache[dev];
    if (d.device != dev) {
        DeviceInfo n;
        n.device = dev;
        if (cudaDeviceGetAttribute(&n.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
                cudaSuccess)
            return NVFP4_ERR_CUDA;
        d = n;
    }
    *out = d;
    return d.major == 10 ? NVFP4_OK : NVFP4_ERR_UNSUPPORTED;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int encode_tiled_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                    uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return NVFP4_ERR_CUDA;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NVFP4_OK : NVFP4_ERR_CUDA;
}

// One block waits on an mbarrier that nothing arrives on; the bounded wait must
// give up, latch the timeout bit and return.
__global__ void wait_selftest_kernel(uint64_t timeout_ns, uint32_t *status) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(smem_u32(&bar), 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (!wait_parity(smem_u32(&bar), 0, timeout_ns, &abort_flag)) report_timeout(&abort_flag, status);
    }
    __syncthreads();
}

// Cross-rank barrier over signal slots in memory every rank has mapped (symmetric
// memory signal pads).  Thread t (t != rank) adds 1 to slot [channel][rank] of rank
// t's pad with release semantics, then waits — bounded — until slot [channel][t] of
// its own pad is non-zero, and takes 1 from it.  Counting, not a 0/1 flag, so a fast
// rank may signal the next barrier of a channel before a slow one has consumed the
// last.  A wait that gives up latches the timeout bit and returns; the slots are then
// out of step and the pads must not be used by this barrier again.
__global__ void rank_barrier_kernel(RankPads pads, int n, int rank, int slot0, uint64_t timeout_ns,
                                    uint32_t *status) {
    const int t = threadIdx.x;
    if (t >= n || t == rank) return;
    unsigned int *remote = reinterpret_cast<unsigned int *>(pads.ptr[t]) + slot0 + rank;
    unsigned int *local = reinterpret_cast<unsigned int *>(pads.ptr[rank]) + slot0 + t;
    __threadfence_system();
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(remote) : "memory");
    const uint64_t t0 = global_timer_ns();
    while (true) {
        unsigned int v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(local) : "memory");
        if (v) break;
        if (global_timer_ns() - t0 > timeout_ns) {
            atomicOr(status, kDevTimeout);
            return;
        }
        __nanosleep(64);
    }
    atomicSub(local, 1u);
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

const char *nvfp4_status_string(int s) {
    switch (s) {
        case NVFP4_OK: return "ok";
        case NVFP4_ERR_INVALID: return "invalid argument";
        case NVFP4_ERR_SHAPE: return "unsupported shape (need M>=1, N%8==0, K%64==0)";
        case NVFP4_ERR_ALIGN: return "pointer not 16-byte aligned";
        case NVFP4_ERR_CUDA: return "CUDA error";
        case NVFP4_ERR_TIMEOUT: return "device wait timed out";
        case NVFP4_ERR_UNSUPPORTED: return "device is not sm_100";
        case NVFP4_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

int nvfp4_version(void) { return (0 << 16) | 3; }

void nvfp4_set_wait_timeout_ns(uint64_t ns) { g_wait_timeout_ns.store(ns ? ns : 1, std::memory_order_relaxed); }

uint64_t nvfp4_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int nvfp4_device_status(void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(s) != cudaSuccess) return NVFP4_ERR_CUDA;
    uint32_t v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess) return NVFP4_ERR_CUDA;
    if (v && cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)) != cudaSuccess) return NVFP4_ERR_CUDA;
    if (v & kDevTimeout) {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64)
            g_timeout_epoch[dev].fetch_add(1, std::memory_order_acq_rel);
        return NVFP4_ERR_TIMEOUT;
    }
    return NVFP4_OK;
}

int nvfp4_rank_barrier(const uint64_t *signal_pads, int n_ranks, int rank, int channel, size_t pad_bytes,
                       void *stream) {
    if (!signal_pads || n_ranks < 1 || n_ranks > kMaxRanks || rank < 0 || rank >= n_ranks || channel < 0)
        return NVFP4_ERR_INVALID;
    // this barrier's slots: the upper half of each pad, n_ranks words per channel
    const size_t words = pad_bytes / 4, slot0 = words / 2 + static_cast<size_t>(channel) * n_ranks;
    if (slot0 + n_ranks > words) return NVFP4_ERR_INVALID;
    RankPads pads;
    for (int r = 0; r < n_ranks; ++r) {
        if (!signal_pads[r] || (signal_pads[r] & 3u)) return NVFP4_ERR_ALIGN;
        pads.ptr[r] = signal_pads[r];
    }
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    if (n_ranks == 1) return NVFP4_OK;
    KernelCtl ctl;
    if ((st = kernel_ctl(&ctl))) return st;
    rank_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(pads, n_ranks, rank, static_cast<int>(slot0),
                                                                        ctl.wait_timeout_ns, ctl.status);
    count_launch();
    return cuda_status(cudaGetLastError());
}

int nvfp4_selftest_wait_timeout(uint64_t timeout_ns) {
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    st = nvfp4_device_status(nullptr);  // clear anything older
    if (st == NVFP4_ERR_CUDA) return st;
    KernelCtl ctl;
    if ((st = kernel_ctl(&ctl))) return st;
    wait_selftest_kernel<<<1, 32>>>(timeout_ns, ctl.status);
    count_launch();
    if (cudaGetLastError() != cudaSuccess) return NVFP4_ERR_CUDA;
    return nvfp4_device_status(nullptr);
}

}  // extern "C"
