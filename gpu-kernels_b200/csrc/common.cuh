// common.cuh — shared host/device plumbing of libnvfp4_b200: status codes, the
// device-side status word, tensor-map encoding, per-device properties.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/nvfp4_b200.h"

namespace nvfp4 {

// Device status word (one per device, a module-scope __device__ variable of
// runtime.cu).  Kernels receive its address in KernelCtl and OR a bit into it
// when a bounded wait gives up; nvfp4_device_status() reads and clears it.
enum : uint32_t { kDevTimeout = 1u };

// Knobs passed by value to every kernel.
struct KernelCtl {
    uint64_t wait_timeout_ns;  // bound of each individual wait
    uint64_t drain_timeout_ns; // bound used while draining after an abort
    uint32_t *status;          // device address of the status word
};

// Number of device-side timeouts nvfp4_device_status has reported on device `dev`.
// A kernel that gave up a wait may leave split-K arrival counters or grid-barrier
// counters non-zero, so a library-owned workspace remembers the count it was last
// cleared at and clears itself again once the count has moved.
uint64_t timeout_epoch(int dev);

// Current limits (nvfp4_set_wait_timeout_ns) and the current device's status word.
int kernel_ctl(KernelCtl *out);
void count_launch();          // bump nvfp4_launch_count()

// Signal pads of the ranks of one node, as this process addresses them.
constexpr int kMaxRanks = 8;
struct RankPads {
    uint64_t ptr[kMaxRanks];
};

// Per-device facts cached on first use.
struct DeviceInfo {
    int device = -1;
    int sm_count = 0;
    int major = 0, minor = 0;
    int max_smem_optin = 0;
};
int device_info(DeviceInfo *out);  // current device; NVFP4_OK or error

// cuTensorMapEncodeTiled obtained through the runtime (the library does not link
// libcuda, so it also loads on machines without a driver).
int encode_tiled_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                    uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle);

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? NVFP4_OK : NVFP4_ERR_CUDA; }

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device-side: record a timeout and raise the CTA-local abort flag.
__device__ __forceinline__ void report_timeout(volatile int *abort, uint32_t *status) {
    *abort = 1;
    atomicOr(status, kDevTimeout);
}

}  // namespace nvfp4
