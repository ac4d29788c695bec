/*
 * nvfp4_b200.h — C ABI of the B200 (sm_100a) NVFP4 block-scaled GEMM and its
 * bf16 -> NVFP4 quantizer (library: gpu-kernels_b200/nvfp4_b200/libnvfp4_b200.so).
 *
 * It is the drop-in boundary for the reference's plugin surface
 * (Parth-Badgujar/gpu-kernels):
 *   matmul/sm100_nvfp4/block_scaled_nvfp4.cuh:7-18   host launcher declarations
 *       void matmul_nvfp4_vN(fp16 *c, const uint8_t *sfa, const uint8_t *sfb,
 *                            const uint8_t *a, const uint8_t *b, int M, int N, int K);
 *   matmul/sm100_nvfp4/runner.cu:61-96               the runner that calls them
 *   matmul/sm100_nvfp4/main.py:9-34                  operand formats / oracle semantics
 *
 * Only plain pointers, sizes and status codes cross it: no CUDA, torch or C++
 * types.  Streams are passed as `void*` (a cudaStream_t / CUstream handle;
 * NULL = the legacy default stream).  All data pointers are DEVICE pointers of
 * the current device unless a function says otherwise.
 *
 * Operand formats (identical to the reference's):
 *   A  [M, K/2]  uint8: e2m1 codes, K-major, element 2i in the low nibble
 *   B  [N, K/2]  uint8: same (B is the "weight", D = A . B^T)
 *   SFA/SFB      uint8 e4m3 codes, one per 16 K-elements, in the 128x4 blocked
 *                layout of [pad128(rows), K/16]:
 *                off(r,k16) = ((r/128)*(K/64) + k16/4)*512 + (r%32)*16
 *                             + ((r/32)%4)*4 + k16%4
 *                (rows padded to a multiple of 128; padding scales must be finite)
 *   D  [M, N]    bf16 (uint16 bit patterns) row-major, D = alpha * A . B^T
 *
 * Shape rules: M >= 1, N >= 8 with N % 8 == 0, K >= 64 with K % 64 == 0 (the bf16
 * row pitch of D is a multiple of 16 bytes).  Pointers 16-byte aligned.
 *
 * Errors: every int-returning function returns NVFP4_OK (0) or a negative
 * status; nothing exits or traps.  Kernel launches are asynchronous; a device
 * side timeout (a bounded wait that gave up) is latched in a per-device status
 * word that nvfp4_device_status() reads and clears.
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NVFP4_API __attribute__((visibility("default")))
#else
#define NVFP4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    NVFP4_OK = 0,
    NVFP4_ERR_INVALID = -1,      /* null pointer or bad argument            */
    NVFP4_ERR_SHAPE = -2,        /* M/N/K violate the shape rules           */
    NVFP4_ERR_ALIGN = -3,        /* pointer not 16-byte aligned             */
    NVFP4_ERR_CUDA = -4,         /* CUDA runtime / driver error             */
    NVFP4_ERR_TIMEOUT = -5,      /* a bounded device wait gave up           */
    NVFP4_ERR_UNSUPPORTED = -6,  /* device is not sm_100 (B200/GB200)       */
    NVFP4_ERR_WORKSPACE = -7     /* workspace missing or too small          */
};

/* Human-readable name of a status code. */
NVFP4_API const char *nvfp4_status_string(int status);

/* Library version as (major << 16) | minor. */
NVFP4_API int nvfp4_version(void);

/*
 * bf16 -> NVFP4 quantizer.  Replaces: nothing in the reference (it has no
 * quantizer; main.py:9-23 draws random codes instead).  Required by the
 * reference path's operands.
 *   X [M, K] bf16 row-major -> Q [M, K/2] e2m1 codes, SF blocked [pad128(M), K/16]
 *   global_scale: DEVICE pointer to one fp32 gs (x ~= q * sf * gs).
 * Per 16-element block: sf = e4m3_rn_sat((amax/6)/gs); q = e2m1_rn_sat(x * (1/(sf*gs))),
 * every fp32 step a single IEEE round-to-nearest operation (bit-exact with the
 * CPU specification).  SF padding rows are written as 0.  X must be 32-byte
 * aligned (one 256-bit load per 16-element block), Q 16-byte, SF 4-byte.
 */
NVFP4_API int nvfp4_quantize(const uint16_t *X, uint8_t *Q, uint8_t *SF, const float *global_scale,
                   int M, int K, void *stream);

/*
 * Tensor amax and global scale: *amax_out = max |X|, *gs_out = amax / (6 * 448)
 * (both DEVICE fp32 pointers; either may be NULL).  n = number of bf16 elements.
 * Replaces: nothing in the reference; it is the first pass of the quantizer
 * when gs is not known ahead of time.
 */
NVFP4_API int nvfp4_global_scale(const uint16_t *X, int64_t n, float *amax_out, float *gs_out,
                       void *stream);
/* nvfp4_global_scale and nvfp4_quantize in one pass over X (M x K bf16, K % 64):
 * amax and gs = amax / (6 * 448) into amax_out / gs_out (device fp32, either may be
 * NULL), then Q and SF with that gs — byte-identical to the two calls in sequence.
 * One cooperative launch: each CTA's amax, a grid barrier, then the quantization
 * re-reads X while it is still in L2.  Uses a small library-owned workspace per
 * (device, stream), allocated on the first call there.  No counterpart in the
 * reference (it has no quantizer). */
NVFP4_API int nvfp4_quantize_dynamic(const uint16_t *X, uint8_t *Q, uint8_t *SF, float *amax_out, float *gs_out,
                                     int M, int K, void *stream);

/*
 * NVFP4 GEMM, D = alpha * A . B^T, bf16 out.  Replaces the reference's best B200
 * launcher matmul_nvfp4_v5 (matmul/sm100_nvfp4/nvfp4_v5.cu:287-309, declared at
 * block_scaled_nvfp4.cuh:15-16), adding alpha, bf16 output, a stream, any
 * M >= 1 / N % 8 / K % 64 shape and a status code.  For M > 128 it runs the
 * persistent, warp-specialised tcgen05 kernels (nvfp4_gemm_persistent: CTA pairs,
 * or single CTAs for grids of at most one wave of 256 x 256 tiles with short K —
 * the two give the same bits).  For
 * M <= 128 (decode shapes; env NVFP4_DECODE_MAX_M lowers the bound, 0 disables)
 * it runs the stream-K decode kernel (nvfp4_gemm_decode) — or, for weights of at
 * least 48 tiles of 256 rows with M >= 64 (M >= 32 for the widest), the persistent
 * single-CTA kernel, which reads the activations once per 256 weight rows — with a
 * decode workspace that
 * this function allocates with cudaMalloc on the first such call per (device,
 * stream) and keeps; make that first call outside CUDA-graph capture.
 */
NVFP4_API int nvfp4_gemm(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
               float alpha, uint16_t *D, int M, int N, int K, void *stream);

/* The persistent tensor-core kernel alone (any M), no workspace, no allocation. */
NVFP4_API int nvfp4_gemm_persistent(const uint8_t *A, const uint8_t *SFA, const uint8_t *B,
               const uint8_t *SFB, float alpha, uint16_t *D, int M, int N, int K, void *stream);

/*
 * Skinny-M (1 <= M <= 128) split-K / stream-K GEMM, bf16 out, bound by HBM bandwidth.
 * Replaces nothing that runs in the reference: its launchers produce zero tiles
 * for M < 128 (matmul/sm100_nvfp4/nvfp4_v5.cu:163-176, 287-309).
 * `workspace` (256-byte aligned, >= nvfp4_gemm_decode_workspace_size(M, N) bytes: a
 * fixed 256 KB region of arrival counters, then the fp32 partial tiles) must be
 * zero-filled before its first use; every call that completes leaves its counters
 * at zero again, so one buffer serves calls of any shape.  After
 * nvfp4_device_status has reported NVFP4_ERR_TIMEOUT, zero it again before reuse.
 * Calls that share a workspace must be ordered (same stream); overlapping calls race.
 * At most 65536 weight tiles (N <= 8388608); workspace_size returns 0 beyond that.
 */
NVFP4_API size_t nvfp4_gemm_decode_workspace_size(int M, int N);
NVFP4_API int nvfp4_gemm_decode(const uint8_t *A, const uint8_t *SFA, const uint8_t *B,
               const uint8_t *SFB, float alpha, uint16_t *D, int M, int N, int K, void *workspace,
               size_t workspace_bytes, void *stream);

/* Same contract, fp16 output (the reference's output type). */
NVFP4_API int nvfp4_gemm_f16(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                   float alpha, uint16_t *D, int M, int N, int K, void *stream);

/*
 * Fused epilogue (no counterpart in the reference, whose kernels only convert the
 * fp32 accumulator to fp16).  Per element of D, in fp32 with one IEEE rounding per
 * operation:
 *   y = alpha * acc;  y += bias[n] (bf16, optional);  y = act(y)
 * with act one of
 *   NVFP4_ACT_NONE, NVFP4_ACT_RELU (max(y, 0)), NVFP4_ACT_SILU (y / (1 + exp(-y))),
 *   NVFP4_ACT_GELU_TANH (0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3)))),
 * silu and gelu with the GPU's tanh instruction (tanh.approx).
 * NVFP4_ACT_SWIGLU gates one half of the columns with the other: B's rows hold gate
 * and up weights interleaved in blocks of 16 (rows 32j .. 32j+15 gate, 32j+16 ..
 * 32j+31 up; bias in the same order), and output column c of the N/2 output columns
 * is silu(y[32*(c/16) + c%16]) * y[32*(c/16) + 16 + c%16] — the SwiGLU FFN's
 * silu(x W1^T) * (x W3^T) from one GEMM over the interleaved weight.  N % 128 == 0;
 * D (or q_out / sf_out) then has N/2 columns.
 * Output: bf16(y) into D, or — when q_out is given — the bf16(y) rows quantized to
 * NVFP4 for the next layer: codes [M, Nout/2] into q_out and blocked e4m3 scales
 * [pad128(M), Nout/16] into sf_out (Nout = N, or N/2 with SwiGLU) with the fp32
 * global scale *out_global_scale (device), byte-identical to nvfp4_quantize applied
 * to the bf16 output.  NVFP4 output needs Nout % 64 == 0; D is then not written and
 * may be NULL.
 */
enum {
    NVFP4_ACT_NONE = 0,
    NVFP4_ACT_RELU = 1,
    NVFP4_ACT_SILU = 2,
    NVFP4_ACT_GELU_TANH = 3,
    NVFP4_ACT_SWIGLU = 4
};
typedef struct nvfp4_epilogue {
    const uint16_t *bias;          /* bf16 [N] (16-byte aligned), or NULL */
    int activation;                /* NVFP4_ACT_* */
    uint8_t *q_out;                /* NVFP4 output codes [M, N/2] (32-byte aligned), or NULL for bf16 D */
    uint8_t *sf_out;               /* its blocked scales [pad128(M) * N/16] (4-byte aligned) */
    const float *out_global_scale; /* device fp32 global scale of the output */
} nvfp4_epilogue;

/* nvfp4_gemm with the fused epilogue `epi` (NULL = plain nvfp4_gemm).  Same kernel
 * choice (split-K decode kernel for M <= 128, the persistent kernels above; SwiGLU
 * always on CTA pairs). */
NVFP4_API int nvfp4_gemm_epilogue(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                                  float alpha, uint16_t *D, int M, int N, int K, const nvfp4_epilogue *epi,
                                  void *stream);

/*
 * Grouped (mixture-of-experts) GEMM and its quantizer — no counterpart in the
 * reference.  G <= 256 groups share N and K.  Group g is rows
 * [m_offsets[g], m_offsets[g+1]) of the stacked activations A [m_total, K/2] (and of
 * D [m_total, N]) and uses expert weight g = rows [g*N, (g+1)*N) of B [G*N, K/2]:
 *     D[r, :] = alpha[g] * A[r, :] . B_g^T        for r in group g.
 * m_offsets (G+1 int32, non-decreasing, clamped to [0, m_total]) and alpha (G fp32)
 * are DEVICE arrays, so routing decided on the GPU needs no host round trip.
 * Block scales of a grouped operand are laid out group by group: group g's blocked
 * [pad128(M_g), K/16] tensor starts at 128-row block sum_{h<g} ceil(M_h/128), so a
 * scale buffer needs (ceil(m_total/128) + G) * 128 * K/16 bytes
 * (nvfp4_quantize_grouped writes this layout).  SFB is the G experts' blocked scale
 * tensors one after another (N % 128 == 0).  D rows outside every group are not
 * written.
 */
NVFP4_API int nvfp4_gemm_grouped(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                                 const float *alpha, uint16_t *D, const int32_t *m_offsets, int groups,
                                 int m_total, int N, int K, void *stream);
/* nvfp4_gemm_grouped with the fused epilogue of nvfp4_gemm_epilogue (epi may be
 * NULL): epi->bias, if given, is [G, N] bf16 (expert g's bias row g); with q_out the
 * output is NVFP4 — codes [m_total, N/2] in stacked row order, scales in the grouped
 * layout above (group g's blocked [pad128(M_g), N/16] tensor from 128-row block
 * sum_{h<g} ceil(M_h/128), padding rows zeroed), i.e. exactly what
 * nvfp4_quantize_grouped makes of the bf16 output, ready as the A operand of the next
 * grouped GEMM.  D may then be NULL.  Rows outside every group are not written. */
NVFP4_API int nvfp4_gemm_grouped_epilogue(const uint8_t *A, const uint8_t *SFA, const uint8_t *B,
                                          const uint8_t *SFB, const float *alpha, uint16_t *D,
                                          const int32_t *m_offsets, int groups, int m_total, int N, int K,
                                          const nvfp4_epilogue *epi, void *stream);
/* bf16 X [m_total, K] -> codes Q [m_total, K/2] and the grouped scale layout above,
 * one global scale for all groups (padding scale rows of every group zeroed). */
NVFP4_API int nvfp4_quantize_grouped(const uint16_t *X, uint8_t *Q, uint8_t *SF, const float *global_scale,
                                     const int32_t *m_offsets, int groups, int m_total, int K, void *stream);

/*
 * Column-parallel GEMM with the all-gather of the output fused into the epilogue (no
 * counterpart in the reference, whose kernels run on one GPU; the multi-GPU plan
 * gathers the N-shards with NCCL).  This rank computes its shard
 *     D_shard[M, N] = alpha * A . B_shard^T          (bf16)
 * and stores it straight into the full [M, ld] bf16 output of every rank at column
 * col_off: dst holds n_dst device addresses of those full outputs as this process
 * sees them (peer buffers mapped over NVLink, e.g. symmetric memory), or — with
 * multicast != 0 — one NVLink multicast address (n_dst = 1) whose stores the switch
 * delivers to every bound GPU, so each rank sends its shard once.  The call ends when
 * this rank's stores are issued; the caller orders the ranks before reading the full
 * output (a cross-rank barrier on the stream).  N, ld and col_off multiples of 16;
 * destinations 32-byte aligned; the CTA-pair kernel runs for every M.
 */
NVFP4_API int nvfp4_gemm_gather(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                                float alpha, int M, int N, int K, const uint64_t *dst, int n_dst, int multicast,
                                int64_t ld, int col_off, void *stream);

/*
 * Cross-rank barrier on `stream` for the ranks of one node (no counterpart in the
 * reference, which has no multi-GPU path).  signal_pads holds n_ranks (<= 8) device
 * addresses, as this process sees them, of each rank's zero-initialised signal pad of
 * pad_bytes bytes — e.g. the signal pads of torch symmetric memory, whose lower half
 * this barrier leaves alone.  Each rank signals every other rank's pad slot for
 * `channel` with a system-scope release, then waits until every other rank has
 * signalled its own; work queued on the stream before the barrier on any rank
 * (NVLink stores included) is then visible to work queued after it on every rank.
 * Every wait is bounded by the nvfp4_set_wait_timeout_ns limit: one that gives up
 * latches NVFP4_ERR_TIMEOUT (nvfp4_device_status), and the pads must not be used by
 * this barrier again.  n_ranks == 1 returns at once.
 */
NVFP4_API int nvfp4_rank_barrier(const uint64_t *signal_pads, int n_ranks, int rank, int channel, size_t pad_bytes,
                                 void *stream);

/*
 * Reference-signature shim: drop-in for matmul_nvfp4_vN in
 * matmul/sm100_nvfp4/runner.cu:61-96 (fp16 D, alpha = 1, legacy default
 * stream, no return value).  The status of the last call is kept for
 * nvfp4_last_status().  `c` is a __half* in the reference; any 2-byte type works.
 */
NVFP4_API void matmul_nvfp4_b200(void *c, const uint8_t *sfa, const uint8_t *sfb, const uint8_t *a,
                       const uint8_t *b, int M, int N, int K);
NVFP4_API int nvfp4_last_status(void);

/*
 * Reads and clears the device-side status word of the current device after
 * synchronising `stream`: NVFP4_OK, or NVFP4_ERR_TIMEOUT if any kernel of this
 * library gave up a bounded wait since the last call.
 */
NVFP4_API int nvfp4_device_status(void *stream);

/*
 * Upper bound, in nanoseconds, of every device-side wait of this library's
 * kernels (default 2e9).  A wait that exceeds it makes the kernel drain its
 * in-flight copies, free its tensor memory, latch NVFP4_ERR_TIMEOUT and return.
 */
NVFP4_API void nvfp4_set_wait_timeout_ns(uint64_t ns);

/*
 * Self-test of the bounded wait: launches one block that waits on a barrier
 * nothing arrives on, with the given limit, and returns the status read back
 * (NVFP4_ERR_TIMEOUT when the limit works).  The context stays usable.
 */
NVFP4_API int nvfp4_selftest_wait_timeout(uint64_t timeout_ns);

/*
 * The GEMM on HOST buffers (A, SFA, B, SFB in, D out; pinned memory for overlap):
 * the device-side counterpart of the reference runner's copy-in / GEMM / copy-out
 * (matmul/sm100_nvfp4/runner.cu:45-59, 78-90), pipelined.  D is cut into blocks of up
 * to 2048 x 2048, taken in growing squares from the top-left corner; operand uploads,
 * per-block GEMMs and 2-D copies of D back to the host run on three internal streams,
 * so the transfers overlap each other and the compute.  Consecutive calls overlap as
 * well (the next call's uploads start once this call's GEMMs have run; D alternates
 * between two device buffers).
 * Asynchronous: `stream` (the caller's) is made to wait for D to reach the host;
 * synchronise it before reading hD.  Device buffers are allocated on first use per
 * device and kept; calls on one device are serialised.
 */
NVFP4_API int nvfp4_gemm_host(const uint8_t *hA, const uint8_t *hSFA, const uint8_t *hB,
               const uint8_t *hSFB, float alpha, uint16_t *hD, int M, int N, int K, void *stream);

/*
 * Allocation-free decode GEMM.  No counterpart in the reference: it exists for
 * callers that cannot let a library allocate device memory — hosts that own all
 * device memory (memory-budgeted servers, plugin interfaces that pass a library
 * only its inputs and outputs) and latency-critical paths where a cudaMalloc,
 * which may synchronise the device, is not acceptable.
 *
 * Same contract and result as nvfp4_gemm_decode, but the split-K scratch is a
 * fixed 4 MiB device array inside the library (held by every GPU that loads the
 * library until exit), so the call allocates nothing; the caller still passes A,
 * SFA, B, SFB and D.  Shapes whose
 * scratch need (nvfp4_gemm_decode_workspace_size) exceeds it are refused with
 * NVFP4_ERR_WORKSPACE — on a 148-SM B200 that admits M <= 16.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) and clears its
 * arrival counters (a memset on `stream`), so make that first call before any
 * stream capture; later calls clear them again only after nvfp4_device_status has
 * reported a device-side timeout (which can leave counters set) — make that call,
 * too, outside capture.  All calls on a device share the one array: calls whose
 * kernels overlap on the GPU (different streams, no ordering) race.
 */
NVFP4_API int nvfp4_gemm_decode_noalloc(const uint8_t *A, const uint8_t *SFA, const uint8_t *B,
               const uint8_t *SFB, float alpha, uint16_t *D, int M, int N, int K, void *stream);

/* Number of kernel launches this library has issued in this process. */
NVFP4_API uint64_t nvfp4_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
