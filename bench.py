"""bench.py — NVFP4 GEMM throughput on B200 (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: D[M,N] = alpha * A[M,K] . B[N,K]^T with
M = N = K = 8192 per GPU, A and B drawn bf16 N(0,1) on the device (seeded) and
quantized to NVFP4 by this library's quantizer; bf16 output.  A step is one GEMM
launch.  Multi-GPU is column-parallel (weak scaling): rank p owns an 8192-column
shard of B (N_total = 8192 * P), A is replicated, no collective is needed for the
result, so none runs in the timed region.

`value` is the whole-job TFLOP/s (sum of 2*M*N_shard*K over ranks / max-over-ranks
device time).  Inputs rotate over enough distinct operand sets to exceed 3x L2.
`e2e` times the same GEMM through the public API from pinned HOST buffers: the
H2D copies of A, SFA, B, SFB and the D2H copy of D are inside the timed region.

`--impl reference` times the reference's path on the host cores: the CPU
dequantise + fp32 GEMM (oracle/, the reference has no CPU implementation of its
own) on a bounded row sample of the same workload.
"""
import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gpu-kernels_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

M_ = N_ = K_ = 8192
METRIC = "NVFP4 GEMM TFLOPS/GPU & % FP4 peak (8192^3); decode-shape HBM GB/s; 1/2/4/8 GPU"
UNIT = "TFLOP/s"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def host_threads():
    """Host cores this process may run on.  Passed explicitly to every oracle call:
    torch.distributed.run exports OMP_NUM_THREADS=1, which would otherwise pin the
    OpenMP default (omp_get_max_threads) of every rank to one thread."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def committed_traffic():
    """DRAM bytes per GEMM launch from the committed ncu capture summary, if any."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled through NVML on a
    background thread (every ~1 ms plus the call's own latency) for the duration of
    the timed region."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.max_mhz = None
        self._stop = None

    def _handle(self, nvml):
        props = torch.cuda.get_device_properties(self.device)
        uuid = str(getattr(props, "uuid", ""))
        if uuid:
            for cand in (uuid if uuid.startswith("GPU-") else "GPU-" + uuid, uuid):
                try:
                    return nvml.nvmlDeviceGetHandleByUUID(cand)
                except Exception:
                    pass
        bus = "%08x:%02x:%02x.0" % (getattr(props, "pci_domain_id", 0), props.pci_bus_id, props.pci_device_id)
        return nvml.nvmlDeviceGetHandleByPciBusId(bus)

    def __enter__(self):
        import threading
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            h = self._handle(nvml)
            self.max_mhz = nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM)
            get_reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as e:  # no NVML: report the gap instead of guessing
            self.error = f"nvml unavailable: {e}"
            return self
        self._stop = threading.Event()

        def loop():
            power, n = 0.0, 0
            while not self._stop.is_set():
                try:
                    if n % 8 == 0:  # power is the slowest query and only reported as a maximum
                        power = nvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    self.samples.append((nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM), power,
                                         int(get_reasons(h))))
                    n += 1
                except Exception:
                    pass
                self._stop.wait(0.0005)

        # The launching thread releases the GIL only briefly (ctypes calls); a short
        # switch interval lets the sampler run every ~0.5 ms instead of every 5 ms.
        self._switch = sys.getswitchinterval()
        sys.setswitchinterval(1e-4)
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)
            sys.setswitchinterval(self._switch)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0,
                    "note": getattr(self, "error", "no sample fell in the timed region")}
        mask = 0
        for _, _, r in self.samples:
            mask |= r
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(v for k, v in self.REASONS.items() if mask & k), "samples": len(self.samples),
                "power_w_max": max(s[1] for s in self.samples), "source": "nvml"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def in_kernel_clock(nv, operands, d, M, N, K, dev):
    """SM clock the GEMM itself runs at: one launch of the traced CTA-pair kernel (the
    diagnostic library, nvfp4_diag; outside every timed region) on the bench's
    operands, clock64 cycles over globaltimer ns of each pair's MMA thread."""
    try:
        import nvfp4_diag
        diag = nvfp4_diag.lib()
    except ImportError:
        return None
    a, sfa, b, sfb, alpha = operands
    sms = torch.cuda.get_device_properties(dev).multi_processor_count  # one trace row per CTA, grid <= #SMs
    tr = torch.zeros(sms * 12, dtype=torch.int64, device=dev)
    st = diag.nvfp4_gemm_trace(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), alpha, d.data_ptr(),
                                   M, N, K, tr.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize()
    if st != 0:
        return None
    t = tr.view(sms, 12)[0::2].double().cpu()
    ok = t[:, 7] > 0
    return float((t[ok, 6] / t[ok, 7]).mean() * 1e3) if ok.any() else None


def make_operand_sets(nv, n_sets, M, N, K, seed, dev):
    """Quantized operand sets generated on the device by the product's own kernels."""
    g = torch.Generator(device=dev)
    sets = []
    for i in range(n_sets):
        g.manual_seed(seed + 1000 * i)
        xa = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        xb = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
        _, gsa = nv.global_scale(xa)
        _, gsb = nv.global_scale(xb)
        a, sfa = nv.quantize(xa, gsa)
        b, sfb = nv.quantize(xb, gsb)
        alpha = float(gsa.item()) * float(gsb.item())
        del xa, xb
        sets.append((a, sfa, b, sfb, alpha))
    torch.cuda.synchronize()
    return sets


class CpuDequantGemm:
    """The reference path on the host cores: dequantise e2m1 x e4m3 to fp32, fp32 GEMM,
    alpha, bf16 (oracle/, all host threads).  B is dequantised once (timed: t_b);
    each step then dequantises a sample of A rows and multiplies them by all of B.
    A full-size job pays t_b once for all M rows, so each step is charged
    t_step + t_b * rows / M."""

    def __init__(self, a, sfa, b, sfb, alpha, M, N, K):
        from oracle import oracle as o
        self.o, self.a, self.sfa, self.alpha, self.M, self.N, self.K = o, a, sfa, alpha, M, N, K
        self.threads = host_threads()
        t0 = time.perf_counter()
        self.bf = o.dequant_rows(b, sfb, 0, N, K, nthreads=self.threads)
        self.t_b = time.perf_counter() - t0

    def step(self, m0, rows):
        t0 = time.perf_counter()
        af = self.o.dequant_rows(self.a, self.sfa, m0, rows, self.K, nthreads=self.threads)
        self.o.sgemm_nt(af, self.bf, self.alpha, nthreads=self.threads)
        return time.perf_counter() - t0 + self.t_b * rows / self.M

    def rows_for(self, seconds):
        t16 = self.step(0, 16)
        t64 = self.step(0, 64)
        per_row = max((t64 - t16) / 48.0, 1e-6)
        return int(min(self.M, max(64, seconds / per_row))) // 16 * 16

    def describe(self, rows):
        return (f"per step: dequantise {rows} rows of A + fp32 GEMM against all of B (N={self.N}, K={self.K}) + "
                f"bf16, plus {rows}/{self.M} of B's one-off dequantisation ({self.t_b:.2f} s); "
                f"{self.threads} host threads")


def cpu_reference_sample(a, sfa, b, sfb, alpha, M, N, K, target_s=12.0):
    """cpu_baseline for our arm: the host dequant GEMM on a row sample of ~target_s."""
    an, sfan, bn, sfbn = (t.cpu().numpy() for t in (a, sfa, b, sfb))
    ref = CpuDequantGemm(an, sfan, bn, sfbn, alpha, M, N, K)
    rows = ref.rows_for(target_s)
    dt = ref.step(0, rows)
    return {"value": 2.0 * rows * N * K / dt / 1e12, "unit": UNIT, "cores": ref.threads, "kind": "port",
            "sample": ref.describe(rows) + f"; {dt:.1f} s"}, rows, dt


def cpu_configs_section():
    """The host reference (oracle/, all host threads) on the other BASELINE configs, each
    in the unit the GPU section for it reports: configs[0] 256^3 (quantize both
    operands + dequant GEMM), configs[2] decode against W1 [28672, 8192] for M in
    {1, 16, 64, 128} (each call dequantises the weight and multiplies: HBM-metric GB/s
    of the same algorithmic bytes), configs[4] (quantize the Student-t activations +
    dequant GEMM of all 4096 rows against W [14336, 4096], whose dequantisation is
    charged once), and a 1024 x 2048 x 8192 slice of configs[3]."""
    from oracle import oracle as o
    import numpy as np
    T = host_threads()
    out = {"cores": T, "kind": "port"}

    def quantized(rows, cols, seed, std=1.0):
        x = o.normal_bf16((rows, cols), seed=seed, std=std, nthreads=T)
        gs = o.global_scale_for(o.amax_bf16(x, nthreads=T))
        q, sf = o.quantize(x, gs, nthreads=T)
        return q, sf, gs

    # 256^3 end to end from bf16
    M = N = K = 256
    xa = o.normal_bf16((M, K), seed=1, nthreads=T)
    xb = o.normal_bf16((N, K), seed=2, nthreads=T)
    t0 = time.perf_counter()
    ga, gb = o.global_scale_for(o.amax_bf16(xa, nthreads=T)), o.global_scale_for(o.amax_bf16(xb, nthreads=T))
    a, sfa = o.quantize(xa, ga, nthreads=T)
    b, sfb = o.quantize(xb, gb, nthreads=T)
    o.gemm(a, sfa, b, sfb, float(np.float32(ga) * np.float32(gb)), M, N, K, nthreads=T)
    dt = time.perf_counter() - t0
    out["c1_256"] = {"ms": dt * 1e3, "tflops": 2.0 * M * N * K / dt / 1e12,
                     "what": "amax + quantize of both bf16 operands + dequant GEMM + bf16"}

    # decode against W1
    N, K = 28672, 8192
    w, wsf, gw = quantized(N, K, 3, std=0.02)
    rows = []
    for M in (1, 16, 64, 128):
        x, xsf, gx = quantized(M, K, 4 + M)
        t0 = time.perf_counter()
        wf = o.dequant_rows(w, wsf, 0, N, K, nthreads=T)
        xf = o.dequant_rows(x, xsf, 0, M, K, nthreads=T)
        o.sgemm_nt(xf, wf, float(np.float32(gx) * np.float32(gw)), nthreads=T)
        dt = time.perf_counter() - t0
        del wf
        nbytes = N * K // 2 + N * K // 16 + M * K // 2 + M * K // 16 + 2 * M * N
        rows.append({"M": M, "N": N, "K": K, "ms": dt * 1e3, "gbs": nbytes / dt / 1e9})
    out["c3_decode_w1"] = rows
    del w, wsf

    # quantize X + GEMM against a pre-quantized W
    M, N, K = 4096, 14336, 4096
    x = o.student_t3_bf16(M, K, seed=9, n_outlier_cols=4, gain=50.0, nthreads=T)
    w, wsf, gw = quantized(N, K, 10, std=0.02)
    t0 = time.perf_counter()
    wf = o.dequant_rows(w, wsf, 0, N, K, nthreads=T)
    t_w = time.perf_counter() - t0
    t0 = time.perf_counter()
    gx = o.global_scale_for(o.amax_bf16(x, nthreads=T))
    xq, xsf = o.quantize(x, gx, nthreads=T)
    xf = o.dequant_rows(xq, xsf, 0, M, K, nthreads=T)
    o.sgemm_nt(xf, wf, float(np.float32(gx) * np.float32(gw)), nthreads=T)
    dt = time.perf_counter() - t0 + t_w
    out["c5"] = {"ms": dt * 1e3, "tflops": 2.0 * M * N * K / dt / 1e12,
                 "what": "amax + quantize of X [4096, 4096] + dequant GEMM against W [14336, 4096] "
                         f"(W's dequantisation, {t_w:.2f} s, included)"}
    del w, wsf, wf, xf

    # the full 16384 x 28672 x 8192 job is 7.7e12 FLOP (~30-50 s on the
    # host, too long for the default run), so a slice of it: 1024 rows of A against
    # 2048 rows of W, full K, both slices dequantised inside the timed region; the rate
    # stands for the whole job.
    M, N, K = 1024, 2048, 8192
    a, sfa, ga = quantized(M, K, 11)
    w, wsf, gw = quantized(N, K, 12, std=0.02)
    t0 = time.perf_counter()
    af = o.dequant_rows(a, sfa, 0, M, K, nthreads=T)
    wf = o.dequant_rows(w, wsf, 0, N, K, nthreads=T)
    o.sgemm_nt(af, wf, float(np.float32(ga) * np.float32(gw)), nthreads=T)
    dt = time.perf_counter() - t0
    full = 2.0 * 16384 * 28672 * 8192
    rate = 2.0 * M * N * K / dt
    out["c4_slice"] = {"ms": dt * 1e3, "tflops": rate / 1e12, "full_job_s_extrapolated": full / rate,
                       "what": "dequant GEMM of A[0:1024] x W[0:2048] at K=8192, a slice of "
                               "configs[3] (16384 x 28672 x 8192)"}
    return out


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as o
    import numpy as np
    M, N, K = M_, N_, K_
    # same workload semantics: N(0,1) bf16 quantized per tensor; operands built on the host
    threads = host_threads()
    xa = o.normal_bf16((M, K), seed=1, nthreads=threads)
    xb = o.normal_bf16((N, K), seed=2, nthreads=threads)
    gsa = o.global_scale_for(o.amax_bf16(xa, nthreads=threads))
    gsb = o.global_scale_for(o.amax_bf16(xb, nthreads=threads))
    a, sfa = o.quantize(xa, gsa, nthreads=threads)
    b, sfb = o.quantize(xb, gsb, nthreads=threads)
    alpha = float(np.float32(gsa) * np.float32(gsb))
    del xa, xb
    ref = CpuDequantGemm(a, sfa, b, sfb, alpha, M, N, K)
    # size each step so the whole run stays within a few minutes
    per_step = max(2.0, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    rows = ref.rows_for(per_step)
    for _ in range(args.warmup):
        ref.step(0, rows)
    times = []
    for s in range(args.steps):
        m0 = (s * rows) % max(1, M - rows + 1)
        times.append(ref.step(m0, rows))
    dt = sum(times)
    value = 2.0 * rows * N * K * len(times) / dt / 1e12
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp4(e2m1)xfp4->fp32",
            "data": "synthetic: bf16 N(0,1) quantized to NVFP4 (seeded)",
            "config": {"workload": "square NVFP4 GEMM M=N=K=8192 (BASELINE configs[1]), CPU row sample",
                       "M": M, "N": N, "K": K, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.threads, "kind": "port",
                             "sample": ref.describe(rows)},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def vendor_scaled_mm(sets, M, N, K, reps=50):
    """Comparison point only (never used by the product): torch._scaled_mm, the
    reference's own oracle (matmul/sm100_nvfp4/main.py:25-34, cuBLASLt block-scaled
    FP4), on the same rotating operand sets, bf16 out."""
    try:
        args = [(a.view(torch.float4_e2m1fn_x2), b.view(torch.float4_e2m1fn_x2).t(),
                 sfa.view(torch.float8_e4m3fn), sfb.view(torch.float8_e4m3fn)) for a, sfa, b, sfb, _ in sets]
        for i in range(3):
            x = args[i % len(args)]
            torch._scaled_mm(x[0], x[1], x[2], x[3], out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            x = args[i % len(args)]
            torch._scaled_mm(x[0], x[1], x[2], x[3], out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        return {"tflops": 2.0 * M * N * K / ms / 1e9, "ms": ms,
                "what": "torch._scaled_mm (cuBLASLt) NVFP4, same operands, bf16 out; comparison only"}
    except Exception as e:  # pragma: no cover - depends on the torch build
        return {"unavailable": f"{type(e).__name__}: {str(e)[:120]}"}


def sustained_section(nv, sets, d, M, N, K, dev, seconds=1.5):
    """The bench GEMM looped back to back for ~`seconds` (after the burst of the
    timed region), with NVML clock samples over the loop and the in-kernel SM clock of
    a traced launch right after it: the rate under the 1 kW power cap."""
    stream = torch.cuda.current_stream(dev)
    flops = 2.0 * M * N * K
    n = len(sets)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)  # calibrate the count of launches from 50 calls
    for i in range(50):
        a, sfa, b, sfb, alpha = sets[i % n]
        nv.gemm(a, sfa, b, sfb, alpha, out=d)
    e1.record(stream)
    torch.cuda.synchronize()
    calls = max(100, int(seconds * 1e3 / (e0.elapsed_time(e1) / 50)))
    with ClockSampler(dev) as clk:
        e0.record(stream)
        for i in range(calls):
            a, sfa, b, sfb, alpha = sets[i % n]
            nv.gemm(a, sfa, b, sfb, alpha, out=d)
        e1.record(stream)
        torch.cuda.synchronize()
    nv.device_status()
    ms = e0.elapsed_time(e1) / calls
    return {"calls": calls, "seconds": calls * ms / 1e3, "ms_per_gemm": ms, "tflops": flops / ms / 1e9,
            "clocks": clk.summary(), "in_kernel_sm_mhz_after": in_kernel_clock(nv, sets[0], d, M, N, K, dev),
            "what": "8192^3 GEMM back to back for >= 1 s, operands rotating as in the timed region"}


# The reference harness's shape list (matmul/sm100_nvfp4/main.py:117-130): it times and
# verifies each of these against torch._scaled_mm.
SWEEP_SHAPES = [(1024, 1024, 1024), (1024, 1024, 2048), (1024, 1024, 4096), (2048, 2048, 2048),
                (2048, 2048, 4096), (2048, 2048, 8192), (4096, 4096, 4096), (4096, 4096, 8192),
                (4096, 4096, 16384), (8192, 8192, 8192), (8192, 8192, 4096), (8192, 8192, 16384)]


def shape_sweep_section(nv, dev, reps=20, check_rows=16):
    """Per shape of the reference harness: this library's nvfp4_gemm and
    torch._scaled_mm (cuBLASLt, the reference's oracle; comparison only) on the same
    operands, each launch timed alone with CUDA events and L2 flushed between launches
    (a 256 MB write) — median TFLOP/s; and `check_rows` sampled rows of our output
    against the CPU oracle (max |D - D_ref| / max |D_ref|, bound 1e-2)."""
    from oracle import oracle as o
    import numpy as np
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev)
    out = []
    for (M, N, K) in SWEEP_SHAPES:
        g.manual_seed(M * 3 + N * 5 + K)
        xa = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        xb = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
        _, gsa = nv.global_scale(xa)
        _, gsb = nv.global_scale(xb)
        a, sfa = nv.quantize(xa, gsa)
        b, sfb = nv.quantize(xb, gsb)
        del xa, xb
        alpha = float((gsa * gsb).item())
        d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)

        def per_launch(fn):
            fn()
            fn()
            ts = []
            for _ in range(reps):
                flush.fill_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            return statistics.median(ts)

        ours = per_launch(lambda: nv.gemm(a, sfa, b, sfb, alpha, out=d))
        row = {"M": M, "N": N, "K": K, "ms": round(ours, 4), "tflops": round(2.0 * M * N * K / ours / 1e9, 1)}
        try:
            va = (a.view(torch.float4_e2m1fn_x2), b.view(torch.float4_e2m1fn_x2).t(),
                  sfa.view(torch.float8_e4m3fn), sfb.view(torch.float8_e4m3fn))
            vend = per_launch(lambda: torch._scaled_mm(va[0], va[1], va[2], va[3], out_dtype=torch.bfloat16))
            row["scaled_mm_ms"] = round(vend, 4)
            row["scaled_mm_tflops"] = round(2.0 * M * N * K / vend / 1e9, 1)
            row["ratio_vs_scaled_mm"] = round(vend / ours, 3)
        except Exception as e:  # pragma: no cover - depends on the torch build
            row["scaled_mm"] = f"unavailable: {type(e).__name__}"
        nv.gemm(a, sfa, b, sfb, alpha, out=d)
        torch.cuda.synchronize()
        nv.device_status()
        m0 = (M // 2) // 128 * 128 + 7  # rows in a middle tile, off the tile edge
        d32, d16 = o.gemm(a.cpu().numpy(), sfa.cpu().numpy(), b.cpu().numpy(), sfb.cpu().numpy(), alpha, M, N, K,
                          m0=m0, mrows=check_rows, nthreads=host_threads())
        ref = o.bf16_bits_to_f32(d16).reshape(check_rows, N)
        got = d[m0:m0 + check_rows].float().cpu().numpy()
        err = float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))
        row["oracle_rel_err"] = float(f"{err:.3e}")
        row["oracle_ok"] = bool(np.isfinite(got).all() and err <= 1e-2)
        out.append(row)
        del a, sfa, b, sfb, d
    del flush
    return {"unit": "TFLOP/s", "timing": f"median of {reps} single launches, L2 flushed before each",
            "check": f"{check_rows} rows per shape against the CPU oracle", "shapes": out}


def decode_section(nv, dev, pk, reps=30):
    """skinny-M GEMMs against the two FFN weights, measured on HBM
    GB/s.  Weights rotate over 3 sets (> 3x L2).  Bytes per call follow the
    algorithmic count N*K/2 + N*K/16 + M*K/2 + M*K/16 + 2*M*N.  `gbs` is device time
    per call with the calls replayed from a CUDA graph (how a decode loop launches
    them); `gbs_eager` is the same calls launched one by one from Python, where the
    host launch path (~15-20 us) can exceed the ~20 us kernel."""
    out = []
    g = torch.Generator(device=dev)
    stream = torch.cuda.Stream(dev)
    for (N, K) in ((28672, 8192), (8192, 28672)):
        ws = []
        for i in range(3):
            g.manual_seed(77 + i)
            w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            _, gs = nv.global_scale(w)
            ws.append(nv.quantize(w, gs))
            del w
        for M in (1, 16, 64, 128):
            g.manual_seed(5 + M)
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            _, gsx = nv.global_scale(x)
            xq, xsf = nv.quantize(x, gsx)
            d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                for i in range(3):  # warm-up on this stream (its workspace is allocated here)
                    nv.gemm(xq, xsf, ws[i % 3][0], ws[i % 3][1], 1.0, out=d)
                stream.synchronize()
                # eager: one Python call per GEMM
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for i in range(reps):
                    nv.gemm(xq, xsf, ws[i % 3][0], ws[i % 3][1], 1.0, out=d)
                e1.record(stream)
                stream.synchronize()
                eager_us = 1e3 * e0.elapsed_time(e1) / reps
            # graph: the same reps calls captured once, replayed
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(reps):
                    nv.gemm(xq, xsf, ws[i % 3][0], ws[i % 3][1], 1.0, out=d)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                graph.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            us = 1e3 * e0.elapsed_time(e1) / reps
            del graph
            nbytes = N * K // 2 + N * K // 16 + M * K // 2 + M * K // 16 + 2 * M * N
            out.append({"M": M, "N": N, "K": K, "us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1),
                        "frac_hbm": round(nbytes / us / 1e3 / pk["hbm_gbs"], 3), "us_eager": round(eager_us, 2),
                        "gbs_eager": round(nbytes / eager_us / 1e3, 1)})
        del ws
    nv.device_status()
    return {"unit": "GB/s", "peak_gbs": pk["hbm_gbs"], "peak_basis": pk["source"] + " HBM copy",
            "timing": "CUDA-graph replay of 30 back-to-back calls, weights rotating over 3 sets", "shapes": out}


def quantize_section(nv, dev, pk, reps=20):
    """Row a9-Q (bf16 -> NVFP4) and BASELINE configs[4] (fused quantize + GEMM on
    heavy-tailed activations): the quantizer's HBM rate on the 8192x8192 operand and
    the 4096x4096 activation, and the end-to-end device time of amax -> quantize ->
    GEMM against a pre-quantized W[14336, 4096].  Timed from CUDA-graph replays."""
    g = torch.Generator(device=dev)
    stream = torch.cuda.Stream(dev)
    res = {"unit": "GB/s", "peak_gbs": pk["hbm_gbs"]}
    for (M, K) in ((8192, 8192), (4096, 4096)):
        g.manual_seed(3)
        xs = [torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16) for _ in range(3)]
        gs = torch.full((1,), 1e-3, dtype=torch.float32, device=dev)
        q = torch.empty(M, K // 2, dtype=torch.uint8, device=dev)
        sf = torch.empty(nv.sf_bytes(M, K), dtype=torch.uint8, device=dev)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(3):
                nv.quantize(xs[i % 3], gs, q_out=q, sf_out=sf)
            stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(reps):
                nv.quantize(xs[i % 3], gs, q_out=q, sf_out=sf)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        us = 1e3 * e0.elapsed_time(e1) / reps
        nbytes = M * K * 2 + M * K // 2 + M * K // 16
        res[f"quantize_{M}x{K}"] = {"us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1),
                                    "frac_hbm": round(nbytes / us / 1e3 / pk["hbm_gbs"], 3)}
        del graph, xs
    # X[4096,4096] Student-t(3) with 4 outlier channels x50, W[14336,4096] N(0, 0.02)
    M, N, K = 4096, 14336, 4096
    g.manual_seed(9)
    z = torch.randn(M, K, device=dev, generator=g)
    chi = (torch.randn(3, M, K, device=dev, generator=g) ** 2).sum(0) / 3
    x = z / chi.sqrt()
    cols = torch.randperm(K, device=dev, generator=g)[:4]
    x[:, cols] *= 50
    x = x.to(torch.bfloat16)
    del z, chi
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    _, gsw = nv.global_scale(w)
    wq, wsf = nv.quantize(w, gsw)
    del w
    amax, gsx = torch.empty(1, device=dev), torch.empty(1, device=dev)
    xq = torch.empty(M, K // 2, dtype=torch.uint8, device=dev)
    xsf = torch.empty(nv.sf_bytes(M, K), dtype=torch.uint8, device=dev)
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    L = nv.lib()

    def two_pass():
        s = torch.cuda.current_stream(dev).cuda_stream
        L.nvfp4_global_scale(x.data_ptr(), x.numel(), amax.data_ptr(), gsx.data_ptr(), s)
        L.nvfp4_quantize(x.data_ptr(), xq.data_ptr(), xsf.data_ptr(), gsx.data_ptr(), M, K, s)
        # the GEMM's alpha would be gs_x * gs_w; gs_x lives on the device here and the
        # timing does not depend on alpha's value, so alpha = 1 is passed
        nv.gemm(xq, xsf, wq, wsf, 1.0, out=d)

    def one_pass():
        s = torch.cuda.current_stream(dev).cuda_stream
        L.nvfp4_quantize_dynamic(x.data_ptr(), xq.data_ptr(), xsf.data_ptr(), amax.data_ptr(), gsx.data_ptr(),
                                 M, K, s)
        nv.gemm(xq, xsf, wq, wsf, 1.0, out=d)

    def graph_us(fn):
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            fn()  # tensor maps and the stream's workspaces are made here
            stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return 1e3 * e0.elapsed_time(e1) / reps

    us2, us1 = graph_us(two_pass), graph_us(one_pass)
    res["fused_quantize_gemm_4096x14336x4096"] = {
        "us": round(us1, 2), "tflops": round(2.0 * M * N * K / us1 / 1e6, 1),
        "us_amax_then_quantize": round(us2, 2),
        "steps": "amax + quantize of X (bf16 Student-t, 4 outlier channels x50) in one cooperative kernel "
                 "(nvfp4_quantize_dynamic) + GEMM vs pre-quantized W; us_amax_then_quantize: the same with "
                 "nvfp4_global_scale and nvfp4_quantize as two steps"}
    nv.device_status()
    return res


def moe_section(nv, dev, reps=20):
    """Grouped (mixture-of-experts) GEMM: Mixtral-8x7B-like expert up-projection,
    8 experts N=14336 K=4096, 4096 tokens x top-2 = 8192 routed rows split by a
    seeded random routing; useful TFLOP/s (2 * sum M_g * N * K / time) beside one
    dense GEMM of the same total shape."""
    G, N, K, tokens, top = 8, 14336, 4096, 4096, 2
    g = torch.Generator().manual_seed(77)
    counts = torch.bincount(torch.randint(0, G, (tokens * top,), generator=g), minlength=G)
    offsets = [0] + torch.cumsum(counts, 0).tolist()
    m_total = offsets[-1]
    gen = torch.Generator(device=dev).manual_seed(78)
    x = torch.randn(m_total, K, device=dev, generator=gen).to(torch.bfloat16)
    _, gsx = nv.global_scale(x)
    offs = torch.tensor(offsets, dtype=torch.int32, device=dev)
    q, sf = nv.quantize_grouped(x, gsx, offs)
    bq = torch.empty(G * N, K // 2, dtype=torch.uint8, device=dev)
    bsf = torch.empty(G * nv.sf_bytes(N, K), dtype=torch.uint8, device=dev)
    alphas = torch.empty(G, dtype=torch.float32, device=dev)
    for e in range(G):
        w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        _, gw = nv.global_scale(w)
        nv.quantize(w, gw, q_out=bq[e * N:(e + 1) * N], sf_out=bsf[e * nv.sf_bytes(N, K):(e + 1) * nv.sf_bytes(N, K)])
        alphas[e:e + 1] = gsx * gw
    d = torch.empty(m_total, N, dtype=torch.bfloat16, device=dev)
    flops = 2.0 * m_total * N * K

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    stream = torch.cuda.Stream(dev)

    def graphed(fn):
        """Device time per call of fn with reps calls replayed from one CUDA graph (how
        a decode loop launches them: no host launch path between the kernels)."""
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()  # tensor maps and this stream's workspaces are made here
            stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps

    ms = timed(lambda: nv.gemm_grouped(q, sf, bq, bsf, alphas, offs, out=d))
    # the same total work as one dense GEMM (expert 0's weights for every row)
    dense_ms = timed(lambda: nv.gemm(q, sf[:nv.sf_bytes(m_total, K)], bq[:N], bsf[:nv.sf_bytes(N, K)], 1.0, out=d))
    nv.device_status()
    out = {"what": "grouped NVFP4 GEMM, 8 experts N=14336 K=4096, 8192 routed rows (4096 tokens x top-2)",
           "rows_per_expert": counts.tolist(), "ms": ms, "tflops": flops / (ms / 1e3) / 1e12,
           "dense_same_shape_ms": dense_ms, "dense_same_shape_tflops": flops / (dense_ms / 1e3) / 1e12}

    # Decode: 32 tokens x top-2 = 64 routed rows.  The grouped call (m_total <= 128:
    # the stream-K kernel over the active experts' weight tiles) is measured on HBM
    # bytes: each active expert's weights and scales read once (the 8 experts' 235 MB
    # exceed L2).  Beside it, one decode GEMM per active expert.
    dec_tokens = 32
    counts_d = torch.bincount(torch.randint(0, G, (dec_tokens * top,), generator=g), minlength=G)
    offs_d_host = [0] + torch.cumsum(counts_d, 0).tolist()
    m_d = offs_d_host[-1]
    offs_d = torch.tensor(offs_d_host, dtype=torch.int32, device=dev)
    qd, sfd = nv.quantize_grouped(x[:m_d], gsx, offs_d)
    dd = torch.empty(m_d, N, dtype=torch.bfloat16, device=dev)
    active = [e for e in range(G) if counts_d[e] > 0]
    w_bytes = len(active) * (N * K // 2 + nv.sf_bytes(N, K))
    dec_ms_eager = timed(lambda: nv.gemm_grouped(qd, sfd, bq, bsf, alphas, offs_d, out=dd))
    dec_ms = graphed(lambda: nv.gemm_grouped(qd, sfd, bq, bsf, alphas, offs_d, out=dd))
    blk0 = nv.grouped_sf_block0(offs_d_host)
    alpha_h = alphas.cpu().tolist()
    sf_blk = 128 * (K // 16)
    per_expert = [(offs_d_host[e], offs_d_host[e + 1], blk0[e]) for e in active]

    def loop():
        for e, (a0, a1, b0) in zip(active, per_expert):
            nv.gemm(qd[a0:a1], sfd[b0 * sf_blk:], bq[e * N:(e + 1) * N],
                    bsf[e * nv.sf_bytes(N, K):(e + 1) * nv.sf_bytes(N, K)], alpha_h[e], out=dd[a0:a1])

    loop_ms = graphed(loop)
    nv.device_status()
    out["decode"] = {"what": "grouped NVFP4 GEMM, 8 experts N=14336 K=4096, 64 routed rows (32 tokens x top-2)",
                     "timing": f"CUDA-graph replay of {reps} calls (ms_eager: launched one by one from Python)",
                     "rows_per_expert": counts_d.tolist(), "ms": dec_ms, "ms_eager": dec_ms_eager,
                     "weight_bytes": w_bytes, "hbm_gbs": w_bytes / (dec_ms / 1e3) / 1e9,
                     "per_expert_decode_calls_ms": loop_ms, "per_expert_hbm_gbs": w_bytes / (loop_ms / 1e3) / 1e9}

    # The expert FFN around the GEMM, SwiGLU form y = W2 (silu(W1 x) * W3 x): W1 and W3
    # interleaved in blocks of 16 rows into one [2 * 14336, 4096] weight per expert, so
    # one grouped GEMM with the SwiGLU epilogue writes the [rows, 14336] hidden state as
    # NVFP4 in the grouped scale layout, which the down-projection W2 [4096, 14336]
    # reads as its A operand.  Beside it the unfused sequence (bf16 SwiGLU output,
    # quantize_grouped, down-projection).
    del bq, bsf
    F = N
    wgu = torch.empty(G * 2 * F, K // 2, dtype=torch.uint8, device=dev)
    wgusf = torch.empty(G * nv.sf_bytes(2 * F, K), dtype=torch.uint8, device=dev)
    alphas_gu = torch.empty(G, dtype=torch.float32, device=dev)
    for e in range(G):
        w1 = (torch.randn(F, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn(F, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        w = nv.swiglu_interleave(w1, w3).contiguous()
        del w1, w3
        _, gw = nv.global_scale(w)
        sfb_e = nv.sf_bytes(2 * F, K)
        nv.quantize(w, gw, q_out=wgu[e * 2 * F:(e + 1) * 2 * F], sf_out=wgusf[e * sfb_e:(e + 1) * sfb_e])
        alphas_gu[e:e + 1] = gsx * gw
        del w
    wdq = torch.empty(G * K, F // 2, dtype=torch.uint8, device=dev)
    wdsf = torch.empty(G * nv.sf_bytes(K, F), dtype=torch.uint8, device=dev)
    gs_down = torch.empty(G, dtype=torch.float32, device=dev)  # each expert's W2 global scale
    for e in range(G):
        w = (torch.randn(K, F, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        _, gw = nv.global_scale(w)
        nv.quantize(w, gw, q_out=wdq[e * K:(e + 1) * K], sf_out=wdsf[e * nv.sf_bytes(K, F):(e + 1) * nv.sf_bytes(K, F)])
        gs_down[e:e + 1] = gw
        del w
    ffn = {"what": "Mixtral-like expert FFN, 8 experts: [W1;W3] interleaved (N=2x14336, K=4096) + SwiGLU -> "
                   "NVFP4 -> W2 (N=4096, K=14336)",
           "weight_bytes": G * (2 * F * K // 2 + nv.sf_bytes(2 * F, K) + K * F // 2 + nv.sf_bytes(K, F))}
    for name, (qq, ss, oo, mm) in (("prefill_8192_rows", (q, sf, offs, m_total)),
                                   ("decode_64_rows", (qd, sfd, offs_d, m_d))):
        h = nv.gemm_grouped_epilogue(qq, ss, wgu, wgusf, alphas_gu, oo, activation="swiglu")
        _, gh = nv.global_scale(h)  # the hidden state's global scale (calibrated once)
        alphas_d = gs_down * gh     # expert e's down-projection alpha: gs(h) * gs(W2[e])
        hq = torch.empty(mm, F // 2, dtype=torch.uint8, device=dev)
        hsf = torch.empty(nv.grouped_sf_bytes(mm, G, F), dtype=torch.uint8, device=dev)
        y = torch.empty(mm, K, dtype=torch.bfloat16, device=dev)

        def fused():
            nv.gemm_grouped_epilogue(qq, ss, wgu, wgusf, alphas_gu, oo, activation="swiglu", out_global_scale=gh,
                                     q_out=hq, sf_out=hsf)
            nv.gemm_grouped(hq, hsf, wdq, wdsf, alphas_d, oo, out=y)

        def unfused():
            nv.gemm_grouped_epilogue(qq, ss, wgu, wgusf, alphas_gu, oo, activation="swiglu", out=h)
            nv.quantize_grouped(h, gh, oo, q_out=hq, sf_out=hsf)
            nv.gemm_grouped(hq, hsf, wdq, wdsf, alphas_d, oo, out=y)

        if mm <= 128:
            # decode right after the prefill above runs at the clock the prefill's power
            # draw left (measured: 0.158 ms on an idle GPU, 0.20 ms after 60 ms of dense
            # GEMMs); measured after a pause, with the right-after figure beside it
            hot_ms = graphed(fused)
            time.sleep(0.5)
        f_ms, u_ms = timed(fused), timed(unfused)
        flops_ffn = 2.0 * mm * K * (2 * F + F)
        ffn[name] = {"fused_ms": f_ms, "unfused_ms": u_ms, "fused_tflops": flops_ffn / (f_ms / 1e3) / 1e12,
                     "fused_weight_gbs": ffn["weight_bytes"] / (f_ms / 1e3) / 1e9}
        if mm <= 128:  # decode: the host launch path is comparable to the kernels
            ffn[name]["fused_ms_eager"], ffn[name]["unfused_ms_eager"] = f_ms, u_ms
            time.sleep(0.5)
            f_ms, u_ms = graphed(fused), graphed(unfused)
            ffn[name].update({"timing": f"CUDA-graph replay of {reps} calls, after a 0.5 s pause",
                              "fused_ms": f_ms, "unfused_ms": u_ms,
                              "fused_tflops": flops_ffn / (f_ms / 1e3) / 1e12,
                              "fused_weight_gbs": ffn["weight_bytes"] / (f_ms / 1e3) / 1e9,
                              "fused_ms_right_after_prefill": hot_ms})
    nv.device_status()
    out["ffn"] = ffn
    return out


def epilogue_section(nv, sets, M, N, K, reps=30):
    """Cost of the fused epilogue at 8192^3: plain bf16 GEMM, GEMM + bias + SiLU with
    NVFP4 output (the next layer's operand), and the unfused sequence (GEMM with
    bias + SiLU in bf16, then nvfp4_quantize)."""
    a, sfa, b, sfb, alpha = sets[0]
    dev = a.device
    bias = torch.zeros(N, dtype=torch.bfloat16, device=dev)
    gs = torch.tensor([1e-3], dtype=torch.float32, device=dev)
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    q = torch.empty(M, N // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(nv.sf_bytes(M, N), dtype=torch.uint8, device=dev)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    plain = timed(lambda: nv.gemm(a, sfa, b, sfb, alpha, out=d))
    fused = timed(lambda: nv.gemm_epilogue(a, sfa, b, sfb, alpha, bias=bias, activation="silu",
                                           out_global_scale=gs, q_out=q, sf_out=sf))

    def unfused():
        nv.gemm_epilogue(a, sfa, b, sfb, alpha, bias=bias, activation="silu", out=d)
        nv.quantize(d, gs, q_out=q, sf_out=sf)

    two = timed(unfused)
    nv.device_status()
    return {"what": "8192^3 GEMM: plain bf16 / bias+SiLU+NVFP4-out fused / bias+SiLU bf16 then nvfp4_quantize",
            "plain_ms": plain, "fused_nvfp4_out_ms": fused, "unfused_ms": two}


def gather_section(nv, dev, world, rank, reps=10):
    """BASELINE configs[3], N-sharded, strong scaling: prefill FFN up-projection
    M=16384, N=28672, K=8192 (7.7e15 FLOP in all), B sharded by 128-row blocks across
    the ranks.  Per call, max over ranks: the shard GEMM alone (at one GPU the whole
    GEMM, the first point of the curve); and with the full output requested on every
    rank (N > 1): GEMM + NCCL all-gather of the bf16 shards
    (nvfp4_b200.dist.gather_columns), and the gather fused into the GEMM epilogue
    (nvfp4_b200.dist.FusedGather, NVLink stores to every rank's buffer)."""
    import torch.distributed as dist
    from nvfp4_b200.dist import FusedGather, gather_columns, shard_bounds
    M, N, K = 16384, 28672, 8192
    g = torch.Generator(device=dev).manual_seed(91)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    _, gx = nv.global_scale(x)
    a, sfa = nv.quantize(x, gx)
    del x
    n0, n1 = shard_bounds(N, world, rank)
    w = (torch.randn(n1 - n0, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    _, gw = nv.global_scale(w)
    bs, ss = nv.quantize(w, gw)
    del w
    alpha = float((gx * gw).item())

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / reps, world)

    d = torch.empty(M, n1 - n0, dtype=torch.bfloat16, device=dev)
    res = {"what": "prefill FFN M=16384 N=28672 K=8192, N-sharded across the GPUs (strong scaling); with the "
                   "full output, bf16 D [16384, 28672] on every rank",
           "full_output_bytes": M * N * 2, "n_gpus": world, "shard_columns": n1 - n0}
    res["shard_gemm_ms"] = timed(lambda: nv.gemm(a, sfa, bs, ss, alpha, out=d))
    if world > 1:
        res["gemm_plus_nccl_all_gather_ms"] = timed(
            lambda: gather_columns(nv.gemm(a, sfa, bs, ss, alpha, out=d), N))
        fg = FusedGather(M, N, dev, multicast=False)
        res["fused_nvlink_stores_ms"] = timed(lambda: fg.gemm(a, sfa, bs, ss, alpha, n0))
        del fg
        dist.barrier()
    nv.device_status()
    flops = 2.0 * M * N * K
    for k in [k for k in res if k.endswith("_ms") and res[k]]:
        res[k.replace("_ms", "_tflops")] = flops / (res[k] / 1e3) / 1e12
    # Roofline of the full-output forms: the slower of this rank's shard GEMM and the
    # NVLink bytes every rank must receive ((P-1)/P of the output) at the measured
    # 770 GB/s per direction of a peer copy on this pool.
    in_bytes = M * N * 2 * (world - 1) / world
    link_ms = in_bytes / 770e9 * 1e3
    bound_ms = max(link_ms, res["shard_gemm_ms"])
    res["roofline"] = {"bound": "nvlink" if link_ms >= res["shard_gemm_ms"] else "tensor",
                       "limiter": ("incoming NVLink bytes of the gather" if link_ms >= res["shard_gemm_ms"]
                                   else "the shard GEMM (tensor pipe)"),
                       "nvlink_in_bytes_per_rank": in_bytes, "nvlink_gbs_basis": 770.0, "bound_ms": bound_ms}
    if world > 1:
        res["roofline"]["frac_fused_stores"] = bound_ms / res["fused_nvlink_stores_ms"]
    del a, sfa, bs, ss, d
    res["down_proj"] = gather_down_proj(nv, dev, world, rank, timed)
    return res


def gather_down_proj(nv, dev, world, rank, timed):
    """BASELINE configs[3]'s down-projection, N-sharded the same way: H [16384, 28672]
    (the up-projection's width) times W_down [8192, 28672], 7.7e15 FLOP in all."""
    from nvfp4_b200.dist import FusedGather, gather_columns, shard_bounds
    M, N, K = 16384, 8192, 28672
    g = torch.Generator(device=dev).manual_seed(93)
    h = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    _, gh = nv.global_scale(h)
    a, sfa = nv.quantize(h, gh)
    del h
    n0, n1 = shard_bounds(N, world, rank)
    w = (torch.randn(n1 - n0, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    _, gw = nv.global_scale(w)
    bs, ss = nv.quantize(w, gw)
    del w
    alpha = float((gh * gw).item())
    d = torch.empty(M, n1 - n0, dtype=torch.bfloat16, device=dev)
    res = {"what": "prefill FFN down-projection M=16384 N=8192 K=28672, N-sharded; with the full output, "
                   "bf16 D [16384, 8192] on every rank", "shard_columns": n1 - n0}
    res["shard_gemm_ms"] = timed(lambda: nv.gemm(a, sfa, bs, ss, alpha, out=d))
    if world > 1:
        res["gemm_plus_nccl_all_gather_ms"] = timed(
            lambda: gather_columns(nv.gemm(a, sfa, bs, ss, alpha, out=d), N))
        fg = FusedGather(M, N, dev, multicast=False)
        res["fused_nvlink_stores_ms"] = timed(lambda: fg.gemm(a, sfa, bs, ss, alpha, n0))
        del fg
        torch.distributed.barrier()
    nv.device_status()
    flops = 2.0 * M * N * K
    for k in [k for k in res if k.endswith("_ms") and res[k]]:
        res[k.replace("_ms", "_tflops")] = flops / (res[k] / 1e3) / 1e12
    return res


def run_moe_workload(args):
    """The mixture-of-experts section alone (grouped prefill and decode, the SwiGLU
    expert FFN), one JSON line: for profiling its kernels."""
    import nvfp4_b200 as nv
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    res = moe_section(nv, dev)
    print(json.dumps({"workload": "moe", **res}), flush=True)
    return 0


def run_decode_workload(args, M, N, K):
    """One skinny-M shape alone (for profiling): weights rotate over 3 sets."""
    import nvfp4_b200 as nv
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    ws = []
    for i in range(3):
        g.manual_seed(77 + i)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        _, gs = nv.global_scale(w)
        ws.append(nv.quantize(w, gs))
        del w
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    _, gsx = nv.global_scale(x)
    xq, xsf = nv.quantize(x, gsx)
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    for i in range(args.warmup):
        nv.gemm(xq, xsf, ws[i % 3][0], ws[i % 3][1], 1.0, out=d)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        nv.gemm(xq, xsf, ws[i % 3][0], ws[i % 3][1], 1.0, out=d)
    e1.record(stream)
    torch.cuda.synchronize()
    nv.device_status()
    us = 1e3 * e0.elapsed_time(e1) / args.steps
    nbytes = N * K // 2 + N * K // 16 + M * K // 2 + M * K // 16 + 2 * M * N
    print(json.dumps({"metric": "decode NVFP4 GEMM HBM GB/s", "value": nbytes / us / 1e3, "unit": "GB/s",
                      "us_per_call": us, "config": {"M": M, "N": N, "K": K}, "steps": args.steps}), flush=True)
    return 0


def run_quantize_workload(args, M, K):
    """The quantizer alone (for profiling): bf16 N(0,1) X [M, K], 3 rotating inputs."""
    import nvfp4_b200 as nv
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    xs = [torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16) for _ in range(3)]
    gs = torch.full((1,), 1e-3, dtype=torch.float32, device=dev)
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(nv.sf_bytes(M, K), dtype=torch.uint8, device=dev)
    for i in range(args.warmup):
        nv.quantize(xs[i % 3], gs, q_out=q, sf_out=sf)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        nv.quantize(xs[i % 3], gs, q_out=q, sf_out=sf)
    e1.record(stream)
    torch.cuda.synchronize()
    us = 1e3 * e0.elapsed_time(e1) / args.steps
    nbytes = M * K * 2 + M * K // 2 + M * K // 16
    print(json.dumps({"metric": "bf16 -> NVFP4 quantize HBM GB/s", "value": nbytes / us / 1e3, "unit": "GB/s",
                      "us_per_call": us, "config": {"M": M, "K": K}, "steps": args.steps}), flush=True)
    return 0


def run_ours(args):
    import nvfp4_b200 as nv
    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    M, N, K = M_, N_, K_
    flops = 2.0 * M * N * K
    in_bytes = M * K // 2 + N * K // 2 + nv.sf_bytes(M, K) + nv.sf_bytes(N, K)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    n_sets = args.sets if args.sets else max(2, -(-3 * l2 // in_bytes))
    sets = make_operand_sets(nv, n_sets, M, N, K, seed=1234 + 7919 * rank, dev=dev)
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        a, sfa, b, sfb, alpha = sets[i % n_sets]
        nv.gemm(a, sfa, b, sfb, alpha, out=d)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    nv.device_status()
    # the SM clock the GEMM runs at as the timed region starts (one traced launch)
    in_kernel_before = in_kernel_clock(nv, sets[0], d, M, N, K, dev)

    # ---- timed region: device time with CUDA events on the launching stream, one pair
    # around the K steps (an event recorded between two GEMMs would keep the second
    # from starting its set-up while the first finishes, as back-to-back GEMMs do)
    launches0 = nv.launch_count()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        barrier(world)
        torch.cuda.synchronize()
        e_start.record(stream)
        for i in range(args.steps):
            step(i)
        e_end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    launches = nv.launch_count() - launches0
    nv.device_status()
    in_kernel_after = in_kernel_clock(nv, sets[0], d, M, N, K, dev)
    local_ms = e_start.elapsed_time(e_end)
    total_ms = max_over_ranks(local_ms, world)
    ms_step = total_ms / args.steps
    value = flops * world * args.steps / (total_ms / 1e3) / 1e12
    kernel_ms = local_ms / args.steps  # this rank's mean time per GEMM launch
    achieved = flops / (kernel_ms / 1e3) / 1e12

    # ---- end to end through the public API from pinned host buffers: nvfp4_gemm_host
    # uploads A, SFA, B, SFB, runs the GEMM block by block and copies D back, the
    # transfers overlapped with each other and with the compute
    a, sfa, b, sfb, alpha = sets[0]
    host_in = [t.cpu().pin_memory() for t in (a, sfa, b, sfb)]
    host_out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out.numel() * host_out.element_size()

    call_streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]

    def e2e_step(i, serial=False):
        # steps go to two caller streams in turn, as a serving loop would issue them:
        # each call is ordered on its own stream, so a step's uploads and GEMMs overlap
        # the previous step's download (serial: every step on one stream)
        with torch.cuda.stream(stream if serial else call_streams[i % 2]):
            nv.gemm_host(host_in[0], host_in[1], host_in[2], host_in[3], alpha, host_out, device=dev)

    def e2e_timed(steps, serial):
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for cs in call_streams:
            cs.wait_stream(stream)
        for i in range(steps):
            e2e_step(i, serial)
        for cs in call_streams:
            stream.wait_stream(cs)
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), world) / steps

    e2e_ms = e2e_value = e2e_serial_ms = None
    if not args.no_e2e:
        e2e_steps = max(4, min(args.steps, 20))
        for i in range(4):
            e2e_step(i)
        e2e_ms = e2e_timed(e2e_steps, serial=False)
        e2e_value = flops * world / (e2e_ms / 1e3) / 1e12
        e2e_serial_ms = e2e_timed(max(3, e2e_steps // 2), serial=True)
        barrier(world)

    pk = peaks()
    fp4_peak_est = 4.0 * pk["bf16_tflops"]
    traffic = committed_traffic().get("gemm_8192", {}).get("dram_bytes_per_launch")
    cpu = None
    vendor = vendor_scaled_mm(sets, M, N, K) if rank == 0 else None
    decode = quant = moe = epi = None
    if not args.no_decode:
        decode = decode_section(nv, dev, pk)
        quant = quantize_section(nv, dev, pk)
        moe = moe_section(nv, dev)
        epi = epilogue_section(nv, sets, M, N, K)
    gath = gather_section(nv, dev, world, rank) if not args.no_gather else None
    sweep = shape_sweep_section(nv, dev) if (rank == 0 and not args.no_sweep) else None
    # last of the GPU sections: a second of GEMMs at the power cap leaves the clocks low
    # for a while, which would slow whatever is measured after it
    sustained = sustained_section(nv, sets, d, M, N, K, dev) if not args.no_sustained else None
    cpu_cfg = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu, _, _ = cpu_reference_sample(a, sfa, b, sfb, alpha, M, N, K, target_s=args.cpu_seconds)
        cpu_cfg = cpu_configs_section()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp4(e2m1)xfp4->fp32",
            "data": "synthetic: bf16 N(0,1) drawn on device (seeded), quantized by nvfp4_quantize",
            "config": {"workload": "square NVFP4 GEMM M=N=K=8192 per GPU (BASELINE configs[1])",
                       "M": M, "N_per_gpu": N, "K": K, "out": "bf16", "alpha": "gsA*gsB",
                       "parallelism": f"column-parallel N shards x{world}",
                       "l2": f"rotating {n_sets} operand sets of {in_bytes / 1e6:.1f} MB (> 3x L2)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp4_peak_est, "unit": "TFLOP/s",
                         "frac": achieved / fp4_peak_est, "traffic": traffic,
                         "peak_basis": f"4 x {pk['source']} dense bf16 ({pk['bf16_tflops']} TFLOP/s): FP4 "
                                       "tensor rate is 4x bf16 per SM; no FP4 peak is measured on this pool",
                         "frac_of_nominal_9000": achieved / 9000.0,
                         "kernel_ms": kernel_ms, "flops_per_launch": flops},
            "gpu_launches": int(launches),
            "clocks": dict(clk.summary(), in_kernel_sm_mhz=in_kernel_before,
                           in_kernel_sm_mhz_after=in_kernel_after,
                           in_kernel_note="SM cycles (clock64) / ns (globaltimer) of the MMA thread over one "
                                          "traced launch of the same GEMM right before the timed region (after "
                                          "warm-up) and right after it; the 1 kW power cap can lower the clock "
                                          "after a long run of these GEMMs"),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "ms_per_step": e2e_ms,
                    "path": "pinned host -> nvfp4_gemm_host -> pinned host; steps on two caller streams in turn "
                            "(each step's uploads and GEMMs overlap the previous step's download)",
                    "ms_per_step_one_stream": e2e_serial_ms,
                    "bound": "host link: the step's copies, not the GEMM (the device-timed GEMM is ~7 % of it)",
                    "host_link_gbs": ((h2d + d2h) / (e2e_ms / 1e3) / 1e9) if e2e_ms else None,
                    "gemm_share": (kernel_ms / e2e_ms) if e2e_ms else None},
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if cpu_cfg is not None:
            line["cpu_configs"] = cpu_cfg
        if vendor is not None:
            line["vendor_scaled_mm"] = vendor
        if decode is not None:
            line["decode"] = decode
        if quant is not None:
            line["quantize"] = quant
        if moe is not None:
            line["moe_grouped"] = moe
        if epi is not None:
            line["fused_epilogue"] = epi
        if gath is not None:
            line["gather"] = gath
        if sustained is not None:
            line["sustained"] = sustained
        if sweep is not None:
            line["shape_sweep"] = sweep
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)  # ~40 ms timed: room for clock samples
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--sets", type=int, default=0, help="operand sets to rotate (default: > 3x L2)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode-shape GB/s section")
    ap.add_argument("--no-gather", action="store_true", help="skip the configs[3] N-sharded section")
    ap.add_argument("--no-sustained", action="store_true", help="skip the >= 1 s sustained GEMM loop")
    ap.add_argument("--no-sweep", action="store_true", help="skip the reference harness's shape sweep")
    ap.add_argument("--workload", default="square",
                    help="square (default, the bench line), decode:M:N:K or quantize:M:K (one kernel, for "
                         "profiling), moe (the mixture-of-experts section alone)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload.startswith("decode:"):
        M, N, K = (int(v) for v in args.workload.split(":")[1:])
        return run_decode_workload(args, M, N, K)
    if args.workload == "moe":
        return run_moe_workload(args)
    if args.workload.startswith("quantize:"):
        M, K = (int(v) for v in args.workload.split(":")[1:])
        return run_quantize_workload(args, M, K)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
