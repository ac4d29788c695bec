"""Diagnostics for the NVFP4 kernels on a B200.

    python -m nvfp4_diag probe [iters]        measured mxf4nvf4 tensor rate per issue mode
    python -m nvfp4_diag trace M N K [reps] [epi]  per-CTA cycle breakdown of the CTA-pair GEMM (last
                                              of reps); epi: one of EPILOGUES (fused epilogue)
    python -m nvfp4_diag decode M N K          timeline of back-to-back decode GEMMs (graph replay)

(run with gpu-kernels_b200/ on sys.path).  Each prints JSON lines.  Everything here
runs the diagnostic library (libnvfp4_diag.so), never the product one.
"""
import ctypes as C
import json
import statistics
import sys

import torch

from nvfp4_diag import check, lib

PROBE_MODES = {0: "single-CTA MMA only", 1: "single-CTA MMA + 3 scale copies each",
               2: "CTA-pair MMA only", 3: "CTA-pair MMA + 3 scale copies each",
               4: "CTA-pair, 12 scale copies per 4-MMA stage first",
               5: "CTA-pair N=192 + 3 scale copies each",
               6: "CTA-pair, 3 scale copies per iteration, no MMA (issue cost)",
               7: "CTA-pair N=64 MMA only (issue cost)",
               8: "CTA-pair N=64 MMA + 2 commits (issue cost)",
               9: "CTA-pair 3 copies + N=64 MMA + 2 commits (issue cost)",
               10: "as 4, pseudo-random operands and scales",
               11: "as 2 (MMA only), pseudo-random operands and scales"}


def probe(iters: int = 20000):
    out = []
    for mode, name in PROBE_MODES.items():
        tf, cyc = C.c_double(), C.c_double()
        check(lib().nvfp4_probe_mma_rate(mode, iters, C.byref(tf), C.byref(cyc)), "probe")
        out.append({"mode": mode, "what": name, "tflops": round(tf.value, 1),
                    "cycles_per_mma": round(cyc.value, 2)})
    return out


# Fused epilogues the trace can run: (activation, bias, NVFP4 output)
EPILOGUES = {"none": ("none", False, False), "relu_bf16": ("relu", False, False),
             "silu_bf16": ("silu", False, False), "bias_silu_bf16": ("silu", True, False),
             "gelu_bf16": ("gelu_tanh", False, False), "fp4": ("none", False, True),
             "bias_silu_fp4": ("silu", True, True)}


def trace(M: int, N: int, K: int, reps: int = 3, epi: str = "none"):
    """Per-CTA cycle breakdown of the CTA-pair kernel (the last of `reps` launches),
    plus the kernel's event time and where the time outside the MMA span goes; with
    `epi`, the same launch with that fused epilogue."""
    from nvfp4_b200._lib import ACTIVATIONS, Epilogue
    from nvfp4_b200.layout import sf_bytes
    from nvfp4_b200.ops import create_tensors
    _l = lib
    slots = 16
    dev = torch.device("cuda", 0)
    a, b, sfa, sfb = create_tensors(M, N, K, seed=1)
    sfa = torch.full_like(sfa, 0x38)
    sfb = torch.full_like(sfb, 0x38)
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    act, with_bias, fp4 = EPILOGUES[epi]
    bias = torch.zeros(N, dtype=torch.bfloat16, device=dev)
    q = torch.empty(M, N // 2, dtype=torch.uint8, device=dev)
    sfo = torch.empty(sf_bytes(M, N), dtype=torch.uint8, device=dev)
    gs = torch.tensor([1e-3], dtype=torch.float32, device=dev)
    E = Epilogue(bias=bias.data_ptr() if with_bias else None, activation=ACTIVATIONS[act],
                 q_out=q.data_ptr() if fp4 else None, sf_out=sfo.data_ptr() if fp4 else None,
                 out_global_scale=gs.data_ptr() if fp4 else None)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count  # one trace row per CTA, grid <= #SMs
    tr = torch.zeros(sms * slots, dtype=torch.int64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(reps):
        if i == reps - 1:
            e0.record()
        check(_l().nvfp4_gemm_trace_epilogue(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), 1.0,
                                             d.data_ptr(), M, N, K, C.byref(E), tr.data_ptr(), s), "trace")
    e1.record()
    torch.cuda.synchronize()
    t = tr.view(sms, slots).cpu()
    ctas = int((t[:, 8] > 0).sum())
    t = t[:ctas]
    leaders = t[0::2]
    span = leaders[:, 6].double()
    rows = {"mma_wait_full": leaders[:, 0], "mma_wait_acc": leaders[:, 1], "producer_wait_empty": t[:, 2],
            "epi_wait_acc_full": t[:, 3], "epi_drain_store": t[:, 4]}
    res = {"M": M, "N": N, "K": K, "epilogue": epi, "event_us": e0.elapsed_time(e1) * 1e3,
           "tiles_per_pair": statistics.mean(leaders[:, 5].tolist()),
           "mma_span_cycles": statistics.mean(span.tolist()),
           "sm_clock_mhz": statistics.mean((leaders[:, 6].double() / leaders[:, 7].double() * 1e3).tolist())}
    for k, v in rows.items():
        res[k + "_cycles"] = statistics.mean(v.double().tolist())
        res[k + "_frac_of_span"] = res[k + "_cycles"] / res["mma_span_cycles"]
    t0 = int(t[:, 8].min())
    us = lambda x: float(x) / 1e3  # noqa: E731
    res.update({
        "cta_span_us": us(t[:, 9].max() - t0),                      # first CTA entry -> last CTA exit
        "entry_spread_us": us(t[:, 8].max() - t0),                  # launch skew across CTAs
        "prologue_us": us((leaders[:, 10] - leaders[:, 8]).double().mean()),  # entry -> first MMA issue
        "mma_span_us_mean": us(leaders[:, 7].double().mean()),
        "last_commit_min_us": us(leaders[:, 11].min() - t0),         # tail imbalance across pairs
        "last_commit_max_us": us(leaders[:, 11].max() - t0),
        "epilogue_tail_us": us((leaders[:, 9] - leaders[:, 11]).double().mean()),  # last commit -> CTA exit
    })
    # accumulator hand-off between tiles 2 and 3 of each pair (%globaltimer ns; pairs
    # with fewer than 4 tiles have no sample)
    sel = (leaders[:, 13] > 0) & (leaders[:, 14] > 0)
    hs, peers = leaders[sel].double(), t[1::2][sel].double()
    if len(hs):
        last_read = torch.maximum(hs[:, 15], peers[:, 15])
        res["handoff_sample_ns"] = {
            "pairs": len(hs),
            "first_slot_landed_after_leader_wake": float((hs[:, 12] - hs[:, 14]).mean()),
            "peer_wake_after_leader": float((peers[:, 14] - hs[:, 14]).mean()),
            "leader_read": float((hs[:, 15] - hs[:, 14]).mean()),  # wake -> last warp read out
            "peer_read": float((peers[:, 15] - peers[:, 14]).mean()),
            "last_read_to_mma_resume": float((hs[:, 13] - last_read).mean()),  # arrivals -> MMA thread
            "leader_wake_to_mma_resume": float((hs[:, 13] - hs[:, 14]).mean()),
        }
    return res


def decode_trace(M: int, N: int, K: int, calls: int = 8, sets: int = 3):
    """Timeline of `calls` back-to-back decode GEMMs replayed from a CUDA graph (weights
    rotating over `sets` copies, as in bench.py's decode section), from the kernel's
    per-CTA %globaltimer stamps.  Per call, in us: gap from the previous call's last
    CTA exit to this call's wait release, first data after release, streaming span,
    tail (last data to last exit), and the call's period."""
    from nvfp4_b200.ops import create_tensors
    _l = lib
    dev = torch.device("cuda", 0)
    ops = [create_tensors(M, N, K, seed=10 + i) for i in range(sets)]
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    ws_bytes = _l().nvfp4_gemm_decode_workspace_size(M, N)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    grid = torch.cuda.get_device_properties(dev).multi_processor_count  # grid <= #SMs
    slots = 9
    tr = torch.zeros(calls, grid * slots, dtype=torch.int64, device=dev)
    s = torch.cuda.Stream()

    def launch(c):
        a, b, sfa, sfb = ops[c % sets]
        check(_l().nvfp4_gemm_decode_trace(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), 1.0,
                                           d.data_ptr(), M, N, K, ws.data_ptr(), ws_bytes, tr[c].data_ptr(),
                                           s.cuda_stream), "decode trace")

    with torch.cuda.stream(s):
        for c in range(calls):
            launch(c)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for c in range(calls):
                launch(c)
    with torch.cuda.stream(s):
        g.replay()
    torch.cuda.synchronize()
    tr.zero_()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    del g
    t = tr.view(calls, grid, slots).cpu()
    used = t[0, :, 0] > 0
    t = t[:, used]
    t0 = int(t[0, :, 0].min())
    us = lambda x: round(float(x) / 1e3, 2)  # noqa: E731
    rows = []
    for c in range(calls):
        tc = t[c]
        row = {"call": c, "entry_first": us(tc[:, 0].min() - t0), "release_first": us(tc[:, 1].min() - t0),
               "release_last": us(tc[:, 1].max() - t0), "first_data_first": us(tc[:, 2].min() - t0),
               "first_data_last": us(tc[:, 2].max() - t0), "last_data_first": us(tc[:, 3].min() - t0),
               "last_data_last": us(tc[:, 3].max() - t0), "exit_last": us(tc[:, 4].max() - t0)}
        if c:
            row["gap_prev_exit_to_release"] = us(tc[:, 1].min() - t[c - 1, :, 4].max())
            row["period"] = us(tc[:, 4].max() - t[c - 1, :, 4].max())
        rows.append(row)
    iters = t[0, :, 5]
    # per-CTA phases of one steady-state call, as percentiles over CTAs (us)
    c = t[calls // 2].double()
    q = torch.tensor([0.0, 0.1, 0.5, 0.9, 1.0], dtype=torch.float64)
    pct = lambda x: [round(v, 2) for v in (torch.quantile(x, q) / 1e3).tolist()]  # noqa: E731
    per_cta = {"percentiles": [0, 10, 50, 90, 100],
               "release_to_first_data": pct(c[:, 2] - c[:, 1]),
               "first_to_last_data": pct(c[:, 3] - c[:, 2]),
               "last_data_to_exit": pct(c[:, 4] - c[:, 3]),
               "entry_to_release": pct(c[:, 1] - c[:, 0]),
               "release_after_first_release": pct(c[:, 1] - c[:, 1].min()),
               "exit_after_first_exit": pct(c[:, 4] - c[:, 4].min())}
    # the last segment's epilogue: last data -> accumulator in registers -> arrival
    # counted -> partials summed (the tile's last contributor) -> CTA exit
    cut = c[:, 7] > 0
    fin = c[:, 8] > 0
    if cut.any():
        per_cta["last_data_to_acc_regs"] = pct(c[cut, 6] - c[cut, 3])
        per_cta["acc_regs_to_counted"] = pct(c[cut, 7] - c[cut, 6])
    if fin.any():
        per_cta["finisher_counted_to_summed"] = pct(c[fin, 8] - c[fin, 7])
        per_cta["finisher_summed_to_exit"] = pct(c[fin, 4] - c[fin, 8])
    nonfin = cut & ~fin
    if nonfin.any():
        per_cta["nonfinisher_counted_to_exit"] = pct(c[nonfin, 4] - c[nonfin, 7])
    tail = ((c[:, 4] - c[:, 3]) / 1e3).tolist()
    slow = [i for i, x in enumerate(tail) if x > 2.0]
    per_cta["slow_tail_ctas"] = slow
    return {"M": M, "N": N, "K": K, "ctas": int(used.sum()), "iters_per_cta": [int(iters.min()), int(iters.max())],
            "graph_us_per_call": e0.elapsed_time(e1) * 1e3 / calls, "per_cta": per_cta, "calls": rows}


def main(argv):
    if argv and argv[0] == "decode":
        M, N, K = (int(x) for x in argv[1:4])
        print(json.dumps(decode_trace(M, N, K)))
        return 0
    if not argv or argv[0] not in ("probe", "trace"):
        print(__doc__)
        return 2
    if argv[0] == "probe":
        for r in probe(int(argv[1]) if len(argv) > 1 else 20000):
            print(json.dumps(r))
    else:
        M, N, K = (int(x) for x in argv[1:4])
        reps = int(argv[4]) if len(argv) > 4 else 3
        print(json.dumps(trace(M, N, K, reps, argv[5] if len(argv) > 5 else "none")))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
