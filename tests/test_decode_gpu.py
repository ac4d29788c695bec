"""GPU parity: the stream-K / swap-AB decode GEMM (M <= 128) against the CPU oracle,
its determinism and workspace reuse, and the nvfp4_gemm dispatch between kernels."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def dev_t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def operands(oracle, M, N, K, seed):
    xa = oracle.normal_bf16((M, K), seed=seed)
    xb = oracle.normal_bf16((N, K), seed=seed + 1, std=0.02)
    ga, gb = oracle.global_scale_for(oracle.amax_bf16(xa)), oracle.global_scale_for(oracle.amax_bf16(xb))
    a, sfa = oracle.quantize(xa, ga)
    b, sfb = oracle.quantize(xb, gb)
    return a, sfa, b, sfb, float(np.float32(ga) * np.float32(gb))


def decode_call(nv, dev, a, sfa, b, sfb, alpha, M, N, K, ws=None):
    L = nv.lib()
    need = L.nvfp4_gemm_decode_workspace_size(M, N)
    assert need > 0
    if ws is None:
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
    ta, tsa, tb, tsb = (dev_t(t, dev) for t in (a, sfa, b, sfb))
    st = L.nvfp4_gemm_decode(ta.data_ptr(), tsa.data_ptr(), tb.data_ptr(), tsb.data_ptr(), alpha, out.data_ptr(),
                             M, N, K, ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    assert st == 0, nv.lib().nvfp4_status_string(st)
    torch.cuda.synchronize()
    nv.device_status()
    return out, ws


def rel_err(oracle, out, a, sfa, b, sfb, alpha, M, N, K):
    _, d16 = oracle.gemm(a, sfa, b, sfb, alpha, M, N, K)
    ref = oracle.bf16_bits_to_f32(d16).reshape(M, N)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.mark.parametrize("M,N,K", [
    (1, 1024, 8192), (16, 2048, 8192), (64, 1024, 4096), (128, 512, 2048),
    (16, 1024, 28672),   # every tile split across many CTAs (stream-K fix-up path)
    (3, 136, 320),       # ragged N, odd M, partial last k-stage
    (9, 8, 64),          # smallest legal shape
    (33, 4096, 1024),
    (16, 149 * 128, 512),  # one cut tile of 2 k-blocks over 148 CTAs: most stream-K ranges empty
])
def test_decode_parity(nv, oracle, cuda_dev, M, N, K):
    a, sfa, b, sfb, alpha = operands(oracle, M, N, K, seed=M * 31 + N)
    out, _ = decode_call(nv, cuda_dev, a, sfa, b, sfb, alpha, M, N, K)
    assert rel_err(oracle, out, a, sfa, b, sfb, alpha, M, N, K) <= TOL


def test_decode_full_w1_shape(nv, oracle, cuda_dev):
    """BASELINE config 3 weight W1 [28672, 8192] N(0,0.02) with M = 16 activations."""
    M, N, K = 16, 28672, 8192
    a, sfa, b, sfb, alpha = operands(oracle, M, N, K, seed=3)
    out, _ = decode_call(nv, cuda_dev, a, sfa, b, sfb, alpha, M, N, K)
    assert rel_err(oracle, out, a, sfa, b, sfb, alpha, M, N, K) <= TOL


def test_decode_deterministic_and_workspace_reusable(nv, oracle, cuda_dev):
    M, N, K = 16, 2048, 28672
    a, sfa, b, sfb, alpha = operands(oracle, M, N, K, seed=5)
    out1, ws = decode_call(nv, cuda_dev, a, sfa, b, sfb, alpha, M, N, K)
    n_tiles = (N + 127) // 128
    counters = ws[: n_tiles * 4].view(torch.int32)
    assert int(counters.abs().sum()) == 0, "arrival counters must be left at zero"
    out2, _ = decode_call(nv, cuda_dev, a, sfa, b, sfb, alpha, M, N, K, ws=ws)
    assert torch.equal(out1, out2), "stream-K fix-up must be deterministic"


def test_decode_rejects_small_workspace(nv, cuda_dev):
    L = nv.lib()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda_dev)
    p = buf.data_ptr()
    st = L.nvfp4_gemm_decode(p, p, p, p, 1.0, p, 16, 28672, 8192, p, 1024, None)
    assert st == -7
    st = L.nvfp4_gemm_decode(p, p, p, p, 1.0, p, 200, 256, 256, p, buf.numel(), None)
    assert st == -2  # M > 128 belongs to the persistent kernel


@pytest.mark.parametrize("M", [1, 16, 128, 129])
def test_gemm_dispatch_matches_persistent(nv, oracle, cuda_dev, M):
    """nvfp4_gemm (decode kernel for M <= 128) and nvfp4_gemm_persistent agree with
    the oracle on the same operands."""
    N, K = 1024, 2048
    a, sfa, b, sfb, alpha = operands(oracle, M, N, K, seed=M)
    ta, tsa, tb, tsb = (dev_t(t, cuda_dev) for t in (a, sfa, b, sfb))
    d1 = nv.gemm(ta, tsa, tb, tsb, alpha)
    d2 = torch.empty_like(d1)
    st = nv.lib().nvfp4_gemm_persistent(ta.data_ptr(), tsa.data_ptr(), tb.data_ptr(), tsb.data_ptr(), alpha,
                                        d2.data_ptr(), M, N, K, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert rel_err(oracle, d1, a, sfa, b, sfb, alpha, M, N, K) <= TOL
    assert rel_err(oracle, d2, a, sfa, b, sfb, alpha, M, N, K) <= TOL


def test_workspace_reused_across_shapes(nv, oracle, cuda_dev):
    """One workspace serves calls of any shape: a call with few weight tiles (whose
    fp32 partials fill the workspace) followed by one with more tiles than CTAs, whose
    cut tiles' arrival counters must still read zero — through nvfp4_gemm's own
    per-stream workspace and through one caller buffer passed to nvfp4_gemm_decode."""
    shapes = [(16, 1024, 4096, 41), (1, 28672, 1024, 42), (64, 2048, 2048, 43), (3, 20480, 512, 44)]
    ops = [operands(oracle, M, N, K, seed) for M, N, K, seed in shapes]
    s = torch.cuda.Stream(cuda_dev)
    with torch.cuda.stream(s):  # a fresh stream: its library workspace starts here
        for (M, N, K, _), (a, sfa, b, sfb, alpha) in zip(shapes, ops):
            d = nv.gemm(*(dev_t(t, cuda_dev) for t in (a, sfa, b, sfb)), alpha)
            s.synchronize()
            nv.device_status()
            assert rel_err(oracle, d, a, sfa, b, sfb, alpha, M, N, K) <= TOL, (M, N, K)
    L = nv.lib()
    ws = torch.zeros(max(L.nvfp4_gemm_decode_workspace_size(M, N) for M, N, _, _ in shapes), dtype=torch.uint8,
                     device=cuda_dev)
    for (M, N, K, _), (a, sfa, b, sfb, alpha) in zip(shapes, ops):
        out, _ = decode_call(nv, cuda_dev, a, sfa, b, sfb, alpha, M, N, K, ws=ws)
        assert rel_err(oracle, out, a, sfa, b, sfb, alpha, M, N, K) <= TOL, (M, N, K)
