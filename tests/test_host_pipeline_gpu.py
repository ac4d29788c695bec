"""GPU: nvfp4_gemm_host (host buffers in and out, copies pipelined with the GEMM).

D is cut into blocks of up to 1024 x 1024 (multiples of the 256 x 256 tile), each
computed by its own GEMM over the full K in the same order as the whole-matrix GEMM,
so the result equals the device GEMM bit for bit — also for ragged shapes whose
edge blocks are partial, for grids that are not square (the growing-square order
then finishes the longer side alone), and on repeated calls that reuse the
pipeline's device buffers.  Rows of each result are also checked against the oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SPEC_TOL = 1e-2


@pytest.mark.parametrize("M,N,K", [
    (2048, 3072, 1024),   # 2 x 3 blocks
    (300, 520, 320),      # one partial block
    (1200, 4104, 2048),   # 2 x 5, ragged on both sides
    (3100, 712, 512),     # 4 x 1: the square stops growing along N
    (256, 5000, 256),     # 1 x 5
])
def test_host_pipeline_matches_device_gemm(nv, oracle, cuda_dev, M, N, K):
    a, sfa = oracle.random_codes(M, K, seed=M, sf_lo=0x30, sf_hi=0x40)
    b, sfb = oracle.random_codes(N, K, seed=N, sf_lo=0x30, sf_hi=0x40)
    host = [torch.from_numpy(t).pin_memory() for t in (a, sfa, b, sfb)]
    dev = [t.to(cuda_dev) for t in host]
    ref = nv.gemm(*dev, 0.75).cpu()
    for _ in range(2):  # the second call reuses the pipeline's device buffers
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
        nv.gemm_host(*host, 0.75, out)
        torch.cuda.synchronize()
        nv.device_status()
        assert torch.isfinite(out.float()).all(), "unwritten block"
        assert torch.equal(out, ref), "differs from the device GEMM"
    got = out.float().numpy()
    for m0 in sorted({0, M // 2, M - 8}):
        d32, d16 = oracle.gemm(a, sfa, b, sfb, 0.75, M, N, K, m0=m0, mrows=8)
        want = oracle.bf16_bits_to_f32(d16).reshape(8, N)
        err = np.abs(got[m0:m0 + 8] - want).max() / max(np.abs(want).max(), 1e-30)
        assert err <= SPEC_TOL, f"rows {m0}..{m0 + 8}: {err:.3e}"


def test_back_to_back_calls_overlap_correctly(nv, oracle, cuda_dev):
    """Calls issued without waiting, in turn on two caller streams (so one call's
    uploads and GEMMs overlap the previous call's download), with shapes that change
    the device buffers' layout between calls: every result equals its device GEMM."""
    shapes = [(2048, 3072, 1024), (2048, 3072, 1024), (1200, 4104, 2048), (2048, 3072, 1024), (3100, 712, 512),
              (3100, 712, 512)]
    cases = []
    for n, (M, N, K) in enumerate(shapes):
        a, sfa = oracle.random_codes(M, K, seed=100 + n, sf_lo=0x30, sf_hi=0x40)
        b, sfb = oracle.random_codes(N, K, seed=200 + n, sf_lo=0x30, sf_hi=0x40)
        host = [torch.from_numpy(t).pin_memory() for t in (a, sfa, b, sfb)]
        ref = nv.gemm(*[t.to(cuda_dev) for t in host], 0.5).cpu()
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
        cases.append((host, ref, out))
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(cuda_dev), torch.cuda.Stream(cuda_dev)]
    for n, (host, _, out) in enumerate(cases):
        with torch.cuda.stream(streams[n % 2]):
            nv.gemm_host(*host, 0.5, out)
    torch.cuda.synchronize()
    nv.device_status()
    for n, (_, ref, out) in enumerate(cases):
        assert torch.equal(out, ref), f"call {n} {shapes[n]}"


def test_grown_operands_wait_for_earlier_downloads(nv, oracle, cuda_dev):
    """A call whose operands take more room than the previous call's moves the D
    buffers: its uploads must not land on memory an earlier call's D is still being
    downloaded from.  A wide D with small operands (a long download), then a square
    problem with large operands, issued without waiting on two streams."""
    shapes = [(4096, 8192, 512), (2048, 2048, 8192), (4096, 8192, 512)]
    cases = []
    for n, (M, N, K) in enumerate(shapes):
        a, sfa = oracle.random_codes(M, K, seed=300 + n, sf_lo=0x30, sf_hi=0x40)
        b, sfb = oracle.random_codes(N, K, seed=400 + n, sf_lo=0x30, sf_hi=0x40)
        host = [torch.from_numpy(t).pin_memory() for t in (a, sfa, b, sfb)]
        ref = nv.gemm(*[t.to(cuda_dev) for t in host], 0.25).cpu()
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
        cases.append((host, ref, out))
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(cuda_dev), torch.cuda.Stream(cuda_dev)]
    for n, (host, _, out) in enumerate(cases):
        with torch.cuda.stream(streams[n % 2]):
            nv.gemm_host(*host, 0.25, out)
    torch.cuda.synchronize()
    nv.device_status()
    for n, (_, ref, out) in enumerate(cases):
        assert torch.equal(out, ref), f"call {n} {shapes[n]}"
