"""GPU: the allocation-free decode GEMM, nvfp4_gemm_decode_noalloc.

It is for callers that cannot let this library allocate device memory (hosts that
own all device memory, such as memory-budgeted servers or plugin interfaces that
hand a library only its inputs and outputs, and latency-critical loops where a
cudaMalloc's possible device-wide synchronisation is not acceptable).  Its split-K
scratch is a fixed 4 MiB device array inside the library, shared by every call.

Checked here through the C ABI: two calls in a row, each against the existing
entry point nvfp4_gemm_decode with a caller-provided workspace and against the CPU
oracle's dequantise-then-fp32 GEMM, within the GEMM tolerance the other tests use
(max |D - D_ref| / max |D_ref| <= 1e-2); and shapes whose scratch need exceeds the
fixed array are refused.  This file is collected
last so that a run stopping at the first failure has already run every other
test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2
SCRATCH_LIMIT = 4 << 20


def _operands(M, N, K, seed, dev):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    codes_a = torch.randint(0, 256, (M, K // 2), dtype=torch.int32, device=dev, generator=g).to(torch.uint8)
    codes_b = torch.randint(0, 256, (N, K // 2), dtype=torch.int32, device=dev, generator=g).to(torch.uint8)
    pad = lambda r: (r + 127) // 128 * 128  # noqa: E731
    # finite e4m3 scale codes in [0x30, 0x40): 0.5 .. 0.94
    sfa = torch.randint(0x30, 0x40, (pad(M) * K // 16,), dtype=torch.int32, device=dev, generator=g).to(torch.uint8)
    sfb = torch.randint(0x30, 0x40, (pad(N) * K // 16,), dtype=torch.int32, device=dev, generator=g).to(torch.uint8)
    return codes_a, sfa, codes_b, sfb


def _with_workspace(L, ops, alpha, M, N, K, dev):
    a, sfa, b, sfb = ops
    need = L.nvfp4_gemm_decode_workspace_size(M, N)
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    d = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    st = L.nvfp4_gemm_decode(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), alpha, d.data_ptr(), M, N,
                             K, ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    assert st == 0, L.nvfp4_status_string(st)
    return d


def _no_alloc(L, ops, alpha, M, N, K, dev):
    a, sfa, b, sfb = ops
    d = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
    st = L.nvfp4_gemm_decode_noalloc(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), alpha,
                                     d.data_ptr(), M, N, K, torch.cuda.current_stream(dev).cuda_stream)
    assert st == 0, L.nvfp4_status_string(st)
    return d


def _rel_err(d, ref):
    d, ref = d.float(), ref.float()
    assert torch.isfinite(d).all()
    return float((d - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("M,N,K", [(1, 28672, 8192), (16, 8192, 28672), (9, 1000, 320)])
def test_no_alloc_matches_workspace_entry_point_twice(nv, oracle, cuda_dev, M, N, K):
    L = nv.lib()
    assert L.nvfp4_gemm_decode_workspace_size(M, N) <= SCRATCH_LIMIT
    for call, (seed, alpha) in enumerate([(11, 1.0), (12, 0.25)]):  # two calls in a row, different data
        ops = _operands(M, N, K, seed + M, cuda_dev)
        d = _no_alloc(L, ops, alpha, M, N, K, cuda_dev)
        ref = _with_workspace(L, ops, alpha, M, N, K, cuda_dev)
        torch.cuda.synchronize()
        nv.device_status()
        err = _rel_err(d, ref)
        assert err <= TOL, f"call {call}: rel err {err:.3e}"
        a, sfa, b, sfb = (t.cpu().numpy() for t in ops)
        _, d16 = oracle.gemm(a, sfa, b, sfb, alpha, M, N, K)
        ref_o = torch.from_numpy(oracle.bf16_bits_to_f32(d16).reshape(M, N))
        err_o = _rel_err(d.cpu(), ref_o)
        assert err_o <= TOL, f"call {call}: rel err against the oracle {err_o:.3e}"


def test_no_alloc_refuses_shapes_beyond_its_scratch(nv, cuda_dev):
    L = nv.lib()
    M, N, K = 64, 8192, 1024
    assert L.nvfp4_gemm_decode_workspace_size(M, N) > SCRATCH_LIMIT
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda_dev)
    p = buf.data_ptr()
    st = L.nvfp4_gemm_decode_noalloc(p, p, p, p, 1.0, p, M, N, K, None)
    assert st == -7  # NVFP4_ERR_WORKSPACE
    assert b"workspace" in L.nvfp4_status_string(st)
