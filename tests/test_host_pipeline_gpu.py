"""GPU: nvfp4_gemm_host (host buffers in and out, copies pipelined with the GEMM)
gives the same D as the device GEMM on the same operands, also for ragged shapes
whose D blocks are partial, and on repeated calls reusing its device buffers."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(2048, 3072, 1024), (300, 520, 320), (1200, 4104, 2048)])
def test_host_pipeline_matches_device_gemm(nv, oracle, cuda_dev, M, N, K):
    a, sfa = oracle.random_codes(M, K, seed=M, sf_lo=0x30, sf_hi=0x40)
    b, sfb = oracle.random_codes(N, K, seed=N, sf_lo=0x30, sf_hi=0x40)
    host = [torch.from_numpy(t).pin_memory() for t in (a, sfa, b, sfb)]
    dev = [t.to(cuda_dev) for t in host]
    ref = nv.gemm(*dev, 0.75)
    for _ in range(2):  # the second call reuses the pipeline's device buffers
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
        nv.gemm_host(*host, 0.75, out)
        torch.cuda.synchronize()
        nv.device_status()
        got, want = out.float(), ref.float().cpu()
        assert torch.isfinite(got).all()
        err = float((got - want).abs().max() / want.abs().max())
        assert err <= 1e-2, err
