"""The reference's .bin interchange and runner CLI (matmul/sm100_nvfp4/main.py:36-44,
runner.cu:36-104): byte formats on the CPU; on a GPU, main.py's verify flow — inputs
from create_tensors, `nvfp4_runner M N K verify`, output checked the way
verify_output does (allclose(atol=rtol=1e-3) against the fp16 reference)."""
import subprocess

import numpy as np
import pytest
import torch


def test_bin_round_trip(nv, tmp_path):
    from nvfp4_b200 import runner_io
    rng = np.random.default_rng(0)
    M, N, K = 256, 128, 512
    a = torch.from_numpy(rng.integers(0, 256, (M, K // 2), dtype=np.uint8))
    b = torch.from_numpy(rng.integers(0, 256, (N, K // 2), dtype=np.uint8))
    sfa = torch.from_numpy(rng.integers(0, 256, M * K // 16, dtype=np.uint8))
    sfb = torch.from_numpy(rng.integers(0, 256, N * K // 16, dtype=np.uint8))
    runner_io.save_tensors(str(tmp_path), a, b, sfa, sfb)
    # main.py writes int8 views: identical bytes
    assert (tmp_path / "a_mat.bin").read_bytes() == a.view(torch.int8).numpy().tobytes()
    la, lb, lsa, lsb = runner_io.load_tensors(str(tmp_path), M, N, K)
    assert np.array_equal(la, a.numpy()) and np.array_equal(lsb, sfb.numpy())


def test_runner_cli_usage_without_gpu(nv):
    from nvfp4_b200 import runner_io
    r = subprocess.run([runner_io.RUNNER], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "Usage" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(512, 1024, 1024), (300, 264, 576)])
def test_runner_verify_like_main_py(nv, oracle, cuda_dev, tmp_path, M, N, K):
    from nvfp4_b200 import runner_io
    a, b, sfa, sfb = nv.create_tensors(M, N, K, seed=42)  # main.py's distribution and layout
    runner_io.save_tensors(str(tmp_path), a, b, sfa, sfb)
    r = runner_io.run(M, N, K, "verify", str(tmp_path))
    assert r.returncode == 0, r.stderr
    c = runner_io.load_output(str(tmp_path), M, N).astype(np.float32)
    d32, _ = oracle.gemm(a.cpu().numpy(), sfa.cpu().numpy(), b.cpu().numpy(), sfb.cpu().numpy(), 1.0, M, N, K)
    ref16 = d32.astype(np.float16).astype(np.float32)
    assert np.allclose(c, ref16, atol=1e-3, rtol=1e-3)  # main.py:61-66
    r = runner_io.run(M, N, K, "benchmark", str(tmp_path))
    assert r.returncode == 0, r.stderr
    assert float(r.stdout.split()[0]) > 0
