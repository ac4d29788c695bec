"""GPU parity: the quantizer kernel must be bit-exact with the CPU specification
(codes, scales and scale padding), and the amax / global-scale kernel exact."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def quantize_both(nv, oracle, x_bits, gs, dev):
    M, K = x_bits.shape
    xt = torch.from_numpy(x_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    q_ref, sf_ref = oracle.quantize(x_bits, gs)
    sf_out = torch.full((sf_ref.size,), 0xAB, dtype=torch.uint8, device=dev)  # poison padding
    q, sf = nv.quantize(xt, torch.tensor([gs], dtype=torch.float32, device=dev), sf_out=sf_out)
    torch.cuda.synchronize()
    return q.cpu().numpy(), sf.cpu().numpy(), q_ref, sf_ref


@pytest.mark.parametrize("M,K", [(1, 64), (128, 256), (200, 320), (513, 1024), (4096, 4096)])
def test_normal_bit_exact(nv, oracle, cuda_dev, M, K):
    x = oracle.normal_bf16((M, K), seed=M + K)
    gs = oracle.global_scale_for(oracle.amax_bf16(x))
    q, sf, q_ref, sf_ref = quantize_both(nv, oracle, x, gs, cuda_dev)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(sf, sf_ref)


def test_c5_student_t_outliers_bit_exact(nv, oracle, cuda_dev):
    """BASELINE config 5 activations: Student-t(3), 4 of 4096 channels x50."""
    x = oracle.student_t3_bf16(4096, 4096, seed=5, n_outlier_cols=4, gain=50.0)
    gs = oracle.global_scale_for(oracle.amax_bf16(x))
    q, sf, q_ref, sf_ref = quantize_both(nv, oracle, x, gs, cuda_dev)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(sf, sf_ref)


def test_ties_and_saturation_bit_exact(nv, oracle, cuda_dev):
    """Blocks whose scaled values sit exactly on e2m1 midpoints (gs = 1, amax = 6 ->
    inv = 1), plus blocks that saturate the scale and blocks of zeros / tiny values."""
    rng = np.random.default_rng(0)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0], np.float32)
    M, K = 256, 256
    x = rng.choice(mids, size=(M, K)) * rng.choice([-1.0, 1.0], size=(M, K))
    x = x.astype(np.float32)
    x[:, ::16] = 6.0  # every block's amax is exactly 6
    x[:8] *= 1e4      # these rows saturate the e4m3 scale
    x[8:16] = 0.0     # all-zero blocks
    x[16:24] *= 1e-6  # subnormal scales
    bits = oracle.f32_to_bf16_bits(x)
    q, sf, q_ref, sf_ref = quantize_both(nv, oracle, bits, 1.0, cuda_dev)
    assert np.array_equal(q, q_ref)
    assert np.array_equal(sf, sf_ref)


@pytest.mark.parametrize("gs", [0.0, float("nan"), -1.0, 2.0 ** -120])
def test_unusable_global_scale(nv, oracle, cuda_dev, gs):
    x = oracle.normal_bf16((128, 128), seed=9)
    q, sf, q_ref, sf_ref = quantize_both(nv, oracle, x, gs, cuda_dev)
    assert np.array_equal(q, q_ref) and np.array_equal(sf, sf_ref)
    assert not sf.any()


def test_global_scale_kernel(nv, oracle, cuda_dev):
    for shape, seed in [((4096, 4096), 1), ((3, 77), 2), ((1, 8), 3)]:
        x = oracle.normal_bf16(shape, seed=seed)
        xt = torch.from_numpy(x.view(np.int16)).to(cuda_dev).view(torch.bfloat16)
        amax, gs = nv.global_scale(xt)
        torch.cuda.synchronize()
        ref = oracle.amax_bf16(x)
        assert amax.item() == ref
        assert gs.item() == oracle.global_scale_for(ref)


def test_quantize_then_gemm_roundtrip(nv, oracle, cuda_dev):
    """C5-style fused flow on the GPU: amax -> gs -> quantize -> GEMM, compared with the
    oracle doing the same steps on the CPU."""
    M, N, K = 512, 1024, 1024
    x = oracle.student_t3_bf16(M, K, seed=31, n_outlier_cols=1, gain=50.0)
    w = oracle.normal_bf16((N, K), seed=32, std=0.02)
    gsw = oracle.global_scale_for(oracle.amax_bf16(w))
    wq, wsf = oracle.quantize(w, gsw)
    xt = torch.from_numpy(x.view(np.int16)).to(cuda_dev).view(torch.bfloat16)
    _, gsx = nv.global_scale(xt)
    xq, xsf = nv.quantize(xt, gsx)
    alpha = float(np.float32(gsx.item()) * np.float32(gsw))
    d = nv.gemm(xq, xsf, torch.from_numpy(wq).to(cuda_dev), torch.from_numpy(wsf).to(cuda_dev), alpha)
    torch.cuda.synchronize()
    gsx_ref = oracle.global_scale_for(oracle.amax_bf16(x))
    xq_ref, xsf_ref = oracle.quantize(x, gsx_ref)
    assert np.array_equal(xq.cpu().numpy(), xq_ref) and np.array_equal(xsf.cpu().numpy(), xsf_ref)
    _, d16 = oracle.gemm(xq_ref, xsf_ref, wq, wsf, alpha, M, N, K)
    ref = oracle.bf16_bits_to_f32(d16).reshape(M, N)
    err = np.abs(d.float().cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err <= 1e-2
