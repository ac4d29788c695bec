"""Fused GEMM epilogue (nvfp4_gemm_epilogue): bias, activation, NVFP4 output.

CPU: the oracle's epilogue against float64 formulas, and the C ABI's host-side
argument checks (they return before any device call).
GPU: the fused kernels against the unfused path and the oracle —
  * no bias / no activation: bit-identical to nvfp4_gemm;
  * relu: bit-identical to relu of nvfp4_gemm (rounding commutes with max(., 0));
  * bias + relu / silu / gelu_tanh: max|D - D_ref| / max|D_ref| <= 1e-2 against the
    oracle (GEMM accumulation order differs; exp/tanh differ by a few fp32 ulp);
  * NVFP4 output: codes and scales byte-identical to nvfp4_quantize of the fused
    bf16 output with the same global scale, padding scale rows zero.
Shapes cover the split-K decode kernel (M <= 128) and the CTA-pair kernel.
"""
import ctypes as C

import numpy as np
import pytest
import torch

ACTS = ["none", "relu", "silu", "gelu_tanh"]


def _ref_act(y, act):
    y = y.astype(np.float64)
    if act == "relu":
        return np.maximum(y, 0)
    if act == "silu":
        return y / (1 + np.exp(-y))
    if act == "gelu_tanh":
        return 0.5 * y * (1 + np.tanh(np.sqrt(2 / np.pi) * (y + 0.044715 * y ** 3)))
    return y


def test_oracle_swiglu_matches_formula(oracle):
    rng = np.random.default_rng(4)
    acc = (rng.standard_normal((6, 96)) * 3).astype(np.float32)
    bias = oracle.f32_to_bf16_bits(rng.standard_normal(96).astype(np.float32))
    y32, y16 = oracle.epilogue(acc, 0.5, bias, "swiglu")
    y = acc.astype(np.float64) * 0.5 + oracle.bf16_bits_to_f32(bias).astype(np.float64)
    g = np.concatenate([y[:, 32 * j:32 * j + 16] for j in range(3)], axis=1)
    u = np.concatenate([y[:, 32 * j + 16:32 * j + 32] for j in range(3)], axis=1)
    assert y32.shape == (6, 48)
    assert np.allclose(y32, g / (1 + np.exp(-g)) * u, rtol=1e-5, atol=1e-6)
    assert np.array_equal(y16, oracle.f32_to_bf16_bits(y32))


def test_swiglu_interleave_layout(nv):
    gate = torch.arange(64 * 3).reshape(64, 3)
    up = -gate
    w = nv.swiglu_interleave(gate, up)
    assert w.shape == (128, 3)
    assert torch.equal(w[0:16], gate[0:16]) and torch.equal(w[16:32], up[0:16])
    assert torch.equal(w[96:112], gate[48:64]) and torch.equal(w[112:128], up[48:64])
    b = nv.swiglu_interleave(np.arange(32), np.arange(32) + 100)
    assert list(b[14:18]) == [14, 15, 100, 101]
    with pytest.raises(ValueError):
        nv.swiglu_interleave(gate[:10], up[:10])


@pytest.mark.parametrize("act", ACTS)
def test_oracle_epilogue_matches_formula(oracle, act):
    rng = np.random.default_rng(3)
    acc = (rng.standard_normal((7, 64)) * 4).astype(np.float32)
    bias = oracle.f32_to_bf16_bits(rng.standard_normal(64).astype(np.float32))
    y32, y16 = oracle.epilogue(acc, 0.75, bias, act)
    want = _ref_act(acc.astype(np.float64) * 0.75 + oracle.bf16_bits_to_f32(bias).astype(np.float64), act)
    assert np.allclose(y32, want, rtol=1e-5, atol=1e-6)
    assert np.array_equal(y16, oracle.f32_to_bf16_bits(y32))


def test_epilogue_host_checks(nv):
    L = nv.lib()
    fake = 0x10000  # never dereferenced: every case fails its host-side check first
    E = nv._lib.Epilogue

    def call(M, N, K, e, d=fake):
        return L.nvfp4_gemm_epilogue(fake, fake, fake, fake, 1.0, d, M, N, K, C.byref(e), None)

    assert call(256, 256, 256, E(activation=7)) == -1                                   # INVALID
    assert call(256, 256, 256, E(bias=fake + 8)) == -3                                  # ALIGN: bias 16 B
    assert call(256, 200, 256, E(q_out=fake, sf_out=fake, out_global_scale=fake)) == -2  # SHAPE: N % 64
    assert call(256, 256, 256, E(q_out=fake, sf_out=None, out_global_scale=fake)) == -1  # INVALID
    assert call(256, 256, 256, E(q_out=fake, sf_out=fake + 2, out_global_scale=fake)) == -3
    assert call(256, 256, 256, E(q_out=fake + 16, sf_out=fake, out_global_scale=fake)) == -3  # q 32 B
    assert call(256, 256, 100, E()) == -2                                               # K % 64
    assert call(256, 192, 256, E(activation=4)) == -2                                   # SwiGLU: N % 128
    assert call(256, 256, 256, E(activation=5)) == -1                                   # unknown activation


# (72, 12544, 512): M <= 128 with a wide weight (49 tiles of 256 rows) runs on the
# persistent single-CTA kernel, the other small-M shapes on the split-K decode kernel
SHAPES = [(16, 1024, 512), (77, 512, 1024), (300, 768, 1024), (520, 1024, 512), (72, 12544, 512)]


def _operands(oracle, M, N, K, seed):
    a, sfa = oracle.random_codes(M, K, seed=seed, sf_lo=0x30, sf_hi=0x40)
    b, sfb = oracle.random_codes(N, K, seed=seed + 1, sf_lo=0x30, sf_hi=0x40)
    return a, sfa, b, sfb


def _dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_plain_and_relu_bit_identical(nv, oracle, cuda_dev, M, N, K):
    a, sfa, b, sfb = (_dev(x, cuda_dev) for x in _operands(oracle, M, N, K, 11))
    d = nv.gemm(a, sfa, b, sfb, 0.5)
    d0 = nv.gemm_epilogue(a, sfa, b, sfb, 0.5)
    dr = nv.gemm_epilogue(a, sfa, b, sfb, 0.5, activation="relu")
    torch.cuda.synchronize()
    nv.device_status()
    assert torch.equal(d0.view(torch.int16), d.view(torch.int16))
    assert torch.equal(dr.float(), d.float().clamp_min(0))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("act", ["relu", "silu", "gelu_tanh"])
def test_bias_activation_vs_oracle(nv, oracle, cuda_dev, M, N, K, act):
    a, sfa, b, sfb = _operands(oracle, M, N, K, 21)
    bias = oracle.f32_to_bf16_bits(np.random.default_rng(5).standard_normal(N).astype(np.float32))
    alpha = 0.25
    d = nv.gemm_epilogue(_dev(a, cuda_dev), _dev(sfa, cuda_dev), _dev(b, cuda_dev), _dev(sfb, cuda_dev), alpha,
                         bias=_dev(bias, cuda_dev).view(torch.bfloat16), activation=act)
    torch.cuda.synchronize()
    nv.device_status()
    acc, _ = oracle.gemm(a, sfa, b, sfb, 1.0, M, N, K)
    _, ref16 = oracle.epilogue(acc, alpha, bias, act)
    ref = oracle.bf16_bits_to_f32(ref16).reshape(M, N)
    got = d.float().cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 1e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("act,with_bias", [("none", False), ("silu", True), ("gelu_tanh", True)])
def test_nvfp4_output_equals_quantized_bf16(nv, oracle, cuda_dev, M, N, K, act, with_bias):
    a, sfa, b, sfb = (_dev(x, cuda_dev) for x in _operands(oracle, M, N, K, 31))
    bias = None
    if with_bias:
        bias = torch.randn(N, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(cuda_dev)
    d = nv.gemm_epilogue(a, sfa, b, sfb, 0.5, bias=bias, activation=act)
    _, gs = nv.global_scale(d)
    sf_poison = torch.full((nv.sf_bytes(M, N),), 0x7E, dtype=torch.uint8, device=cuda_dev)
    q, sf = nv.gemm_epilogue(a, sfa, b, sfb, 0.5, bias=bias, activation=act, out_global_scale=gs,
                             sf_out=sf_poison)
    q_ref, sf_ref = nv.quantize(d, gs)
    torch.cuda.synchronize()
    nv.device_status()
    assert torch.equal(q, q_ref)
    assert torch.equal(sf, sf_ref)  # padding rows included (nvfp4_quantize zeroes them too)


@pytest.mark.gpu
def test_torch_ops_epilogue(nv, oracle, cuda_dev):
    import nvfp4_b200.torch_ops  # noqa: F401
    M, N, K = 300, 512, 512
    a, sfa, b, sfb = (_dev(x, cuda_dev) for x in _operands(oracle, M, N, K, 41))
    bias = torch.zeros(N, dtype=torch.bfloat16, device=cuda_dev)
    d1 = torch.ops.nvfp4_b200.gemm_epilogue(a, sfa, b, sfb, 1.0, bias, "relu")
    d2 = nv.gemm_epilogue(a, sfa, b, sfb, 1.0, bias=bias, activation="relu")
    _, gs = nv.global_scale(d1)
    q1, s1 = torch.ops.nvfp4_b200.gemm_nvfp4_out(a, sfa, b, sfb, 1.0, gs, bias, "relu")
    q2, s2 = nv.quantize(d1, gs)
    torch.cuda.synchronize()
    assert torch.equal(d1, d2) and torch.equal(q1, q2) and torch.equal(s1, s2)


SWIGLU_SHAPES = [(16, 1024, 512), (77, 512, 1024), (300, 768, 1024), (520, 1024, 512), (72, 12544, 512)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", SWIGLU_SHAPES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_swiglu_vs_oracle(nv, oracle, cuda_dev, M, N, K, with_bias):
    """SwiGLU over gate / up columns interleaved in blocks of 16: [M, N/2] output
    against the oracle (max relative error 1e-2), decode and CTA-pair kernels."""
    a, sfa, b, sfb = _operands(oracle, M, N, K, 51)
    bias = oracle.f32_to_bf16_bits(np.random.default_rng(6).standard_normal(N).astype(np.float32))
    alpha = 0.25
    d = nv.gemm_epilogue(_dev(a, cuda_dev), _dev(sfa, cuda_dev), _dev(b, cuda_dev), _dev(sfb, cuda_dev), alpha,
                         bias=_dev(bias, cuda_dev).view(torch.bfloat16) if with_bias else None, activation="swiglu")
    torch.cuda.synchronize()
    nv.device_status()
    assert d.shape == (M, N // 2)
    acc, _ = oracle.gemm(a, sfa, b, sfb, 1.0, M, N, K)
    _, ref16 = oracle.epilogue(acc.reshape(M, N), alpha, bias if with_bias else None, "swiglu")
    ref = oracle.bf16_bits_to_f32(ref16).reshape(M, N // 2)
    got = d.float().cpu().numpy()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 1e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", SWIGLU_SHAPES)
def test_swiglu_nvfp4_output_equals_quantized_bf16(nv, oracle, cuda_dev, M, N, K):
    a, sfa, b, sfb = (_dev(x, cuda_dev) for x in _operands(oracle, M, N, K, 61))
    bias = torch.randn(N, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).to(cuda_dev)
    d = nv.gemm_epilogue(a, sfa, b, sfb, 0.5, bias=bias, activation="swiglu")
    _, gs = nv.global_scale(d)
    q, sf = nv.gemm_epilogue(a, sfa, b, sfb, 0.5, bias=bias, activation="swiglu", out_global_scale=gs,
                             sf_out=torch.full((nv.sf_bytes(M, N // 2),), 0x7E, dtype=torch.uint8, device=cuda_dev))
    q_ref, sf_ref = nv.quantize(d, gs)
    torch.cuda.synchronize()
    nv.device_status()
    assert q.shape == (M, N // 4)
    assert torch.equal(q, q_ref)
    assert torch.equal(sf, sf_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [16, 300])
def test_swiglu_equals_two_gemms(nv, cuda_dev, M):
    """silu(x Wg^T) * (x Wu^T) from one GEMM over swiglu_interleave(Wg, Wu) equals the
    same from two GEMMs: row-wise block scales make quantizing the interleaved weight
    the same as interleaving the quantized weights."""
    F, K = 512, 1024
    g = torch.Generator(device=cuda_dev).manual_seed(12)
    x = torch.randn(M, K, device=cuda_dev, generator=g).to(torch.bfloat16)
    wg = (torch.randn(F, K, device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
    wu = (torch.randn(F, K, device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
    _, gx = nv.global_scale(x)
    _, gw = nv.global_scale(torch.cat((wg, wu)))
    xq, xsf = nv.quantize(x, gx)
    wq, wsf = nv.quantize(nv.swiglu_interleave(wg, wu).contiguous(), gw)
    gq, gsf = nv.quantize(wg, gw)
    uq, usf = nv.quantize(wu, gw)
    alpha = float(gx.item() * gw.item())
    h = nv.gemm_epilogue(xq, xsf, wq, wsf, alpha, activation="swiglu")
    dg = nv.gemm(xq, xsf, gq, gsf, alpha).float()
    du = nv.gemm(xq, xsf, uq, usf, alpha).float()
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(dg) * du
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err <= 2e-2, err
