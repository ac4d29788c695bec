"""Grouped (mixture-of-experts) GEMM and quantizer.

Group g = rows [m_offsets[g], m_offsets[g+1]) of the stacked activations, expert
weight g = rows [g*N, (g+1)*N) of B; scales of a grouped operand are each group's
blocked tensor starting on a 128-row block (the layout MoE kernels use for
per-expert scale factors).  The oracle is applied group by group:
  * quantizer: codes and every group's scale blocks byte-identical to the oracle's
    quantizer run on that group alone (padding rows zero);
  * GEMM: each group's D rows against the oracle GEMM of (A_g, B_g, alpha_g) with
    max|D - D_ref| / max|D_ref| <= 1e-2; rows outside every group untouched;
  * device-side routing: one captured CUDA graph replayed after the offsets change
    in place follows the new routing;
  * fused epilogue (nvfp4_gemm_grouped_epilogue): per-expert bias + activation per
    group against the oracle's epilogue; NVFP4 output byte-identical to
    quantize_grouped of the fused bf16 output (the next grouped GEMM's operand).
With at most 128 rows in all (decode) the stream-K kernel runs over the active
experts' weight tiles only; above that the CTA-pair kernel's grouped scheduler.
"""
import ctypes as C

import numpy as np
import pytest
import torch


def test_grouped_layout_rules(nv):
    assert nv.grouped_sf_bytes(1000, 4, 1024) == (8 + 4) * 128 * 64
    assert nv.grouped_sf_block0([0, 100, 100, 357, 900]) == [0, 1, 1, 4, 9]


def test_grouped_host_checks(nv):
    L = nv.lib()
    f = 0x10000
    assert L.nvfp4_gemm_grouped(f, f, f, f, f, f, f, 0, 256, 256, 256, None) == -2     # no groups
    assert L.nvfp4_gemm_grouped(f, f, f, f, f, f, f, 257, 256, 256, 256, None) == -2   # > 256 groups
    assert L.nvfp4_gemm_grouped(f, f, f, f, f, f, f, 4, 256, 200, 256, None) == -2     # N % 128
    assert L.nvfp4_gemm_grouped(f, f, f, f, f, f, None, 4, 256, 256, 256, None) == -1  # no offsets
    assert L.nvfp4_gemm_grouped(f + 8, f, f, f, f, f, f, 4, 256, 256, 256, None) == -3
    assert L.nvfp4_quantize_grouped(f, f, f, f, f, 0, 256, 256, None) == -2
    assert L.nvfp4_quantize_grouped(f + 16, f, f, f, f, 4, 256, 256, None) == -3      # X 32-byte aligned


def _group_rows(offsets, m_total):
    out = []
    for g in range(len(offsets) - 1):
        a = min(max(offsets[g], 0), m_total)
        z = min(max(offsets[g + 1], a), m_total)
        out.append((a, z))
    return out


CASES = [
    # (offsets, m_total, N, K): empty group, groups not 128/256-aligned, rows outside all groups
    ([0, 100, 100, 357, 900], 1000, 512, 1024),
    # N % 256 == 128: the last column tile of an expert reads into the next expert's rows
    ([0, 600, 640, 1500], 1500, 384, 512),
    # eight experts, one of them holding most rows
    ([0, 7, 300, 301, 2400, 2401, 2402, 2600, 3000], 3072, 1024, 2048),
    # decode sizes (m_total <= 128: the stream-K kernel over active experts only):
    # empty experts, a one-row expert, rows outside every group
    ([0, 3, 3, 10, 40], 48, 512, 1024),
    ([0, 0, 9, 9, 9, 30, 31, 31, 64], 64, 1024, 2048),
    ([0, 128], 128, 256, 512),
    # the group limit: 256 experts, 96 routed rows over a few dozen of them
    ([0] + np.cumsum(np.bincount(np.random.default_rng(5).integers(0, 256, 96), minlength=256)).tolist(),
     96, 128, 256),
]


def _make(oracle, nv, dev, offsets, m_total, N, K, seed):
    G = len(offsets) - 1
    x = oracle.normal_bf16((m_total, K), seed=seed)
    gsa = oracle.global_scale_for(oracle.amax_bf16(x))
    xt = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    offs = torch.tensor(offsets, dtype=torch.int32, device=dev)
    q, sf = nv.quantize_grouped(xt, torch.tensor([gsa], dtype=torch.float32, device=dev), offs)
    bq, bsf, alphas = [], [], []
    for g in range(G):
        w = oracle.normal_bf16((N, K), seed=seed + 100 + g, std=0.02)
        gsb = oracle.global_scale_for(oracle.amax_bf16(w))
        qb, sfb = oracle.quantize(w, gsb)
        bq.append(qb)
        bsf.append(sfb)
        alphas.append(np.float32(gsa) * np.float32(gsb))
    return x, gsa, offs, q, sf, np.concatenate(bq), np.concatenate(bsf), np.array(alphas, dtype=np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("offsets,m_total,N,K", CASES)
def test_quantize_grouped_matches_oracle_per_group(nv, oracle, cuda_dev, offsets, m_total, N, K):
    x, gsa, offs, q, sf, *_ = _make(oracle, nv, cuda_dev, offsets, m_total, N, K, seed=5)
    torch.cuda.synchronize()
    q, sf = q.cpu().numpy(), sf.cpu().numpy()
    blk = 128 * K // 16
    block0 = 0
    for a, z in _group_rows(offsets, m_total):
        if z == a:
            continue
        q_ref, sf_ref = oracle.quantize(x[a:z], gsa)
        assert np.array_equal(q[a:z], q_ref)
        nb = (z - a + 127) // 128
        assert np.array_equal(sf[block0 * blk:(block0 + nb) * blk], sf_ref), (a, z)
        block0 += nb
    # rows outside every group still get codes (same per-block arithmetic)
    last = _group_rows(offsets, m_total)[-1][1]
    if last < m_total:
        q_ref, _ = oracle.quantize(x[last:], gsa)
        assert np.array_equal(q[last:], q_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("offsets,m_total,N,K", CASES)
def test_gemm_grouped_matches_oracle_per_group(nv, oracle, cuda_dev, offsets, m_total, N, K):
    x, gsa, offs, q, sf, bq, bsf, alphas = _make(oracle, nv, cuda_dev, offsets, m_total, N, K, seed=7)
    out = torch.full((m_total, N), 7.0, dtype=torch.bfloat16, device=cuda_dev)  # sentinel outside the groups
    d = nv.gemm_grouped(q, sf, torch.from_numpy(bq).to(cuda_dev), torch.from_numpy(bsf).to(cuda_dev),
                        torch.from_numpy(alphas).to(cuda_dev), offs, out=out)
    torch.cuda.synchronize()
    nv.device_status()
    got = d.float().cpu().numpy()
    qh, sfh = q.cpu().numpy(), sf.cpu().numpy()
    blk = 128 * K // 16
    block0 = 0
    covered = np.zeros(m_total, dtype=bool)
    for g, (a, z) in enumerate(_group_rows(offsets, m_total)):
        if z == a:
            continue
        nb = (z - a + 127) // 128
        _, d16 = oracle.gemm(qh[a:z], sfh[block0 * blk:(block0 + nb) * blk], bq[g * N:(g + 1) * N],
                             bsf[g * (N // 128) * blk:(g + 1) * (N // 128) * blk], float(alphas[g]), z - a, N, K)
        ref = oracle.bf16_bits_to_f32(d16).reshape(z - a, N)
        err = np.abs(got[a:z] - ref).max() / np.abs(ref).max()
        assert err <= 1e-2, (g, err)
        covered[a:z] = True
        block0 += nb
    assert (got[~covered] == 7.0).all()


@pytest.mark.gpu
def test_gemm_grouped_graph_follows_device_routing(nv, oracle, cuda_dev):
    offsets, m_total, N, K = [0, 300, 700, 1024], 1024, 256, 512
    x, gsa, offs, q, sf, bq, bsf, alphas = _make(oracle, nv, cuda_dev, offsets, m_total, N, K, seed=9)
    b, sfb, al = (torch.from_numpy(t).to(cuda_dev) for t in (bq, bsf, alphas))
    out = torch.zeros(m_total, N, dtype=torch.bfloat16, device=cuda_dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        nv.gemm_grouped(q, sf, b, sfb, al, offs, out=out)  # warm-up: tensor maps, attributes
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            nv.gemm_grouped(q, sf, b, sfb, al, offs, out=out)
    graph.replay()
    torch.cuda.synchronize()
    first = out.clone()
    # new routing written on the device: every row to expert 2 (the activations are
    # re-quantized into the captured buffers for the new grouping first)
    new = torch.tensor([0, 0, 0, 1024], dtype=torch.int32, device=cuda_dev)
    xt = torch.from_numpy(x.view(np.int16)).to(cuda_dev).view(torch.bfloat16)
    nv.quantize_grouped(xt, torch.tensor([gsa], dtype=torch.float32, device=cuda_dev), new, q_out=q, sf_out=sf)
    offs.copy_(new)
    graph.replay()
    torch.cuda.synchronize()
    del graph
    ref = nv.gemm(q, sf[:nv.sf_bytes(m_total, K)], b[2 * N:], sfb[2 * (N // 128) * 128 * K // 16:], float(alphas[2]))
    torch.cuda.synchronize()
    got, want = out.float(), ref.float()
    assert (got - want).abs().max().item() <= 1e-2 * want.abs().max().item()
    assert not torch.equal(first, out)


@pytest.mark.gpu
def test_gemm_grouped_decode_graph_follows_device_routing(nv, oracle, cuda_dev):
    """The decode-size grouped kernel (m_total <= 128) derives its schedule from the
    device-side offsets, so a captured call follows a routing written after capture:
    three experts, then every row in one expert (a 64-row tile)."""
    offsets, m_total, N, K = [0, 20, 50, 64], 64, 256, 512
    x, gsa, offs, q, sf, bq, bsf, alphas = _make(oracle, nv, cuda_dev, offsets, m_total, N, K, seed=13)
    b, sfb, al = (torch.from_numpy(t).to(cuda_dev) for t in (bq, bsf, alphas))
    out = torch.zeros(m_total, N, dtype=torch.bfloat16, device=cuda_dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        nv.gemm_grouped(q, sf, b, sfb, al, offs, out=out)  # warm-up: tensor maps, this stream's workspace
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            nv.gemm_grouped(q, sf, b, sfb, al, offs, out=out)
    graph.replay()
    torch.cuda.synchronize()
    first = out.clone()
    qh, sfh = q.cpu().numpy(), sf.cpu().numpy()
    blk = 128 * K // 16
    for g, (a, z) in enumerate(_group_rows(offsets, m_total)):
        _, d16 = oracle.gemm(qh[a:z], sfh[g * blk:(g + 1) * blk], bq[g * N:(g + 1) * N],
                             bsf[g * (N // 128) * blk:(g + 1) * (N // 128) * blk], float(alphas[g]), z - a, N, K)
        ref = oracle.bf16_bits_to_f32(d16).reshape(z - a, N)
        assert np.abs(first[a:z].float().cpu().numpy() - ref).max() <= 1e-2 * np.abs(ref).max(), g
    new = torch.tensor([0, 0, 64, 64], dtype=torch.int32, device=cuda_dev)
    xt = torch.from_numpy(x.view(np.int16)).to(cuda_dev).view(torch.bfloat16)
    nv.quantize_grouped(xt, torch.tensor([gsa], dtype=torch.float32, device=cuda_dev), new, q_out=q, sf_out=sf)
    offs.copy_(new)
    graph.replay()
    torch.cuda.synchronize()
    nv.device_status()
    del graph
    _, d16 = oracle.gemm(q.cpu().numpy(), sf.cpu().numpy()[:blk], bq[N:2 * N], bsf[(N // 128) * blk:2 * (N // 128) * blk],
                         float(alphas[1]), m_total, N, K)
    ref = oracle.bf16_bits_to_f32(d16).reshape(m_total, N)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 1e-2 * np.abs(ref).max()
    assert not torch.equal(first, out)


def test_grouped_epilogue_host_checks(nv):
    L = nv.lib()
    f = 0x10000
    E = nv._lib.Epilogue
    call = lambda e, N=256: L.nvfp4_gemm_grouped_epilogue(f, f, f, f, f, f, f, 4, 256, N, 256,  # noqa: E731
                                                          C.byref(e), None)
    assert call(E(activation=9)) == -1                                                   # unknown activation
    assert call(E(bias=f + 8)) == -3                                                     # bias 16-byte aligned
    assert call(E(q_out=f, sf_out=None, out_global_scale=f)) == -1                       # scales missing
    assert call(E(q_out=f + 16, sf_out=f, out_global_scale=f)) == -3                     # codes 32-byte aligned


EPI_CASES = [CASES[0], CASES[2], CASES[3], CASES[4]]


@pytest.mark.gpu
@pytest.mark.parametrize("offsets,m_total,N,K", EPI_CASES)
@pytest.mark.parametrize("act", ["relu", "silu", "gelu_tanh", "swiglu"])
def test_gemm_grouped_epilogue_vs_oracle(nv, oracle, cuda_dev, offsets, m_total, N, K, act):
    """Per-expert bias + activation fused into the grouped GEMM, each group against the
    oracle's GEMM and epilogue (max relative error 1e-2)."""
    x, gsa, offs, q, sf, bq, bsf, alphas = _make(oracle, nv, cuda_dev, offsets, m_total, N, K, seed=11)
    G = len(offsets) - 1
    bias = oracle.f32_to_bf16_bits(np.random.default_rng(3).standard_normal((G, N)).astype(np.float32))
    No = N // 2 if act == "swiglu" else N
    out = torch.full((m_total, No), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    d = nv.gemm_grouped_epilogue(q, sf, torch.from_numpy(bq).to(cuda_dev), torch.from_numpy(bsf).to(cuda_dev),
                                 torch.from_numpy(alphas).to(cuda_dev), offs,
                                 bias=torch.from_numpy(bias.view(np.int16)).to(cuda_dev).view(torch.bfloat16),
                                 activation=act, out=out)
    torch.cuda.synchronize()
    nv.device_status()
    got = d.float().cpu().numpy()
    qh, sfh = q.cpu().numpy(), sf.cpu().numpy()
    blk = 128 * K // 16
    block0 = 0
    covered = np.zeros(m_total, dtype=bool)
    for g, (a, z) in enumerate(_group_rows(offsets, m_total)):
        if z == a:
            continue
        nb = (z - a + 127) // 128
        acc, _ = oracle.gemm(qh[a:z], sfh[block0 * blk:(block0 + nb) * blk], bq[g * N:(g + 1) * N],
                             bsf[g * (N // 128) * blk:(g + 1) * (N // 128) * blk], 1.0, z - a, N, K)
        _, ref16 = oracle.epilogue(acc.reshape(z - a, N), float(alphas[g]), bias[g], act)
        ref = oracle.bf16_bits_to_f32(ref16).reshape(z - a, No)
        err = np.abs(got[a:z] - ref).max() / np.abs(ref).max()
        assert err <= 1e-2, (g, err)
        covered[a:z] = True
        block0 += nb
    assert (got[~covered] == 7.0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("offsets,m_total,N,K", CASES)
@pytest.mark.parametrize("act", ["silu", "swiglu"])
def test_gemm_grouped_nvfp4_out_equals_quantize_grouped(nv, oracle, cuda_dev, offsets, m_total, N, K, act):
    """NVFP4 output of the grouped GEMM (silu or swiglu, per-expert bias): codes and
    grouped scales byte-identical to quantize_grouped of the fused bf16 output, so it
    can be the A operand of the next grouped GEMM as it stands."""
    if act == "swiglu" and N % 128:
        pytest.skip("SwiGLU needs N % 128 == 0")
    x, gsa, offs, q, sf, bq, bsf, alphas = _make(oracle, nv, cuda_dev, offsets, m_total, N, K, seed=13)
    G = len(offsets) - 1
    No = N // 2 if act == "swiglu" else N
    b, sfb, al = (torch.from_numpy(t).to(cuda_dev) for t in (bq, bsf, alphas))
    bias = torch.randn(G, N, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(cuda_dev)
    d = nv.gemm_grouped_epilogue(q, sf, b, sfb, al, offs, bias=bias, activation=act)
    _, gs = nv.global_scale(d)
    q2, sf2 = nv.gemm_grouped_epilogue(q, sf, b, sfb, al, offs, bias=bias, activation=act, out_global_scale=gs)
    q_ref, sf_ref = nv.quantize_grouped(d, gs, offs)
    torch.cuda.synchronize()
    nv.device_status()
    used = nv.grouped_sf_block0([min(max(o, 0), m_total) for o in offsets])[-1] * 128 * No // 16
    rows = np.zeros(m_total, dtype=bool)
    for a, z in _group_rows(offsets, m_total):
        rows[a:z] = True
    rows_t = torch.from_numpy(rows).to(cuda_dev)
    assert torch.equal(q2[rows_t], q_ref[rows_t])
    assert torch.equal(sf2[:used], sf_ref[:used])
