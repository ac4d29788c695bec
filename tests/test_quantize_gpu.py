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


def _every_amax_blocks():
    """One 16-element block per non-negative bf16 value from +0 to +inf (32641 blocks):
    the block holds +v, -v and fifteenths of v, so its amax is exactly v."""
    vals = np.arange(0, 0x7F81, dtype=np.uint32)
    K = 1024
    per_row = K // 16
    rows = (len(vals) + per_row - 1) // per_row
    blocks = np.zeros((rows * per_row, 16), dtype=np.uint16)
    v = vals.astype(np.uint16)
    blocks[: len(vals), 0] = v
    blocks[: len(vals), 1] = v | 0x8000
    f = (vals << 16).view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        small = (f / 15.0).astype(np.float32)
    small_bits = (small.view(np.uint32) >> 16).astype(np.uint16)  # truncation keeps it below v
    blocks[: len(vals), 2:] = small_bits[:, None]
    return blocks.reshape(rows, K)


GS_SWEEP = [1.0, 1.0 / 2688.0, 3.7e-5, 0.123, 1e30, 2.0 ** -100, 3.0e38]


@pytest.mark.parametrize("gs", GS_SWEEP)
def test_scale_code_of_every_bf16_amax(nv, oracle, cuda_dev, gs):
    """Every possible bf16 block amax, +inf included, over global scales from 2^-100
    to 3e38: the quantizer's scale codes (and, for finite blocks, element codes)
    equal the specification's."""
    x = _every_amax_blocks()
    q, sf, q_ref, sf_ref = quantize_both(nv, oracle, x, gs, cuda_dev)
    assert np.array_equal(sf, sf_ref)
    # Codes of the +inf block (block 0x7F80: row 510, bytes 0-7) are outside the
    # specification, which wants finite inputs: at gs = 3e38 its reciprocal underflows
    # to 0 and inf * 0 is NaN.  Every finite block must match.
    finite = np.ones(q.shape, dtype=bool)
    finite[0x7F80 // 64, 0:8] = False
    assert np.array_equal(q[finite], q_ref[finite])


@pytest.mark.parametrize("gs", GS_SWEEP + [0.0, float("nan"), -1.0, 2.0 ** -120])
def test_table_scale_codes_every_bf16_amax(nv, oracle, cuda_dev, gs):
    """The fused GEMM epilogue's division-free scale codes (threshold tables built per
    launch, a first guess corrected by two comparisons; nvfp4_scale_codes of the
    diagnostic library (the same sources, nvfp4_diag) runs that
    arithmetic) against the specification's code for every bf16 amax from +0 to +inf,
    negative zero and negative values (the sign is ignored) included."""
    import nvfp4_diag
    diag = nvfp4_diag.lib()
    x = _every_amax_blocks()
    _, sf_ref = oracle.quantize(x, gs)
    rows, K = x.shape
    ref = oracle.sf_unpack(sf_ref, rows, K).reshape(-1)[: 0x7F81]
    vals = np.arange(0, 0x7F81, dtype=np.uint16)
    for amax in (vals, vals | np.uint16(0x8000)):
        t = torch.from_numpy(amax.view(np.int16)).to(cuda_dev)
        codes = torch.empty(len(vals), dtype=torch.uint8, device=cuda_dev)
        g = torch.tensor([gs], dtype=torch.float32, device=cuda_dev)
        st = diag.nvfp4_scale_codes(t.data_ptr(), len(vals), g.data_ptr(), codes.data_ptr(),
                                        torch.cuda.current_stream(cuda_dev).cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        got = codes.cpu().numpy()
        bad = np.nonzero(got != ref)[0]
        assert bad.size == 0, [(hex(int(amax[i])), int(got[i]), int(ref[i])) for i in bad[:8]]


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


@pytest.mark.parametrize("M,K", [(1, 64), (200, 320), (513, 1024), (4096, 4096)])
def test_quantize_dynamic_equals_global_scale_then_quantize(nv, oracle, cuda_dev, M, K):
    """One cooperative kernel (amax, grid barrier, gs, quantize) against the two calls:
    the same gs and the same bytes, twice in a row (the barrier resets itself)."""
    x = oracle.student_t3_bf16(M, K, seed=M + 3, n_outlier_cols=1, gain=50.0)
    xt = torch.from_numpy(x.view(np.int16)).to(cuda_dev).view(torch.bfloat16)
    _, gs = nv.global_scale(xt)
    q_ref, sf_ref = nv.quantize(xt, gs)
    for _ in range(2):
        q, sf, gs2 = nv.quantize_dynamic(xt)
        torch.cuda.synchronize()
        nv.device_status()
        assert gs2.item() == gs.item()
        assert torch.equal(q, q_ref) and torch.equal(sf, sf_ref)
    q_o, sf_o = oracle.quantize(x, float(gs.item()))
    assert np.array_equal(q.cpu().numpy(), q_o) and np.array_equal(sf.cpu().numpy(), sf_o)


def test_quantize_dynamic_in_cuda_graph(nv, cuda_dev):
    M, K = 1024, 2048
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(cuda_dev)
    q = torch.empty(M, K // 2, dtype=torch.uint8, device=cuda_dev)
    sf = torch.empty(nv.sf_bytes(M, K), dtype=torch.uint8, device=cuda_dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        nv.quantize_dynamic(x, q_out=q, sf_out=sf)  # the stream's workspace is made here
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            nv.quantize_dynamic(x, q_out=q, sf_out=sf)
    x.mul_(3.0)  # new data, new global scale, same buffers
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    nv.device_status()
    del g
    _, gs = nv.global_scale(x)
    q_ref, sf_ref = nv.quantize(x, gs)
    assert torch.equal(q, q_ref) and torch.equal(sf, sf_ref)
