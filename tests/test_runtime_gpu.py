"""GPU: error handling of the C ABI — bounded waits report a timeout instead of
hanging, bad arguments are refused on the host, and the context stays usable."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_timeout_selftest_reports_and_recovers(nv, oracle, cuda_dev):
    # a barrier that nothing arrives on, 1 ms limit: the kernel must give up
    assert nv.selftest_wait_timeout(1_000_000) == -5
    # the status word was read and cleared; the context still runs real work
    a, sfa = oracle.random_codes(128, 256, seed=1, sf_lo=0x30, sf_hi=0x38)
    b, sfb = oracle.random_codes(256, 256, seed=2, sf_lo=0x30, sf_hi=0x38)
    dev = lambda t: torch.from_numpy(t).to(cuda_dev)  # noqa: E731
    d = nv.gemm(dev(a), dev(sfa), dev(b), dev(sfb), 1.0)
    nv.device_status()
    ref32, _ = oracle.gemm(a, sfa, b, sfb, 1.0, 128, 256, 256)
    assert np.abs(d.float().cpu().numpy() - ref32).max() <= 1e-2 * np.abs(ref32).max()


def test_bad_arguments_raise(nv, cuda_dev):
    a = torch.zeros(128, 128, dtype=torch.uint8, device=cuda_dev)
    sfa = torch.zeros(128 * 16, dtype=torch.uint8, device=cuda_dev)
    b = torch.zeros(12, 128, dtype=torch.uint8, device=cuda_dev)  # N = 12: not a multiple of 8
    sfb = torch.zeros(128 * 16, dtype=torch.uint8, device=cuda_dev)
    with pytest.raises(nv.NVFP4Error) as e:
        nv.gemm(a, sfa, b, sfb)
    assert e.value.status == -2
    x = torch.zeros(64, 96, dtype=torch.bfloat16, device=cuda_dev)  # K = 96
    with pytest.raises(nv.NVFP4Error):
        nv.quantize(x, 1.0)
    base = torch.zeros(4096, dtype=torch.uint8, device=cuda_dev)
    st = nv.lib().nvfp4_gemm(base.data_ptr() + 8, base.data_ptr(), base.data_ptr(), base.data_ptr(), 1.0,
                             base.data_ptr(), 8, 8, 64, None)
    assert st == -3
    nv.device_status()


def test_launch_counter_counts_our_kernels(nv, cuda_dev):
    x = torch.randn(128, 256, device=cuda_dev).to(torch.bfloat16)
    n0 = nv.launch_count()
    q, sf = nv.quantize(x, 0.001)
    torch.cuda.synchronize()
    assert nv.launch_count() == n0 + 1


def test_workspaces_cleared_again_after_a_reported_timeout(nv, oracle, cuda_dev):
    """A kernel that gave up a wait may leave split-K arrival counters set, so once
    nvfp4_device_status has reported a timeout, the library-owned decode workspace of
    a stream and the allocation-free scratch are cleared again before their next use:
    decode GEMMs before and after a reported timeout give the same, correct result."""
    M, N, K = 16, 2048, 4096  # 16 weight tiles over 148 CTAs: every tile cut (counters in use)
    a, sfa = oracle.random_codes(M, K, seed=21, sf_lo=0x30, sf_hi=0x38)
    b, sfb = oracle.random_codes(N, K, seed=22, sf_lo=0x30, sf_hi=0x38)
    ta, tsa, tb, tsb = (torch.from_numpy(t).to(cuda_dev) for t in (a, sfa, b, sfb))
    L = nv.lib()
    s = torch.cuda.Stream(cuda_dev)

    def both():
        with torch.cuda.stream(s):
            d = nv.gemm(ta, tsa, tb, tsb, 0.5)
            dn = torch.empty_like(d)
            st = L.nvfp4_gemm_decode_noalloc(ta.data_ptr(), tsa.data_ptr(), tb.data_ptr(), tsb.data_ptr(), 0.5,
                                             dn.data_ptr(), M, N, K, s.cuda_stream)
            assert st == 0, L.nvfp4_status_string(st)
        s.synchronize()
        nv.device_status()
        return d, dn

    before = both()
    assert nv.selftest_wait_timeout(1_000_000) == -5  # reported: the timeout count moves
    after = both()
    ref32, _ = oracle.gemm(a, sfa, b, sfb, 0.5, M, N, K)
    for d in before + after:
        assert np.abs(d.float().cpu().numpy() - ref32).max() <= 1e-2 * np.abs(ref32).max()
    assert torch.equal(before[0], after[0]) and torch.equal(before[1], after[1])
