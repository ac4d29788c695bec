"""CPU: the column-parallel (N-sharded) path's host logic with gloo ranks.

Each rank computes its D shard with the CPU oracle (standing in for the GPU
kernel, which the sharding code takes as a function) and the shards are
all-gathered; the result must equal the unsharded oracle GEMM exactly.  Also:
shard bounds, the contiguity of each rank's blocked-scale slice, and a rank that
fails before the collective turning into an error on its peer, not a hang."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_and_align():
    from nvfp4_b200.dist import shard_bounds
    for N in (8, 128, 136, 1000, 8192, 28672, 28680):
        for world in (1, 2, 3, 4, 8):
            bounds = [shard_bounds(N, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == N
            for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
                assert a1 == b0
            for n0, n1 in bounds:
                assert n0 <= n1
                assert n0 % 128 == 0 or n0 == n1 == N  # empty trailing shards sit at N


def test_shard_weight_scale_slice_is_the_blocked_layout_of_the_rows(oracle):
    from nvfp4_b200.dist import shard_weight
    from nvfp4_b200.layout import to_blocked
    N, K = 1000, 256
    b, sfb = oracle.random_codes(N, K, seed=3, sf_lo=0x30, sf_hi=0x40)
    sf_rm = oracle.sf_unpack(sfb, N, K)
    tb, tsfb = torch.from_numpy(b), torch.from_numpy(sfb)
    for world in (2, 3, 8):
        for rank in range(world):
            bs, ss = shard_weight(tb, tsfb, K, world, rank)
            rows = bs.shape[0]
            if rows == 0:
                continue
            start = rank and sum(shard_weight(tb, tsfb, K, world, r)[0].shape[0] for r in range(rank))
            expect = to_blocked(torch.from_numpy(sf_rm[start:start + rows]))
            assert torch.equal(ss[: expect.numel()], expect)


def _worker(rank, world, port, M, N, K, q):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "gpu-kernels_b200")]
    from oracle import oracle as o
    from nvfp4_b200.dist import column_parallel_gemm, shard_weight
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        a, sfa = o.random_codes(M, K, seed=1, sf_lo=0x30, sf_hi=0x40)
        b, sfb = o.random_codes(N, K, seed=2, sf_lo=0x30, sf_hi=0x40)
        bs, ss = shard_weight(torch.from_numpy(b), torch.from_numpy(sfb), K, world, rank)

        def cpu_gemm(a_, sfa_, b_, sfb_, alpha):
            n = b_.shape[0]
            d32, _ = o.gemm(a_.numpy(), sfa_.numpy(), b_.numpy(), sfb_.numpy(), alpha, M, n, K, nthreads=1)
            return torch.from_numpy(d32)

        d = column_parallel_gemm(torch.from_numpy(a), torch.from_numpy(sfa), bs, ss, 0.5, N, gather=True,
                                 gemm_fn=cpu_gemm)
        if rank == 0:
            full, _ = o.gemm(a, sfa, b, sfb, 0.5, M, N, K, nthreads=1)
            q.put(bool(np.array_equal(d.numpy(), full)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 512), (2, 392), (4, 1000)])
def test_column_parallel_gather_matches_unsharded(world, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 96, N, 256, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def _failing_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(3)  # dies between steps, before the collective
    try:
        t = torch.zeros(4)
        out = torch.empty(8)
        dist.all_gather_into_tensor(out, t)
        q.put("no error")
    except Exception as e:  # the peer learns of the failure as an error
        q.put(type(e).__name__)


def test_dead_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert procs[1].exitcode == 3
    assert q.get(timeout=5) != "no error"


def test_gemm_gather_host_checks(nv):
    """nvfp4_gemm_gather rejects bad arguments on the host, before any device call."""
    import ctypes as C
    L = nv.lib()
    f = 0x10000
    dst = (C.c_uint64 * 2)(f, f + 4096)

    def call(M=256, N=256, K=256, d=dst, n_dst=2, mc=0, ld=512, col_off=256):
        return L.nvfp4_gemm_gather(f, f, f, f, 1.0, M, N, K, d, n_dst, mc, ld, col_off, None)

    assert call(N=200) == -2                    # N % 16
    assert call(ld=400) == -2                   # ld < col_off + N
    assert call(col_off=8) == -2                # col_off % 16
    assert call(n_dst=9) == -2                  # more ranks than the kernel carries
    assert call(mc=1) == -2                     # a multicast address is one destination
    assert call(d=None) == -1
    bad = (C.c_uint64 * 2)(f, f + 16)           # destinations 32-byte aligned
    assert call(d=bad) == -3
    zero = (C.c_uint64 * 2)(f, 0)
    assert call(d=zero) == -1
