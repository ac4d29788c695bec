"""GPU, 2+ devices: the column-parallel NVFP4 GEMM over NCCL.

Each rank computes its 128-row-block shard of B with the CTA-pair kernel and the
bf16 shards are all-gathered; the gathered D must equal the unsharded GEMM on one
GPU bit for bit (every output element is accumulated by one CTA over the same K
order however N is split).  Skipped when fewer than two GPUs are visible."""
import datetime
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _operands(M, N, K, dev):
    sys.path[:0] = [os.path.join(ROOT, "gpu-kernels_b200")]
    import nvfp4_b200 as nv
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    xa = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    xb = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    _, ga = nv.global_scale(xa)
    _, gb = nv.global_scale(xb)
    a, sfa = nv.quantize(xa, ga)
    b, sfb = nv.quantize(xb, gb)
    return nv, a, sfa, b, sfb


def _rank(rank, world, port, M, N, K, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        nv, a, sfa, b, sfb = _operands(M, N, K, dev)
        from nvfp4_b200.dist import column_parallel_gemm, shard_weight
        bs, ss = shard_weight(b, sfb, K, world, rank)
        d = column_parallel_gemm(a, sfa, bs.contiguous(), ss.contiguous(), 0.5, N, gather=True)
        torch.cuda.synchronize()
        nv.device_status()
        if rank == 0:
            full = nv.gemm(a, sfa, b, sfb, 0.5)
            torch.cuda.synchronize()
            q.put(bool(torch.equal(d, full)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(512, 3072, 1024), (300, 1288, 2048)])
def test_column_parallel_nccl_matches_single_gpu(M, N, K):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    _join_without_kill(procs, 300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def _agree(dist, world, value):
    """Every rank's value (an all-gather of Python objects, bounded by the process
    group's timeout)."""
    vals = [None] * world
    dist.all_gather_object(vals, value)
    return vals


def _rank_fused(rank, world, port, M, N, K, q):
    """Fused GEMM + all-gather (nvfp4_gemm_gather through symmetric memory): NVLink
    stores to every rank's buffer first; the NVLink-multicast form only once every rank
    matched and every rank has a multicast address.  Every wait here is bounded: the
    process group's 60 s timeout, and the library's own device waits (its rank barrier
    included, limit 5 s) — so every rank returns by itself, and it releases its
    symmetric buffers and the process group on the way out whatever happened."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    result = {"unicast": None, "multicast": None}
    fg = probe = d = d2 = None
    try:
        nv, a, sfa, b, sfb = _operands(M, N, K, dev)
        nv.set_wait_timeout_ns(5_000_000_000)
        from nvfp4_b200.dist import FusedGather, shard_bounds, shard_weight
        bs, ss = shard_weight(b, sfb, K, world, rank)
        n0, _ = shard_bounds(N, world, rank)
        full = nv.gemm(a, sfa, b, sfb, 0.5)
        fg = FusedGather(M, N, dev, multicast=False)
        fg.out.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        d = fg.gemm(a, sfa, bs.contiguous(), ss.contiguous(), 0.5, n0)
        torch.cuda.synchronize()
        nv.device_status()  # raises if a bounded wait gave up
        result["unicast"] = bool(torch.equal(d, full))
        if all(_agree(dist, world, result["unicast"])):
            try:
                probe = FusedGather(M, N, dev, multicast=True)
            except RuntimeError:
                probe = None
            have = probe is not None and probe.multicast
            if all(_agree(dist, world, have)):  # every rank takes the multicast arm, or none does
                probe.out.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                d2 = probe.gemm(a, sfa, bs.contiguous(), ss.contiguous(), 0.5, n0)
                torch.cuda.synchronize()
                nv.device_status()
                result["multicast"] = bool(torch.equal(d2, full))
            else:
                result["multicast"] = "unavailable"
        if rank == 0:
            q.put(result)
    finally:
        try:
            torch.cuda.synchronize()
        finally:
            fg = probe = d = d2 = None  # symmetric buffers released before the group goes
            dist.destroy_process_group()


def _join_without_kill(procs, limit_s):
    """Wait for the ranks; never kill one (a rank may hold memory bound to an NVLink
    multicast object).  Every wait inside the ranks is bounded, so they end by
    themselves; a rank still running after `limit_s` fails the test."""
    import time
    deadline = time.monotonic() + limit_s
    for p in procs:
        p.join(timeout=max(0.0, deadline - time.monotonic()))
    alive = [i for i, p in enumerate(procs) if p.is_alive()]
    assert not alive, f"ranks {alive} still running after {limit_s} s"


@pytest.mark.parametrize("M,N,K", [(512, 3072, 1024), (300, 1280, 2048)])
def test_fused_gather_matches_single_gpu(M, N, K):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_fused, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    _join_without_kill(procs, 300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=5)
    print("fused gather:", res)
    assert res["unicast"] is True
    assert res["multicast"] in (True, "unavailable")
