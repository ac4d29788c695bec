"""Column-parallel (N-sharded) NVFP4 GEMM across the GPUs of one node.

D = alpha * A . B^T with B [N, K/2] split by rows: rank p owns B rows
[n0_p, n1_p) and the matching slice of the blocked scales.  Shards are whole
128-row scale blocks, so each rank's slice of SFB is one contiguous byte range
(the blocked layout's outermost dimension is the 128-row block).  A and SFA are
replicated.  Each rank computes D_p = A . B_p^T [M, n1_p - n0_p] with no
communication; the full D is assembled with one all-gather only when asked for.

The reference has no multi-GPU path (its kernels and runner use one GPU and no
communication library); this module is new.  It is backend-agnostic (NCCL on GPUs, gloo in the
CPU tests) and takes the per-rank GEMM as a function so the host logic can be
tested without a GPU.
"""
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

SF_BLOCK = 128


def shard_bounds(N: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [n0, n1) of B owned by `rank`: the ceil(N/128) scale blocks are dealt
    out as evenly as possible (earlier ranks take the remainder), the last shard is
    clipped to N."""
    if not (0 <= rank < world):
        raise ValueError("rank out of range")
    blocks = (N + SF_BLOCK - 1) // SF_BLOCK
    base, rem = divmod(blocks, world)
    b0 = rank * base + min(rank, rem)
    b1 = b0 + base + (1 if rank < rem else 0)
    return min(b0 * SF_BLOCK, N), min(b1 * SF_BLOCK, N)


def shard_weight(b: torch.Tensor, sfb: torch.Tensor, K: int, world: int, rank: int):
    """This rank's (B rows, blocked SFB bytes) as views of the full operands."""
    N = b.shape[0]
    n0, n1 = shard_bounds(N, world, rank)
    per_block = SF_BLOCK * (K // 16)
    sf0 = (n0 // SF_BLOCK) * per_block
    sf1 = ((n1 + SF_BLOCK - 1) // SF_BLOCK) * per_block
    return b[n0:n1], sfb[sf0:sf1]


def column_parallel_gemm(a: torch.Tensor, sfa: torch.Tensor, b_shard: torch.Tensor, sfb_shard: torch.Tensor,
                         alpha: float, N: int, gather: bool = False, group=None,
                         gemm_fn: Optional[Callable] = None) -> torch.Tensor:
    """D_p for this rank, or (gather=True) the full [M, N] D on every rank.

    gemm_fn(a, sfa, b, sfb, alpha) -> [M, n_p] defaults to nvfp4_b200.gemm.
    """
    if gemm_fn is None:
        from .ops import gemm as gemm_fn
    if b_shard.shape[0] == 0:  # more ranks than 128-row blocks: nothing to compute here
        d_p = torch.empty(a.shape[0], 0, dtype=torch.bfloat16, device=a.device)
    else:
        d_p = gemm_fn(a, sfa, b_shard, sfb_shard, alpha)
    if not gather:
        return d_p
    return gather_columns(d_p, N, group=group)


def gather_columns(d_p: torch.Tensor, N: int, group=None) -> torch.Tensor:
    """All-gather column shards [M, n_p] (shard_bounds layout) into [M, N].

    Shards are padded to the largest shard so one all_gather_into_tensor moves
    everything ([P, M, n_max]); the local permute to [M, N] follows."""
    world = dist.get_world_size(group)
    M = d_p.shape[0]
    widths = [shard_bounds(N, world, r) for r in range(world)]
    n_max = max(n1 - n0 for n0, n1 in widths)
    send = d_p
    if d_p.shape[1] != n_max:
        send = torch.zeros(M, n_max, dtype=d_p.dtype, device=d_p.device)
        send[:, : d_p.shape[1]] = d_p
    recv = torch.empty(world * M, n_max, dtype=d_p.dtype, device=d_p.device)
    dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
    recv = recv.view(world, M, n_max)
    out = torch.empty(M, N, dtype=d_p.dtype, device=d_p.device)
    for r, (n0, n1) in enumerate(widths):
        out[:, n0:n1] = recv[r, :, : n1 - n0]
    return out


class FusedGather:
    """Column-parallel GEMM with the all-gather fused into the GEMM epilogue.

    The full [M, N] bf16 output lives in symmetric memory (one buffer per rank, mapped
    into every rank over NVLink).  `gemm` runs this rank's shard with
    nvfp4_gemm_gather, whose epilogue stores each output tile straight into every
    rank's full output — with one multimem store to the buffer's NVLink multicast
    address when the fabric offers one (the switch replicates it, so each GPU sends
    its shard once), else with one NVLink store per rank.  Two device-side barriers
    across the ranks (nvfp4_rank_barrier over the symmetric memory's signal pads, every
    wait bounded) bracket the GEMM: the first keeps a rank from writing into a peer's
    output before that peer's stream has reached this call (it may still be reading the
    previous result), the second orders all stores before anyone reads.  A barrier that
    times out latches NVFP4_ERR_TIMEOUT (nvfp4_device_status raises) and leaves the
    object unusable.  Unlike gather_columns, no separate collective moves the shards
    and no per-shard copy follows.  Shard widths and column offsets must be multiples
    of 16.

    Collective: every rank constructs it with the same (M, N) and calls `gemm` in the
    same order.
    """

    # Ranks from which the multicast form is the default: none within one node.
    # Measured for a 940 MB output (M=16384, N=28672): 2 ranks 0.86 ms with per-rank
    # stores vs 1.47 ms multicast, 4 ranks 1.11 vs 1.36 ms, 8 ranks 1.28 vs 1.35 ms.
    # Every rank must receive (P-1)/P of the output whichever form sends it, so the
    # incoming NVLink traffic bounds both (8 ranks: 822 MB at 770 GB/s = 1.07 ms);
    # multicast only saves outgoing traffic, and its stores through the switch run
    # slower than plain NVLink stores.
    MULTICAST_MIN_RANKS = 9

    def __init__(self, M: int, N: int, device: torch.device, group=None, multicast: Optional[bool] = None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        name = self.group.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            symm_mem.enable_symm_mem_for_group(name)
        self.M, self.N = M, N
        self.out = symm_mem.empty((M, N), dtype=torch.bfloat16, device=device)
        self.handle = symm_mem.rendezvous(self.out, name)
        rank = dist.get_rank(self.group)
        ptrs = list(self.handle.buffer_ptrs)
        off = self.out.data_ptr() - ptrs[rank]  # the tensor's place inside each rank's allocation
        want = multicast if multicast is not None else dist.get_world_size(self.group) >= self.MULTICAST_MIN_RANKS
        mc = int(self.handle.multicast_ptr or 0) if want else 0
        if multicast is True and not mc:
            raise RuntimeError("no NVLink multicast address for this buffer (NVLS unavailable)")
        self.multicast = bool(mc)
        self.dst = [mc + off] if mc else [p + off for p in ptrs]
        self.rank, self.world = rank, dist.get_world_size(self.group)
        self.pads = list(self.handle.signal_pad_ptrs)
        self.pad_bytes = int(self.handle.signal_pad_size)

    def _barrier(self, channel: int, stream: int) -> None:
        import ctypes as C
        from ._lib import check, lib
        arr = (C.c_uint64 * len(self.pads))(*self.pads)
        check(lib().nvfp4_rank_barrier(arr, self.world, self.rank, channel, self.pad_bytes, stream),
              "nvfp4_rank_barrier")

    def gemm(self, a: torch.Tensor, sfa: torch.Tensor, b_shard: torch.Tensor, sfb_shard: torch.Tensor,
             alpha: float, col_off: int) -> torch.Tensor:
        """Full D [M, N] on every rank; this rank contributes columns
        [col_off, col_off + b_shard.shape[0])."""
        import ctypes as C
        from ._lib import check, lib
        M, K, n = a.shape[0], a.shape[1] * 2, b_shard.shape[0]
        if M != self.M or col_off + n > self.N:
            raise ValueError("shard does not fit the gathered output")
        arr = (C.c_uint64 * len(self.dst))(*self.dst)
        stream = torch.cuda.current_stream(a.device).cuda_stream
        self._barrier(0, stream)
        if n > 0:
            check(lib().nvfp4_gemm_gather(a.data_ptr(), sfa.data_ptr(), b_shard.data_ptr(), sfb_shard.data_ptr(),
                                          float(alpha), M, n, K, arr, len(self.dst), int(self.multicast), self.N,
                                          col_off, stream), "nvfp4_gemm_gather")
        self._barrier(1, stream)
        return self.out
