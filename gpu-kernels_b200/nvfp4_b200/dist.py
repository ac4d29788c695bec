"""Column-parallel (N-sharded) NVFP4 GEMM across the GPUs of one node.

D = alpha * A . B^T with B [N, K/2] split by rows: rank p owns B rows
[n0_p, n1_p) and the matching slice of the blocked scales.  Shards are whole
128-row scale blocks, so each rank's slice of SFB is one contiguous byte range
(the blocked layout's outermost dimension is the 128-row block).  A and SFA are
replicated.  Each rank computes D_p = A . B_p^T [M, n1_p - n0_p] with no
communication; the full D is assembled with one all-gather only when asked for.

The reference has no multi-GPU path (SURVEY: "Distributed communication backend:
none"); this module is new.  It is backend-agnostic (NCCL on GPUs, gloo in the
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
