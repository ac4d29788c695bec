"""Scale-factor layout helpers (torch, any device).

The reference stores one e4m3 scale per 16 K-elements in the cuBLAS "128x4
blocked" layout built in matmul/sm100_nvfp4/main.py:16-22:

    sf.reshape(rows/128, 4, 32, K/64, 4).permute(0, 3, 2, 1, 4).flatten()

so that each 128-row x 64-K block is 512 contiguous bytes whose line i (16 B)
holds rows i, i+32, i+64, i+96 — the order tcgen05.cp 32x128b.warpx4 replicates
into tensor memory for the block-scaled MMA.
"""
import torch


def pad128(rows: int) -> int:
    return (rows + 127) // 128 * 128


def sf_bytes(rows: int, K: int) -> int:
    """Size of a blocked scale tensor for `rows` rows (padded to 128) and K."""
    return pad128(rows) * (K // 16)


def sf_offset(r: int, k16: int, K: int) -> int:
    return ((r // 128) * (K // 64) + k16 // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + k16 % 4


def to_blocked(sf_rowmajor: torch.Tensor) -> torch.Tensor:
    """[rows, K/16] uint8 (row-major) -> flat blocked uint8 of pad128(rows)*K/16.
    Padding rows are zero."""
    rows, kb = sf_rowmajor.shape
    assert kb % 4 == 0, "K must be a multiple of 64"
    rp = pad128(rows)
    src = sf_rowmajor.view(torch.uint8)
    if rp != rows:
        src = torch.cat([src, src.new_zeros(rp - rows, kb)], 0)
    return src.reshape(rp // 128, 4, 32, kb // 4, 4).permute(0, 3, 2, 1, 4).contiguous().flatten()


def from_blocked(sf_blocked: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """Inverse of to_blocked: flat blocked -> [rows, K/16] uint8."""
    rp, kb = pad128(rows), K // 16
    t = sf_blocked.view(torch.uint8).reshape(rp // 128, kb // 4, 32, 4, 4).permute(0, 3, 2, 1, 4)
    return t.reshape(rp, kb)[:rows].contiguous()


def grouped_sf_bytes(m_total: int, groups: int, K: int) -> int:
    """Capacity of a grouped scale buffer: each group's blocked tensor starts on a
    128-row block, so at most ceil(m_total/128) + groups blocks of 128 x K/16 bytes."""
    return ((m_total + 127) // 128 + groups) * 128 * (K // 16)


def grouped_sf_block0(m_offsets):
    """First 128-row scale block of each group (host copy of the device rule)."""
    out, b = [], 0
    for g in range(len(m_offsets) - 1):
        out.append(b)
        b += (max(0, m_offsets[g + 1] - m_offsets[g]) + 127) // 128
    out.append(b)
    return out


def swiglu_interleave(gate, up, block: int = 16):
    """Interleave the rows of a gate and an up weight (or bias) of F rows each into the
    [2F, ...] order the "swiglu" epilogue reads: rows 32j .. 32j+15 = gate rows
    16j .. 16j+15, rows 32j+16 .. 32j+31 = the matching up rows.  Works on torch
    tensors or numpy arrays; quantize the interleaved bf16 weight as usual."""
    if gate.shape != up.shape or gate.shape[0] % block:
        raise ValueError(f"gate and up must have the same shape with rows a multiple of {block}")
    F = gate.shape[0]
    rest = tuple(gate.shape[1:])
    try:
        import torch
        if isinstance(gate, torch.Tensor):
            return torch.stack((gate.reshape(F // block, block, *rest), up.reshape(F // block, block, *rest)),
                               dim=1).reshape(2 * F, *rest)
    except ImportError:
        pass
    import numpy as np
    return np.stack((gate.reshape(F // block, block, *rest), up.reshape(F // block, block, *rest)),
                    axis=1).reshape(2 * F, *rest)
