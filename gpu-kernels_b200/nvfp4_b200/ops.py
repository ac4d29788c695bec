"""torch-facing front end of the C ABI (the reference's Python side,
matmul/sm100_nvfp4/main.py, works on torch tensors in exactly these formats).

Operands may be given as uint8 / int8 / float4_e2m1fn_x2 (codes) and uint8 /
float8_e4m3fn (scales) tensors: only the bytes matter.  All calls are
asynchronous on torch's current CUDA stream and raise NVFP4Error on a bad
status.  Nothing here computes on the CPU.
"""
import ctypes as C
from typing import Optional, Tuple, Union

import torch

from ._lib import ACTIVATIONS, Epilogue, NVFP4Error, check, lib
from .layout import grouped_sf_bytes, sf_bytes, to_blocked


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _bytes_tensor(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.element_size() != 1:
        raise ValueError(f"{name} must be a 1-byte dtype (codes/scales), got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _scale_tensor(gs: Union[torch.Tensor, float], device: torch.device) -> torch.Tensor:
    if isinstance(gs, torch.Tensor):
        if gs.dtype != torch.float32 or gs.numel() != 1 or gs.device != device:
            raise ValueError("global_scale must be a 1-element float32 tensor on the input's device")
        return gs
    return torch.tensor([float(gs)], dtype=torch.float32, device=device)


def global_scale(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(amax, gs) of a bf16 tensor as 1-element fp32 device tensors, gs = amax/(6*448)."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 CUDA tensor")
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    gs = torch.empty(1, dtype=torch.float32, device=x.device)
    check(lib().nvfp4_global_scale(x.data_ptr(), x.numel(), amax.data_ptr(), gs.data_ptr(),
                                   _stream(x.device)), "nvfp4_global_scale")
    return amax, gs


def quantize(x: torch.Tensor, global_scale: Union[torch.Tensor, float],
             q_out: Optional[torch.Tensor] = None,
             sf_out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (codes uint8 [M, K/2], blocked e4m3 scales uint8 [pad128(M)*K/16])."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bf16 CUDA tensor")
    M, K = x.shape
    gs = _scale_tensor(global_scale, x.device)
    q = q_out if q_out is not None else torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    sf = sf_out if sf_out is not None else torch.empty(sf_bytes(M, K), dtype=torch.uint8, device=x.device)
    check(lib().nvfp4_quantize(x.data_ptr(), q.data_ptr(), sf.data_ptr(), gs.data_ptr(), M, K,
                               _stream(x.device)), "nvfp4_quantize")
    return q, sf


def gemm(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float = 1.0,
         out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """D[M, N] = alpha * A . B^T for NVFP4 A [M, K/2], B [N, K/2] with blocked scales."""
    for t, n in ((a, "a"), (sfa, "sfa"), (b, "b"), (sfb, "sfb")):
        _bytes_tensor(t, n)
    M, K = a.shape[0], a.shape[1] * 2
    N = b.shape[0]
    if b.shape[1] * 2 != K:
        raise ValueError("A and B must have the same K")
    if sfa.numel() < sf_bytes(M, K) or sfb.numel() < sf_bytes(N, K):
        raise ValueError("scale tensors too small for the blocked layout (rows padded to 128)")
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("out_dtype must be bf16 or fp16")
    d = out if out is not None else torch.empty(M, N, dtype=out_dtype, device=a.device)
    if d.dtype != out_dtype or d.shape != (M, N) or not d.is_contiguous():
        raise ValueError("out must be a contiguous [M, N] tensor of out_dtype")
    fn = lib().nvfp4_gemm if out_dtype == torch.bfloat16 else lib().nvfp4_gemm_f16
    check(fn(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), float(alpha), d.data_ptr(), M, N, K,
             _stream(a.device)), "nvfp4_gemm")
    return d


def gemm_epilogue(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float = 1.0,
                  bias: Optional[torch.Tensor] = None, activation: str = "none",
                  out_global_scale: Union[torch.Tensor, float, None] = None, out: Optional[torch.Tensor] = None,
                  q_out: Optional[torch.Tensor] = None, sf_out: Optional[torch.Tensor] = None):
    """D = act(alpha * A . B^T + bias) in one kernel (nvfp4_gemm_epilogue).

    Without `out_global_scale`: returns bf16 D [M, N].  With it: D is quantized to
    NVFP4 in the epilogue (N % 64 == 0) and (codes uint8 [M, N/2], blocked scales
    uint8 [pad128(M) * N/16]) are returned — the bytes nvfp4_quantize would give
    for the bf16 result.  activation "swiglu": B's rows are gate / up weights
    interleaved in blocks of 16 (swiglu_interleave), bias likewise, and the output
    has N/2 columns, silu(gate) * up (N % 128 == 0)."""
    for t, n in ((a, "a"), (sfa, "sfa"), (b, "b"), (sfb, "sfb")):
        _bytes_tensor(t, n)
    M, K, N = a.shape[0], a.shape[1] * 2, b.shape[0]
    if b.shape[1] * 2 != K:
        raise ValueError("A and B must have the same K")
    if sfa.numel() < sf_bytes(M, K) or sfb.numel() < sf_bytes(N, K):
        raise ValueError("scale tensors too small for the blocked layout (rows padded to 128)")
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}")
    e = Epilogue()
    e.activation = ACTIVATIONS[activation]
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != N or not bias.is_cuda or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous bf16 CUDA tensor of N elements")
        e.bias = bias.data_ptr()
    No = N // 2 if activation == "swiglu" else N  # output columns
    d = None
    if out_global_scale is None:
        d = out if out is not None else torch.empty(M, No, dtype=torch.bfloat16, device=a.device)
        if d.dtype != torch.bfloat16 or d.shape != (M, No) or not d.is_contiguous():
            raise ValueError(f"out must be a contiguous bf16 [M, {No}] tensor")
        d_ptr = d.data_ptr()
    else:
        gs = _scale_tensor(out_global_scale, a.device)
        q = q_out if q_out is not None else torch.empty(M, No // 2, dtype=torch.uint8, device=a.device)
        sf = sf_out if sf_out is not None else torch.empty(sf_bytes(M, No), dtype=torch.uint8, device=a.device)
        e.q_out, e.sf_out, e.out_global_scale = q.data_ptr(), sf.data_ptr(), gs.data_ptr()
        d_ptr = None
    check(lib().nvfp4_gemm_epilogue(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), float(alpha), d_ptr,
                                    M, N, K, C.byref(e), _stream(a.device)), "nvfp4_gemm_epilogue")
    return d if d is not None else (q, sf)


def quantize_dynamic(x: torch.Tensor, q_out: Optional[torch.Tensor] = None,
                     sf_out: Optional[torch.Tensor] = None):
    """global_scale + quantize in one kernel (nvfp4_quantize_dynamic): bf16 [M, K] ->
    (codes [M, K/2], blocked scales, gs fp32 [1] on the device), byte-identical to
    quantize(x, global_scale(x)[1])."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bf16 CUDA tensor")
    M, K = x.shape
    q = q_out if q_out is not None else torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    sf = sf_out if sf_out is not None else torch.empty(sf_bytes(M, K), dtype=torch.uint8, device=x.device)
    gs = torch.empty(1, dtype=torch.float32, device=x.device)
    check(lib().nvfp4_quantize_dynamic(x.data_ptr(), q.data_ptr(), sf.data_ptr(), None, gs.data_ptr(), M, K,
                                       _stream(x.device)), "nvfp4_quantize_dynamic")
    return q, sf, gs


def _offsets_tensor(m_offsets: torch.Tensor, device: torch.device) -> torch.Tensor:
    if m_offsets.dtype != torch.int32 or m_offsets.dim() != 1 or m_offsets.numel() < 2 or \
            m_offsets.device != device or not m_offsets.is_contiguous():
        raise ValueError("m_offsets must be a contiguous 1-D int32 tensor of groups + 1 entries on the device")
    return m_offsets


def quantize_grouped(x: torch.Tensor, global_scale: Union[torch.Tensor, float], m_offsets: torch.Tensor,
                     q_out: Optional[torch.Tensor] = None,
                     sf_out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [m_total, K] stacked by group -> (codes [m_total, K/2], grouped scales of
    grouped_sf_bytes(m_total, groups, K) bytes: each group's blocked tensor starting on
    a 128-row block).  m_offsets: device int32 [groups + 1]."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bf16 CUDA tensor")
    m_total, K = x.shape
    offs = _offsets_tensor(m_offsets, x.device)
    G = offs.numel() - 1
    gs = _scale_tensor(global_scale, x.device)
    q = q_out if q_out is not None else torch.empty(m_total, K // 2, dtype=torch.uint8, device=x.device)
    sf = sf_out if sf_out is not None else torch.empty(grouped_sf_bytes(m_total, G, K), dtype=torch.uint8,
                                                       device=x.device)
    check(lib().nvfp4_quantize_grouped(x.data_ptr(), q.data_ptr(), sf.data_ptr(), gs.data_ptr(), offs.data_ptr(), G,
                                       m_total, K, _stream(x.device)), "nvfp4_quantize_grouped")
    return q, sf


def gemm_grouped(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alphas: torch.Tensor,
                 m_offsets: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Grouped (mixture-of-experts) GEMM: rows [m_offsets[g], m_offsets[g+1]) of the
    stacked A times expert g's weight B[g*N:(g+1)*N], scaled by alphas[g] -> bf16 D
    [m_total, N].  sfa in the grouped layout (quantize_grouped), sfb the experts'
    blocked scales concatenated; alphas fp32 [groups] and m_offsets int32 [groups + 1]
    on the device.  Rows outside every group are left as they are in `out`."""
    for t, n in ((a, "a"), (sfa, "sfa"), (b, "b"), (sfb, "sfb")):
        _bytes_tensor(t, n)
    offs = _offsets_tensor(m_offsets, a.device)
    G = offs.numel() - 1
    m_total, K = a.shape[0], a.shape[1] * 2
    if b.shape[1] * 2 != K or b.shape[0] % G:
        raise ValueError("B must be [groups * N, K/2] with A's K")
    N = b.shape[0] // G
    if sfa.numel() < grouped_sf_bytes(m_total, G, K) or sfb.numel() < G * sf_bytes(N, K):
        raise ValueError("scale tensors too small for the grouped layout")
    if alphas.dtype != torch.float32 or alphas.numel() != G or alphas.device != a.device:
        raise ValueError("alphas must be a float32 tensor of groups entries on the device")
    d = out if out is not None else torch.zeros(m_total, N, dtype=torch.bfloat16, device=a.device)
    if d.dtype != torch.bfloat16 or d.shape != (m_total, N) or not d.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [m_total, N] tensor")
    check(lib().nvfp4_gemm_grouped(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), alphas.data_ptr(),
                                   d.data_ptr(), offs.data_ptr(), G, m_total, N, K, _stream(a.device)),
          "nvfp4_gemm_grouped")
    return d


def gemm_grouped_epilogue(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor,
                          alphas: torch.Tensor, m_offsets: torch.Tensor, bias: Optional[torch.Tensor] = None,
                          activation: str = "none", out_global_scale: Union[torch.Tensor, float, None] = None,
                          out: Optional[torch.Tensor] = None, q_out: Optional[torch.Tensor] = None,
                          sf_out: Optional[torch.Tensor] = None):
    """gemm_grouped with the fused epilogue (nvfp4_gemm_grouped_epilogue): D =
    act(alphas[g] * A . B_g^T + bias[g]) per group, bias bf16 [groups, N] (optional).
    Without `out_global_scale`: returns bf16 D [m_total, N].  With it: returns
    (codes uint8 [m_total, N/2], scales in the grouped layout of
    grouped_sf_bytes(m_total, groups, N) bytes) — what quantize_grouped makes of the
    bf16 result, ready as the A operand of the next grouped GEMM (N % 128 == 0).
    activation "swiglu" as in gemm_epilogue: N/2 output columns."""
    for t, n in ((a, "a"), (sfa, "sfa"), (b, "b"), (sfb, "sfb")):
        _bytes_tensor(t, n)
    offs = _offsets_tensor(m_offsets, a.device)
    G = offs.numel() - 1
    m_total, K = a.shape[0], a.shape[1] * 2
    if b.shape[1] * 2 != K or b.shape[0] % G:
        raise ValueError("B must be [groups * N, K/2] with A's K")
    N = b.shape[0] // G
    if sfa.numel() < grouped_sf_bytes(m_total, G, K) or sfb.numel() < G * sf_bytes(N, K):
        raise ValueError("scale tensors too small for the grouped layout")
    if alphas.dtype != torch.float32 or alphas.numel() != G or alphas.device != a.device:
        raise ValueError("alphas must be a float32 tensor of groups entries on the device")
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}")
    e = Epilogue()
    e.activation = ACTIVATIONS[activation]
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != G * N or not bias.is_cuda or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous bf16 CUDA tensor of groups * N elements")
        e.bias = bias.data_ptr()
    No = N // 2 if activation == "swiglu" else N  # output columns
    d = None
    if out_global_scale is None:
        d = out if out is not None else torch.zeros(m_total, No, dtype=torch.bfloat16, device=a.device)
        if d.dtype != torch.bfloat16 or d.shape != (m_total, No) or not d.is_contiguous():
            raise ValueError(f"out must be a contiguous bf16 [m_total, {No}] tensor")
        d_ptr = d.data_ptr()
    else:
        gs = _scale_tensor(out_global_scale, a.device)
        q = q_out if q_out is not None else torch.zeros(m_total, No // 2, dtype=torch.uint8, device=a.device)
        sf = sf_out if sf_out is not None else torch.zeros(grouped_sf_bytes(m_total, G, No), dtype=torch.uint8,
                                                           device=a.device)
        e.q_out, e.sf_out, e.out_global_scale = q.data_ptr(), sf.data_ptr(), gs.data_ptr()
        d_ptr = None
    check(lib().nvfp4_gemm_grouped_epilogue(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(),
                                            alphas.data_ptr(), d_ptr, offs.data_ptr(), G, m_total, N, K, C.byref(e),
                                            _stream(a.device)), "nvfp4_gemm_grouped_epilogue")
    return d if d is not None else (q, sf)


def gemm_host(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float,
              out: torch.Tensor, device: Optional[torch.device] = None) -> torch.Tensor:
    """D = alpha * A . B^T from and to HOST tensors (pin them for overlap): uploads,
    per-block GEMMs and the copy of D back are pipelined inside the library.
    Asynchronous on the device's current stream; synchronise before reading `out`."""
    for t, n in ((a, "a"), (sfa, "sfa"), (b, "b"), (sfb, "sfb")):
        if t.is_cuda or t.element_size() != 1 or not t.is_contiguous():
            raise ValueError(f"{n} must be a contiguous 1-byte host tensor")
    M, K, N = a.shape[0], a.shape[1] * 2, b.shape[0]
    if out.is_cuda or out.dtype != torch.bfloat16 or out.shape != (M, N) or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [M, N] host tensor")
    dev = device or torch.device("cuda", torch.cuda.current_device())
    check(lib().nvfp4_gemm_host(a.data_ptr(), sfa.data_ptr(), b.data_ptr(), sfb.data_ptr(), float(alpha),
                                out.data_ptr(), M, N, K, _stream(dev)), "nvfp4_gemm_host")
    return out


def matmul_nvfp4(c: torch.Tensor, sfa: torch.Tensor, sfb: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                 M: int, N: int, K: int) -> None:
    """Reference launcher signature (matmul/sm100_nvfp4/block_scaled_nvfp4.cuh:7-18):
    fp16 c [M, N] = A . B^T on the legacy default stream, through the C shim
    matmul_nvfp4_b200; raises if the call's status is not OK."""
    lib().matmul_nvfp4_b200(c.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), a.data_ptr(), b.data_ptr(), M, N, K)
    check(lib().nvfp4_last_status(), "matmul_nvfp4_b200")


def create_tensors(M: int, N: int, K: int, sf_vec_size: int = 16, seed: int = 42, device: str = "cuda"):
    """Operands in the reference's test distribution (matmul/sm100_nvfp4/main.py:9-23):
    uniformly random e2m1 byte codes, e4m3 scale codes 0..3, scales blocked."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    a = torch.randint(-128, 127, (M, K // 2), dtype=torch.int8, device=device, generator=g)
    b = torch.randint(-128, 127, (N, K // 2), dtype=torch.int8, device=device, generator=g)
    sfa = torch.randint(0, 4, (M, K // sf_vec_size), dtype=torch.int8, device=device, generator=g)
    sfb = torch.randint(0, 4, (N, K // sf_vec_size), dtype=torch.int8, device=device, generator=g)
    return (a.view(torch.uint8), b.view(torch.uint8), to_blocked(sfa.view(torch.uint8)),
            to_blocked(sfb.view(torch.uint8)))


def device_status(device: Optional[torch.device] = None) -> None:
    """Synchronise and raise NVFP4Error(NVFP4_ERR_TIMEOUT) if a kernel gave up a wait."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    check(lib().nvfp4_device_status(_stream(dev)), "device status")


def set_wait_timeout_ns(ns: int) -> None:
    lib().nvfp4_set_wait_timeout_ns(int(ns))


def selftest_wait_timeout(ns: int = 1_000_000) -> int:
    return lib().nvfp4_selftest_wait_timeout(int(ns))


def launch_count() -> int:
    return int(lib().nvfp4_launch_count())


__all__ = ["NVFP4Error", "global_scale", "quantize", "quantize_grouped", "gemm", "gemm_epilogue", "gemm_grouped",
           "gemm_host", "matmul_nvfp4",
           "create_tensors", "device_status", "set_wait_timeout_ns", "selftest_wait_timeout", "launch_count"]
