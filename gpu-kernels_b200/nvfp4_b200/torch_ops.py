"""PyTorch custom operators over the C ABI: torch.ops.nvfp4_b200.gemm, .quantize,
.gemm_epilogue (bias + activation fused) and .gemm_nvfp4_out (the epilogue's
result quantized to NVFP4 for the next layer).

Registered with torch.library, so they carry schemas, run under torch.compile /
FX tracing as opaque ops (fake implementations give output shapes without a GPU)
and can be called from TorchScript-free model code the way the reference's
harness calls torch._scaled_mm (matmul/sm100_nvfp4/main.py:25-34).  The CUDA
implementations are the library's kernels; there is no CPU implementation.
"""
from typing import Optional, Tuple

import torch

from .layout import sf_bytes
from .ops import gemm as _gemm
from .ops import gemm_epilogue as _gemm_epilogue
from .ops import quantize as _quantize


@torch.library.custom_op("nvfp4_b200::gemm", mutates_args=(), device_types="cuda")
def gemm(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float,
         fp16_out: bool = False) -> torch.Tensor:
    """D = alpha * A . B^T; A [M, K/2] and B [N, K/2] e2m1 codes, blocked e4m3 scales;
    bf16 (or fp16) [M, N]."""
    return _gemm(a, sfa, b, sfb, alpha, out_dtype=torch.float16 if fp16_out else torch.bfloat16)


@gemm.register_fake
def _gemm_fake(a, sfa, b, sfb, alpha, fp16_out=False):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.float16 if fp16_out else torch.bfloat16)


@torch.library.custom_op("nvfp4_b200::quantize", mutates_args=(), device_types="cuda")
def quantize(x: torch.Tensor, global_scale: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (e2m1 codes uint8 [M, K/2], blocked e4m3 scales uint8 [pad128(M)*K/16])."""
    return _quantize(x, global_scale)


@quantize.register_fake
def _quantize_fake(x, global_scale):
    M, K = x.shape
    return (x.new_empty((M, K // 2), dtype=torch.uint8), x.new_empty((sf_bytes(M, K),), dtype=torch.uint8))


@torch.library.custom_op("nvfp4_b200::gemm_epilogue", mutates_args=(), device_types="cuda")
def gemm_epilogue(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float,
                  bias: Optional[torch.Tensor] = None, activation: str = "none") -> torch.Tensor:
    """bf16 D = act(alpha * A . B^T + bias) in one kernel."""
    return _gemm_epilogue(a, sfa, b, sfb, alpha, bias=bias, activation=activation)


@gemm_epilogue.register_fake
def _gemm_epilogue_fake(a, sfa, b, sfb, alpha, bias=None, activation="none"):
    N = b.shape[0] // 2 if activation == "swiglu" else b.shape[0]
    return a.new_empty((a.shape[0], N), dtype=torch.bfloat16)


@torch.library.custom_op("nvfp4_b200::gemm_nvfp4_out", mutates_args=(), device_types="cuda")
def gemm_nvfp4_out(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float,
                   out_global_scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
                   activation: str = "none") -> Tuple[torch.Tensor, torch.Tensor]:
    """act(alpha * A . B^T + bias) quantized to NVFP4 in the epilogue: (codes [M, N/2],
    blocked scales [pad128(M) * N/16]), the next layer's operand."""
    return _gemm_epilogue(a, sfa, b, sfb, alpha, bias=bias, activation=activation,
                          out_global_scale=out_global_scale)


@gemm_nvfp4_out.register_fake
def _gemm_nvfp4_out_fake(a, sfa, b, sfb, alpha, out_global_scale, bias=None, activation="none"):
    M, N = a.shape[0], b.shape[0] // 2 if activation == "swiglu" else b.shape[0]
    return (a.new_empty((M, N // 2), dtype=torch.uint8), a.new_empty((sf_bytes(M, N),), dtype=torch.uint8))
