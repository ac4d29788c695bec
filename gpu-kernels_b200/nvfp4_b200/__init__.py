"""nvfp4_b200 — B200-native (sm_100a) NVFP4 block-scaled GEMM and bf16 -> NVFP4 quantizer.

Host-side mirror of the reference's plugin surface (Parth-Badgujar/gpu-kernels,
matmul/sm100_nvfp4/): the C ABI lives in libnvfp4_b200.so (include/nvfp4_b200.h);
this package binds it for torch tensors.  Import path: put `gpu-kernels_b200/`
on sys.path (the repository's conftest, bench.py and __graft_entry__ do).
"""
from ._lib import LIB_PATH, NVFP4Error, SIGNATURES, lib  # noqa: F401
from .layout import (from_blocked, grouped_sf_block0, grouped_sf_bytes, pad128, sf_bytes, sf_offset,  # noqa: F401
                     swiglu_interleave, to_blocked)
from .ops import (create_tensors, device_status, gemm, gemm_epilogue, gemm_grouped,  # noqa: F401
                  gemm_grouped_epilogue, gemm_host, global_scale, launch_count, matmul_nvfp4, quantize,
                  quantize_dynamic, quantize_grouped, selftest_wait_timeout, set_wait_timeout_ns)
from . import runner_io  # noqa: F401,E402
from . import torch_ops  # noqa: F401,E402  (registers torch.ops.nvfp4_b200.gemm / .quantize)
