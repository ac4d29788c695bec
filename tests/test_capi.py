"""CPU: the C-ABI library loads and exports every symbol include/nvfp4_b200.h
declares; host-side argument checks answer without touching a GPU."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nvfp4_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^NVFP4_API\s+[\w\s\*]*?\b(\w+)\s*\(", text, re.M)))


def test_header_declares_the_boundary():
    names = declared_symbols()
    for required in ("nvfp4_quantize", "nvfp4_gemm", "matmul_nvfp4_b200", "nvfp4_global_scale",
                     "nvfp4_device_status", "nvfp4_selftest_wait_timeout"):
        assert required in names


def test_library_exports_every_declared_symbol(nv):
    L = nv.lib()
    raw = C.CDLL(nv.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(raw, name), f"{name} not exported"
        assert name in nv.SIGNATURES, f"{name} missing from the ctypes signature table"
    assert set(nv.SIGNATURES) == set(declared_symbols())
    assert L.nvfp4_version() > 0


def test_status_strings(nv):
    L = nv.lib()
    for code in range(0, -8, -1):
        assert L.nvfp4_status_string(code)
    assert b"unknown" in L.nvfp4_status_string(-99)


@pytest.mark.parametrize("M,N,K,status", [
    (0, 256, 256, -2), (128, 4, 256, -2), (128, 12, 256, -2), (128, 256, 32, -2), (128, 256, 96, -2),
])
def test_gemm_rejects_bad_shapes_on_host(nv, M, N, K, status):
    L = nv.lib()
    p = C.c_void_p(1 << 20)  # never dereferenced: validation runs first
    assert L.nvfp4_gemm(p, p, p, p, 1.0, p, M, N, K, None) == status


def test_gemm_rejects_null_and_misaligned(nv):
    L = nv.lib()
    p = C.c_void_p(1 << 20)
    assert L.nvfp4_gemm(None, p, p, p, 1.0, p, 128, 256, 256, None) == -1
    assert L.nvfp4_gemm(C.c_void_p((1 << 20) + 8), p, p, p, 1.0, p, 128, 256, 256, None) == -3
    assert L.nvfp4_quantize(p, p, p, None, 128, 256, None) == -1
    assert L.nvfp4_quantize(p, p, p, p, 128, 100, None) == -2


def test_no_gpu_call_fails_cleanly_without_device(nv):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    L = nv.lib()
    p = C.c_void_p(1 << 20)
    # valid arguments reach the device query, which reports an error (no crash, no exit)
    assert L.nvfp4_gemm(p, p, p, p, 1.0, p, 128, 256, 256, None) in (-4, -6)


def test_quantize_dynamic_rejects_bad_arguments_on_host(nv):
    L = nv.lib()
    f = 0x10000  # never dereferenced: every case fails its host-side check first
    assert L.nvfp4_quantize_dynamic(None, f, f, None, f, 128, 256, None) == -1      # no X
    assert L.nvfp4_quantize_dynamic(f, f, f, None, f, 128, 100, None) == -2         # K % 64
    assert L.nvfp4_quantize_dynamic(f, f, f, None, f, 0, 256, None) == -2           # M < 1
    assert L.nvfp4_quantize_dynamic(f + 16, f, f, None, f, 128, 256, None) == -3    # X 32-byte aligned
    assert L.nvfp4_quantize_dynamic(f, f, f, None, f + 2, 128, 256, None) == -3     # gs 4-byte aligned


DIAG_HEADER = os.path.join(ROOT, "gpu-kernels_b200", "nvfp4_diag", "nvfp4_diag.h")


def test_product_library_holds_no_diagnostics(nv):
    """The traced kernels, the tensor-rate probe and the scale-code check are in the
    separate diagnostic library only."""
    raw = C.CDLL(nv.LIB_PATH)
    diag_names = re.findall(r"^NVFP4_API\s+[\w\s\*]*?\b(\w+)\s*\(", open(DIAG_HEADER).read(), re.M)
    assert diag_names
    for name in diag_names:
        assert name not in declared_symbols()
        assert not hasattr(raw, name), f"{name} exported by the product library"


def test_diagnostic_library_exports_its_header_and_the_product_api():
    import nvfp4_diag
    L = nvfp4_diag.lib()
    text = open(DIAG_HEADER).read()
    for name in re.findall(r"^NVFP4_API\s+[\w\s\*]*?\b(\w+)\s*\(", text, re.M) + declared_symbols():
        assert hasattr(L, name), f"{name} not exported by the diagnostic library"


def test_rank_barrier_rejects_bad_arguments_on_host(nv):
    L = nv.lib()
    pads = (C.c_uint64 * 2)(1 << 20, 1 << 21)
    assert L.nvfp4_rank_barrier(None, 2, 0, 0, 4096, None) == -1              # no pads
    assert L.nvfp4_rank_barrier(pads, 9, 0, 0, 4096, None) == -1              # more than 8 ranks
    assert L.nvfp4_rank_barrier(pads, 2, 2, 0, 4096, None) == -1              # rank out of range
    assert L.nvfp4_rank_barrier(pads, 2, 0, 1024, 4096, None) == -1           # channel beyond the pad
    bad = (C.c_uint64 * 2)(1 << 20, (1 << 21) + 2)
    assert L.nvfp4_rank_barrier(bad, 2, 0, 0, 4096, None) == -3               # 4-byte aligned slots


def test_gemm_host_rejects_bad_arguments_on_host(nv):
    """The host-buffer entry point validates before touching a device or a buffer."""
    L = nv.lib()
    p = C.c_void_p(1 << 20)  # never dereferenced: validation runs first
    assert L.nvfp4_gemm_host(None, p, p, p, 1.0, p, 128, 256, 256, None) == -1     # no A
    assert L.nvfp4_gemm_host(p, p, p, p, 1.0, None, 128, 256, 256, None) == -1     # no D
    assert L.nvfp4_gemm_host(p, p, p, p, 1.0, p, 0, 256, 256, None) == -2          # M < 1
    assert L.nvfp4_gemm_host(p, p, p, p, 1.0, p, 128, 12, 256, None) == -2         # N % 8
    assert L.nvfp4_gemm_host(p, p, p, p, 1.0, p, 128, 256, 96, None) == -2         # K % 64
