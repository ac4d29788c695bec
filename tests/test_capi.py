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
