"""ctypes binding of libnvfp4_diag.so — the diagnostic build of the NVFP4 library
(nvfp4_diag.h): every product entry point plus the traced GEMM launches, the
tensor-rate probe and the scale-code check of the fused epilogue's tables.

It is a separate library so that the product (nvfp4_b200, libnvfp4_b200.so) holds
none of this.  The command line (`python -m nvfp4_diag ...`, gpu-kernels_b200/ on
sys.path) measures the kernels; tests use `lib()` for the scale-code check.
"""
import ctypes as C
import os
import threading

from nvfp4_b200._lib import SIGNATURES, Epilogue, NVFP4Error

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnvfp4_diag.so")

_vp = C.c_void_p
DIAG_SIGNATURES = {
    "nvfp4_gemm_trace": (C.c_int, [_vp, _vp, _vp, _vp, C.c_float, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp]),
    "nvfp4_gemm_trace_epilogue": (C.c_int, [_vp, _vp, _vp, _vp, C.c_float, _vp, C.c_int, C.c_int, C.c_int,
                                            C.POINTER(Epilogue), _vp, _vp]),
    "nvfp4_gemm_decode_trace": (C.c_int, [_vp, _vp, _vp, _vp, C.c_float, _vp, C.c_int, C.c_int, C.c_int, _vp,
                                          C.c_size_t, _vp, _vp]),
    "nvfp4_probe_mma_rate": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "nvfp4_scale_codes": (C.c_int, [_vp, C.c_int64, _vp, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


def lib():
    """Load (once) and return the diagnostic library; raises if it is absent."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing: build it with `python gpu-kernels_b200/build.py`")
                L = C.CDLL(LIB_PATH)
                for name, (res, args) in {**SIGNATURES, **DIAG_SIGNATURES}.items():
                    f = getattr(L, name)
                    f.restype = res
                    f.argtypes = args
                _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != 0:
        raise NVFP4Error(status, where)
