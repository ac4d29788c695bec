"""ctypes binding of libnvfp4_b200.so (the C ABI declared in include/nvfp4_b200.h).

The shared library is built in-tree (gpu-kernels_b200/build.py) and loaded from
this directory.  There is no fallback: if the library is missing or does not
load, every call raises.
"""
import ctypes as C
import os
import threading

# The in-tree build; NVFP4_B200_LIB names another build of the same library (for
# comparing builds side by side).
LIB_PATH = os.environ.get("NVFP4_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                            "libnvfp4_b200.so")

# Every exported symbol, with (restype, argtypes).  Keep in step with the header.
_u8p, _u16p, _f32p, _vp = C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p


class Epilogue(C.Structure):
    """struct nvfp4_epilogue of the header."""
    _fields_ = [("bias", C.c_void_p), ("activation", C.c_int), ("q_out", C.c_void_p), ("sf_out", C.c_void_p),
                ("out_global_scale", C.c_void_p)]


ACTIVATIONS = {"none": 0, "relu": 1, "silu": 2, "gelu_tanh": 3, "swiglu": 4}

SIGNATURES = {
    "nvfp4_status_string": (C.c_char_p, [C.c_int]),
    "nvfp4_version": (C.c_int, []),
    "nvfp4_quantize": (C.c_int, [_u16p, _u8p, _u8p, _f32p, C.c_int, C.c_int, _vp]),
    "nvfp4_global_scale": (C.c_int, [_u16p, C.c_int64, _f32p, _f32p, _vp]),
    "nvfp4_gemm": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int, _vp]),
    "nvfp4_gemm_f16": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int, _vp]),
    "nvfp4_gemm_persistent": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int, _vp]),
    "nvfp4_gemm_epilogue": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int,
                                      C.POINTER(Epilogue), _vp]),
    "nvfp4_gemm_decode_workspace_size": (C.c_size_t, [C.c_int, C.c_int]),
    "nvfp4_gemm_decode": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int, _vp,
                                    C.c_size_t, _vp]),
    "matmul_nvfp4_b200": (None, [_vp, _u8p, _u8p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]),
    "nvfp4_last_status": (C.c_int, []),
    "nvfp4_device_status": (C.c_int, [_vp]),
    "nvfp4_set_wait_timeout_ns": (None, [C.c_uint64]),
    "nvfp4_selftest_wait_timeout": (C.c_int, [C.c_uint64]),
    "nvfp4_launch_count": (C.c_uint64, []),
    "nvfp4_quantize_dynamic": (C.c_int, [_u16p, _u8p, _u8p, _f32p, _f32p, C.c_int, C.c_int, _vp]),
    "nvfp4_gemm_grouped": (C.c_int, [_u8p, _u8p, _u8p, _u8p, _f32p, _u16p, _vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                     _vp]),
    "nvfp4_gemm_grouped_epilogue": (C.c_int, [_u8p, _u8p, _u8p, _u8p, _f32p, _u16p, _vp, C.c_int, C.c_int,
                                              C.c_int, C.c_int, C.POINTER(Epilogue), _vp]),
    "nvfp4_quantize_grouped": (C.c_int, [_u16p, _u8p, _u8p, _f32p, _vp, C.c_int, C.c_int, C.c_int, _vp]),
    "nvfp4_gemm_gather": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, C.c_int, C.c_int, C.c_int,
                                    C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_int64, C.c_int, _vp]),
    "nvfp4_rank_barrier": (C.c_int, [C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_int, C.c_size_t, _vp]),
    "nvfp4_gemm_host": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int, _vp]),
    "nvfp4_gemm_decode_noalloc": (C.c_int, [_u8p, _u8p, _u8p, _u8p, C.c_float, _u16p, C.c_int, C.c_int, C.c_int,
                                            _vp]),
}

STATUS = {
    0: "NVFP4_OK", -1: "NVFP4_ERR_INVALID", -2: "NVFP4_ERR_SHAPE", -3: "NVFP4_ERR_ALIGN",
    -4: "NVFP4_ERR_CUDA", -5: "NVFP4_ERR_TIMEOUT", -6: "NVFP4_ERR_UNSUPPORTED",
    -7: "NVFP4_ERR_WORKSPACE",
}

_lock = threading.Lock()
_lib = None


class NVFP4Error(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        name = STATUS.get(status, str(status))
        msg = ""
        if _lib is not None:
            msg = _lib.nvfp4_status_string(status).decode()
        super().__init__(f"{where}: {name} ({msg})")


def lib():
    """Load (once) and return the library; raises if it is absent."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python gpu-kernels_b200/build.py` "
                        "(there is no CPU fallback)")
                L = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(L, name)
                    f.restype = res
                    f.argtypes = args
                _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != 0:
        raise NVFP4Error(status, where)
