"""numpy front-end of the CPU oracle library — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
leg may import this module; it is the checker, never the thing measured or
shipped.  Every function mirrors one in nvfp4_oracle.c, which restates the
reference's path (matmul/sm100_nvfp4/main.py:9-34).

Arrays: bf16 tensors are passed as numpy uint16 bit patterns; NVFP4 codes as
uint8 [rows, K/2] (element 2i in the low nibble); scales as uint8 e4m3 codes
in the blocked layout, length pad128(rows) * K/16.
"""
import ctypes as C
import os

import numpy as np

from . import build_oracle

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_oracle.OUT
        if not os.path.exists(path):
            path = build_oracle.build()
        L = C.CDLL(path)
        u8p, u16p, f32p = C.POINTER(C.c_uint8), C.POINTER(C.c_uint16), C.POINTER(C.c_float)
        i64 = C.c_int64
        L.nvfp4o_e2m1_decode.restype = C.c_float
        L.nvfp4o_e2m1_decode.argtypes = [C.c_uint8]
        L.nvfp4o_e2m1_encode.restype = C.c_uint8
        L.nvfp4o_e2m1_encode.argtypes = [C.c_float]
        L.nvfp4o_e4m3_decode.restype = C.c_float
        L.nvfp4o_e4m3_decode.argtypes = [C.c_uint8]
        L.nvfp4o_e4m3_encode.restype = C.c_uint8
        L.nvfp4o_e4m3_encode.argtypes = [C.c_float]
        L.nvfp4o_f32_to_bf16.restype = C.c_uint16
        L.nvfp4o_f32_to_bf16.argtypes = [C.c_float]
        L.nvfp4o_sf_offset.restype = C.c_size_t
        L.nvfp4o_sf_offset.argtypes = [i64, i64, i64]
        L.nvfp4o_sf_bytes.restype = C.c_size_t
        L.nvfp4o_sf_bytes.argtypes = [i64, i64]
        L.nvfp4o_sf_pack.argtypes = [u8p, u8p, i64, i64]
        L.nvfp4o_sf_unpack.argtypes = [u8p, u8p, i64, i64]
        L.nvfp4o_quantize.argtypes = [u16p, u8p, u8p, C.c_float, i64, i64, C.c_int]
        L.nvfp4o_amax_bf16.restype = C.c_float
        L.nvfp4o_amax_bf16.argtypes = [u16p, i64, C.c_int]
        L.nvfp4o_dequant.argtypes = [u8p, u8p, f32p, i64, i64, C.c_int]
        L.nvfp4o_gemm_rows.argtypes = [u8p, u8p, u8p, u8p, C.c_float, i64, i64, i64, i64, i64,
                                       f32p, u16p, C.c_int]
        L.nvfp4o_dequant_rows.argtypes = [u8p, u8p, f32p, i64, i64, i64, C.c_int]
        L.nvfp4o_sgemm_nt.argtypes = [f32p, f32p, C.c_float, i64, i64, i64, f32p, u16p, C.c_int]
        L.nvfp4o_fill_normal_bf16.argtypes = [u16p, i64, C.c_uint64, C.c_float, C.c_int]
        L.nvfp4o_fill_student_t3_bf16.argtypes = [u16p, i64, i64, C.c_uint64, C.c_int, C.c_float,
                                                   C.c_int]
        L.nvfp4o_epilogue.argtypes = [f32p, u16p, C.c_int, C.c_float, i64, i64, f32p, u16p, C.c_int]
        L.nvfp4o_epilogue_swiglu.argtypes = [f32p, u16p, C.c_float, i64, i64, f32p, u16p, C.c_int]
        L.nvfp4o_max_threads.restype = C.c_int
        _lib = L
    return _lib


def _p(a, ct):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.POINTER(ct))


def max_threads() -> int:
    return lib().nvfp4o_max_threads()


# ---- codecs ---------------------------------------------------------------
def e2m1_decode(code: int) -> float:
    return lib().nvfp4o_e2m1_decode(code)


def e2m1_encode(x: float) -> int:
    return lib().nvfp4o_e2m1_encode(x)


def e4m3_decode(code: int) -> float:
    return lib().nvfp4o_e4m3_decode(code)


def e4m3_encode(x: float) -> int:
    return lib().nvfp4o_e4m3_encode(x)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """RN-even fp32 -> bf16 bit patterns (vectorised restatement of the C helper)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- layout -------------------------------------------------------------
def sf_offset(r: int, k16: int, K: int) -> int:
    return lib().nvfp4o_sf_offset(r, k16, K)


def sf_bytes(rows: int, K: int) -> int:
    return lib().nvfp4o_sf_bytes(rows, K)


def sf_pack(sf_rowmajor: np.ndarray, rows: int, K: int) -> np.ndarray:
    src = np.ascontiguousarray(sf_rowmajor, dtype=np.uint8).reshape(rows, K // 16)
    out = np.empty(sf_bytes(rows, K), dtype=np.uint8)
    lib().nvfp4o_sf_pack(_p(src, C.c_uint8), _p(out, C.c_uint8), rows, K)
    return out


def sf_unpack(sf_blocked: np.ndarray, rows: int, K: int) -> np.ndarray:
    src = np.ascontiguousarray(sf_blocked, dtype=np.uint8)
    out = np.empty((rows, K // 16), dtype=np.uint8)
    lib().nvfp4o_sf_unpack(_p(src, C.c_uint8), _p(out, C.c_uint8), rows, K)
    return out


# ---- quantizer / dequant / GEMM --------------------------------------------
def quantize(x_bf16: np.ndarray, global_scale: float, nthreads: int = 0):
    """bf16 bits [M,K] -> (Q uint8 [M,K/2], SF uint8 blocked [pad128(M)*K/16])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    q = np.empty((M, K // 2), dtype=np.uint8)
    sf = np.empty(sf_bytes(M, K), dtype=np.uint8)
    lib().nvfp4o_quantize(_p(x, C.c_uint16), _p(q, C.c_uint8), _p(sf, C.c_uint8),
                          float(global_scale), M, K, nthreads)
    return q, sf


def amax_bf16(x_bf16: np.ndarray, nthreads: int = 0) -> float:
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    return lib().nvfp4o_amax_bf16(_p(x, C.c_uint16), x.size, nthreads)


def global_scale_for(amax: float) -> float:
    """gs = amax / (6 * 448) in fp32 (one IEEE division), 0 for an all-zero tensor."""
    return float(np.float32(amax) / np.float32(2688.0))


def dequant(q: np.ndarray, sf: np.ndarray, rows: int, K: int, nthreads: int = 0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    sf = np.ascontiguousarray(sf, dtype=np.uint8)
    out = np.empty((rows, K), dtype=np.float32)
    lib().nvfp4o_dequant(_p(q, C.c_uint8), _p(sf, C.c_uint8), _p(out, C.c_float), rows, K, nthreads)
    return out


def gemm(a, sfa, b, sfb, alpha, M, N, K, m0=0, mrows=None, nthreads=0):
    """Host dequant + fp32 GEMM over A rows [m0, m0+mrows): returns (D32, D_bf16_bits)."""
    mrows = M - m0 if mrows is None else mrows
    arrs = [np.ascontiguousarray(t, dtype=np.uint8) for t in (a, sfa, b, sfb)]
    d32 = np.empty((mrows, N), dtype=np.float32)
    d16 = np.empty((mrows, N), dtype=np.uint16)
    lib().nvfp4o_gemm_rows(*[_p(t, C.c_uint8) for t in arrs], float(alpha), M, N, K, m0, mrows,
                           _p(d32, C.c_float), _p(d16, C.c_uint16), nthreads)
    return d32, d16


def dequant_rows(q, sf, r0: int, nrows: int, K: int, nthreads: int = 0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    sf = np.ascontiguousarray(sf, dtype=np.uint8)
    out = np.empty((nrows, K), dtype=np.float32)
    lib().nvfp4o_dequant_rows(_p(q, C.c_uint8), _p(sf, C.c_uint8), _p(out, C.c_float), r0, nrows, K, nthreads)
    return out


def sgemm_nt(af: np.ndarray, bf: np.ndarray, alpha: float, nthreads: int = 0):
    """fp32 D = alpha * af . bf^T -> (D32, D_bf16_bits)."""
    af = np.ascontiguousarray(af, dtype=np.float32)
    bf = np.ascontiguousarray(bf, dtype=np.float32)
    mrows, K = af.shape
    ncols = bf.shape[0]
    d32 = np.empty((mrows, ncols), dtype=np.float32)
    d16 = np.empty((mrows, ncols), dtype=np.uint16)
    lib().nvfp4o_sgemm_nt(_p(af, C.c_float), _p(bf, C.c_float), float(alpha), mrows, ncols, K,
                          _p(d32, C.c_float), _p(d16, C.c_uint16), nthreads)
    return d32, d16


ACTIVATIONS = {"none": 0, "relu": 1, "silu": 2, "gelu_tanh": 3, "swiglu": 4}


def epilogue(acc: np.ndarray, alpha: float, bias_bf16=None, activation: str = "none", nthreads: int = 0):
    """act(alpha * acc + bias) over a [rows, N] fp32 accumulator -> (Y32, Y_bf16_bits).
    activation "swiglu": gate / up columns interleaved in blocks of 16, output
    [rows, N/2] = silu(gate) * up (nvfp4o_epilogue_swiglu)."""
    acc = np.ascontiguousarray(acc, dtype=np.float32)
    rows, N = acc.shape
    out_n = N // 2 if activation == "swiglu" else N
    y32 = np.empty((rows, out_n), dtype=np.float32)
    y16 = np.empty((rows, out_n), dtype=np.uint16)
    bp = None
    if bias_bf16 is not None:
        bias_bf16 = np.ascontiguousarray(bias_bf16, dtype=np.uint16)
        assert bias_bf16.size == N
        bp = _p(bias_bf16, C.c_uint16)
    if activation == "swiglu":
        assert N % 32 == 0
        lib().nvfp4o_epilogue_swiglu(_p(acc, C.c_float), bp, float(alpha), rows, N, _p(y32, C.c_float),
                                     _p(y16, C.c_uint16), nthreads)
    else:
        lib().nvfp4o_epilogue(_p(acc, C.c_float), bp, ACTIVATIONS[activation], float(alpha), rows, N,
                              _p(y32, C.c_float), _p(y16, C.c_uint16), nthreads)
    return y32, y16


# ---- deterministic inputs ---------------------------------------------------
def normal_bf16(shape, seed: int, std: float = 1.0, nthreads: int = 0) -> np.ndarray:
    out = np.empty(shape, dtype=np.uint16)
    lib().nvfp4o_fill_normal_bf16(_p(out, C.c_uint16), out.size, seed, std, nthreads)
    return out


def student_t3_bf16(rows: int, cols: int, seed: int, n_outlier_cols: int = 0,
                    gain: float = 50.0, nthreads: int = 0) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.uint16)
    lib().nvfp4o_fill_student_t3_bf16(_p(out, C.c_uint16), rows, cols, seed, n_outlier_cols,
                                      gain, nthreads)
    return out


def random_codes(rows: int, K: int, seed: int, sf_lo: int = 0, sf_hi: int = 4):
    """Reference-style operands (matmul/sm100_nvfp4/main.py:9-23): uniformly random
    e2m1 byte codes and e4m3 scale codes in [sf_lo, sf_hi), packed blocked."""
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 256, size=(rows, K // 2), dtype=np.uint16).astype(np.uint8)
    sf_rm = rng.integers(sf_lo, sf_hi, size=(rows, K // 16), dtype=np.uint16).astype(np.uint8)
    return q, sf_pack(sf_rm, rows, K)
