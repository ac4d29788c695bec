"""The reference's file interchange (matmul/sm100_nvfp4/main.py:36-44, runner.cu:14-53,
78-90) and the runner executable built next to the library.

    save_tensors(dir, a, b, sfa, sfb)   a_mat.bin, b_mat.bin, a_scales.bin, b_scales.bin
    load_output(dir, M, N)              c_out_b200.bin -> fp16 [M, N]
    run(M, N, K, "verify"|"benchmark", dir)   nvfp4_runner (the runner's CLI contract)

Byte formats are exactly the reference's: raw int8 views of the e2m1 codes and of
the blocked e4m3 scale codes, fp16 for D.
"""
import os
import subprocess

import numpy as np
import torch

RUNNER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "nvfp4_runner")
FILES = ("a_mat.bin", "b_mat.bin", "a_scales.bin", "b_scales.bin")


def _bytes(t) -> bytes:
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().contiguous().view(torch.int8).numpy().tobytes()
    return np.ascontiguousarray(t).view(np.int8).tobytes()


def save_tensors(directory: str, a, b, sfa, sfb) -> None:
    os.makedirs(directory, exist_ok=True)
    for name, t in zip(FILES, (a, b, sfa, sfb)):
        with open(os.path.join(directory, name), "wb") as f:
            f.write(_bytes(t))


def load_tensors(directory: str, M: int, N: int, K: int):
    """The four input files back as uint8 numpy arrays (shapes as the runner reads them)."""
    sizes = (M * K // 2, N * K // 2, M * K // 16, N * K // 16)
    out = []
    for name, n in zip(FILES, sizes):
        data = np.fromfile(os.path.join(directory, name), dtype=np.uint8)
        if data.size < n:
            raise ValueError(f"{name}: {data.size} bytes, expected at least {n}")
        out.append(data)
    a, b, sfa, sfb = out
    return a.reshape(M, K // 2), b.reshape(N, K // 2), sfa, sfb


def load_output(directory: str, M: int, N: int, name: str = "c_out_b200.bin") -> np.ndarray:
    return np.fromfile(os.path.join(directory, name), dtype=np.float16).reshape(M, N)


def run(M: int, N: int, K: int, mode: str, directory: str = ".", timeout: float = 600) -> subprocess.CompletedProcess:
    if not os.path.exists(RUNNER):
        raise FileNotFoundError(f"{RUNNER} missing: build with gpu-kernels_b200/build.py")
    return subprocess.run([RUNNER, str(M), str(N), str(K), mode, directory], capture_output=True, text=True,
                          timeout=timeout)
