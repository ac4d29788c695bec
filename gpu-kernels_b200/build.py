"""Build libnvfp4_b200.so in-tree for sm_100a.

    python gpu-kernels_b200/build.py [--force]

nvcc cross-compiles without a GPU.  The library links the CUDA runtime
statically and resolves cuTensorMapEncodeTiled through the runtime's driver
entry-point query, so it loads on machines without a CUDA driver (and fails
with NVFP4_ERR_CUDA / NVFP4_ERR_UNSUPPORTED there instead of at load time).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "nvfp4_b200", "libnvfp4_b200.so")
RUNNER = os.path.join(HERE, "nvfp4_b200", "nvfp4_runner")
SOURCES = ["runtime.cu", "quantize.cu", "gemm.cu", "gemm_pair.cu", "gemm_decode.cu", "probe.cu", "host_pipeline.cu",
           "capi.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared", "-cudart", "static"]


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh"))]
    files.append(os.path.join(INCLUDE, "nvfp4_b200.h"))
    files.append(os.path.abspath(__file__))
    return files


def build(force: bool = False, verbose: bool = False) -> str:
    """Build the library and the runner executable (which links it from its own
    directory); returns the library path."""
    if not force and os.path.exists(OUT) and os.path.exists(RUNNER):
        newest = max(os.path.getmtime(f) for f in _inputs())
        if min(os.path.getmtime(OUT), os.path.getmtime(RUNNER)) >= newest:
            return OUT
    cmd = [NVCC, *FLAGS, "-I", INCLUDE, "-o", OUT + ".tmp", *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    lib_dir = os.path.dirname(OUT)
    runner = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-cudart", "static", "-I", INCLUDE, "-o", RUNNER + ".tmp",
              os.path.join(CSRC, "runner_main.cu"), "-L" + lib_dir, "-lnvfp4_b200", "-Xlinker", "-rpath=$ORIGIN"]
    subprocess.check_call(runner)
    os.replace(RUNNER + ".tmp", RUNNER)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
