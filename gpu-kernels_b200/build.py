"""Build libnvfp4_b200.so (the product), libnvfp4_diag.so (its diagnostic twin) and
the runner executable in-tree for sm_100a.

    python gpu-kernels_b200/build.py [--force] [-v]

nvcc cross-compiles without a GPU.  Each translation unit compiles to an object
under gpu-kernels_b200/_build/ in parallel (the decode kernel's instantiations are
one unit per padded row count), then the libraries are linked.  The library links
the CUDA runtime statically and resolves cuTensorMapEncodeTiled through the
runtime's driver entry-point query, so it loads on machines without a CUDA driver
(and fails with NVFP4_ERR_CUDA / NVFP4_ERR_UNSUPPORTED there instead of at load time).

The diagnostic library is the product's objects with the CTA-pair kernel rebuilt
with NVFP4_DIAG (its cycle-trace variant) plus the diagnostic sources
(nvfp4_diag/csrc); the product library contains none of them.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
DIAG_CSRC = os.path.join(HERE, "nvfp4_diag", "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "nvfp4_b200", "libnvfp4_b200.so")
DIAG_OUT = os.path.join(HERE, "nvfp4_diag", "libnvfp4_diag.so")
RUNNER = os.path.join(HERE, "nvfp4_b200", "nvfp4_runner")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                 "-I", INCLUDE, "-I", CSRC]
DECODE_MPADS = (8, 16, 32, 64, 128)

# (object name, source, extra flags)
PRODUCT_UNITS = [("runtime", os.path.join(CSRC, "runtime.cu"), []),
                 ("quantize", os.path.join(CSRC, "quantize.cu"), []),
                 ("gemm", os.path.join(CSRC, "gemm.cu"), []),
                 ("gemm_pair", os.path.join(CSRC, "gemm_pair.cu"), []),
                 ("gemm_decode", os.path.join(CSRC, "gemm_decode.cu"), []),
                 ("host_pipeline", os.path.join(CSRC, "host_pipeline.cu"), []),
                 ("capi", os.path.join(CSRC, "capi.cu"), [])]
PRODUCT_UNITS += [(f"decode_inst_{m}", os.path.join(CSRC, "decode_inst.cu"), [f"-DNVFP4_DECODE_MPAD={m}"])
                  for m in DECODE_MPADS]
DIAG_UNITS = [("gemm_pair_diag", os.path.join(CSRC, "gemm_pair.cu"), ["-DNVFP4_DIAG"]),
              ("probe", os.path.join(DIAG_CSRC, "probe.cu"), []),
              ("diag_capi", os.path.join(DIAG_CSRC, "diag_capi.cu"), [])]


def _headers():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    files += [os.path.join(INCLUDE, "nvfp4_b200.h"), os.path.join(HERE, "nvfp4_diag", "nvfp4_diag.h"),
              os.path.abspath(__file__)]
    return files


def _inputs():
    return _headers() + [src for _, src, _ in PRODUCT_UNITS + DIAG_UNITS] + [os.path.join(CSRC, "runner_main.cu")]


def _obj(name):
    return os.path.join(OBJ, name + ".o")


def _compile(unit, force, headers_mtime, verbose):
    name, src, extra = unit
    out = _obj(name)
    if not force and os.path.exists(out) and os.path.getmtime(out) >= max(headers_mtime, os.path.getmtime(src)):
        return out
    cmd = [NVCC, *CFLAGS, *extra, "-c", src, "-o", out + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(out + ".tmp", out)
    return out


def _link(out, objs):
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", out + ".tmp", *objs]
    subprocess.check_call(cmd)
    os.replace(out + ".tmp", out)


def build(force: bool = False, verbose: bool = False, jobs: int = 0) -> str:
    """Build both libraries and the runner executable (which links the product library
    from its own directory); returns the product library's path."""
    outs = (OUT, DIAG_OUT, RUNNER)
    if not force and all(os.path.exists(p) for p in outs):
        if min(os.path.getmtime(p) for p in outs) >= max(os.path.getmtime(f) for f in _inputs()):
            return OUT
    os.makedirs(OBJ, exist_ok=True)
    hm = max(os.path.getmtime(f) for f in _headers())
    units = PRODUCT_UNITS + DIAG_UNITS
    # longest units first: the decode instantiations and the CTA-pair kernel dominate
    order = sorted(units, key=lambda u: (not u[0].startswith(("decode_inst", "gemm_pair")), u[0]))
    with ThreadPoolExecutor(max_workers=jobs or max(1, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda u: _compile(u, force, hm, verbose), order))
    product = [_obj(n) for n, _, _ in PRODUCT_UNITS]
    _link(OUT, product)
    _link(DIAG_OUT, [o for o in product if not o.endswith("/gemm_pair.o")] + [_obj(n) for n, _, _ in DIAG_UNITS])
    lib_dir = os.path.dirname(OUT)
    runner = [NVCC, *ARCH, "-O2", "-std=c++17", "-cudart", "static", "-I", INCLUDE, "-o", RUNNER + ".tmp",
              os.path.join(CSRC, "runner_main.cu"), "-L" + lib_dir, "-lnvfp4_b200", "-Xlinker", "-rpath=$ORIGIN"]
    subprocess.check_call(runner)
    os.replace(RUNNER + ".tmp", RUNNER)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
