"""Build the CPU oracle library (test infrastructure) in-tree.

    python oracle/build_oracle.py      -> oracle/liboracle_nvfp4.so

Flags: no fast-math and no FMA contraction, so the quantizer's fp32 steps are
single correctly-rounded IEEE operations (the GPU kernel mirrors them with
__f*_rn intrinsics).  The GEMM micro-kernel selects AVX2/FMA at run time.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "nvfp4_oracle.c")
OUT = os.path.join(HERE, "liboracle_nvfp4.so")


def build(force: bool = False) -> str:
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= max(os.path.getmtime(SRC),
                                             os.path.getmtime(os.path.join(HERE, "nvfp4_oracle.h")))):
        return OUT
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp",
           "-ffp-contract=off", "-fno-fast-math", "-Wall", "-Wno-unused-function",
           SRC, "-o", OUT + ".tmp", "-lm"]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
