"""CPU: pin the oracle's dequant + fp32 GEMM against the reference's oracle.

tests/golden/*.npz hold NVFP4 operands and torch._scaled_mm outputs
(matmul/sm100_nvfp4/main.py:25-34) computed on a B200 by
tests/golden/make_golden.py.  The oracle must reproduce them: this fixes the
operand semantics the GPU kernel is then checked against (nibble order, e4m3
scale decoding, blocked scale layout, D = A . B^T).
"""
import glob
import os

import numpy as np
import pytest

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def test_golden_vectors_present():
    assert len(GOLDEN) >= 3, "golden vectors missing: run tests/golden/make_golden.py on a B200"


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_matches_scaled_mm(oracle, path):
    z = np.load(path)
    M, N, K = int(z["M"]), int(z["N"]), int(z["K"])
    d32, d16 = oracle.gemm(z["a"], z["sfa"], z["b"], z["sfb"], 1.0, M, N, K)
    ref = z["d32"]
    scale = np.abs(ref).max()
    assert scale > 0
    # fp32 sums in a different order: agreement to a few fp32 ulps of the row scale
    assert np.abs(d32 - ref).max() <= 1e-5 * scale
    # fp16 output as main.py checks it: allclose(atol=rtol=1e-3) against _scaled_mm's fp16
    ours16 = d32.astype(np.float16).astype(np.float32)
    assert np.allclose(ours16, z["d16"].astype(np.float32), atol=1e-3, rtol=1e-3)
