"""Generate the GEMM golden vectors with the reference's own oracle, torch._scaled_mm
(matmul/sm100_nvfp4/main.py:25-34), on a B200.

    python tests/golden/make_golden.py       (needs an sm_100 GPU; writes tests/golden/*.npz)

Each case stores the NVFP4 operands (e2m1 codes, blocked e4m3 scales, exactly the
formats main.py:9-23 builds) and _scaled_mm's fp32 and fp16 outputs.  The CPU
oracle is checked against these in tests/test_oracle_golden.py; nothing here
is read at run time by the product.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    # name, M, N, K, scale-code range, seed
    ("refstyle_128x128x256", 128, 128, 256, (0, 4), 42),      # main.py's distribution exactly
    ("wide_128x256x512", 128, 256, 512, (0x30, 0x40), 7),     # scales ~0.5..1.9
    ("wide_256x256x1024", 256, 256, 1024, (0x20, 0x48), 11),  # scales 2^-3 .. 3.75
]


def blocked(sf_rm: np.ndarray, rows: int, K: int) -> np.ndarray:
    t = torch.from_numpy(sf_rm.astype(np.uint8).view(np.int8))
    t = t.reshape(rows // 128, 4, 32, K // 64, 4).permute(0, 3, 2, 1, 4)
    return t.contiguous().flatten().numpy().view(np.uint8)


def scaled_mm(a, b, sfa, sfb, out_dtype):
    """torch._scaled_mm as main.py calls it; newer torch spells the block-scaled
    recipe explicitly through torch.nn.functional.scaled_mm."""
    try:
        return torch._scaled_mm(a, b.t(), sfa, sfb, bias=None, out_dtype=out_dtype)
    except Exception as first:  # pragma: no cover - depends on the torch build
        F = torch.nn.functional
        if not hasattr(F, "scaled_mm"):
            raise first
        from torch.nn.functional import ScalingType, SwizzleType
        return F.scaled_mm(a, b.t(), sfa, ScalingType.BlockWise1x16, sfb, ScalingType.BlockWise1x16,
                           swizzle_a=SwizzleType.SWIZZLE_32_4_4, swizzle_b=SwizzleType.SWIZZLE_32_4_4,
                           output_dtype=out_dtype)


def main():
    assert torch.cuda.is_available(), "needs a GPU"
    dev = torch.device("cuda")
    meta = {"torch": torch.__version__, "device": torch.cuda.get_device_name(0), "cases": []}
    for name, M, N, K, (lo, hi), seed in CASES:
        rng = np.random.default_rng(seed)
        a = rng.integers(0, 256, (M, K // 2)).astype(np.uint8)
        b = rng.integers(0, 256, (N, K // 2)).astype(np.uint8)
        sfa_rm = rng.integers(lo, hi, (M, K // 16)).astype(np.uint8)
        sfb_rm = rng.integers(lo, hi, (N, K // 16)).astype(np.uint8)
        sfa, sfb = blocked(sfa_rm, M, K), blocked(sfb_rm, N, K)
        ta = torch.from_numpy(a).to(dev).view(torch.float4_e2m1fn_x2)
        tb = torch.from_numpy(b).to(dev).view(torch.float4_e2m1fn_x2)
        tsa = torch.from_numpy(sfa).to(dev).view(torch.float8_e4m3fn)
        tsb = torch.from_numpy(sfb).to(dev).view(torch.float8_e4m3fn)
        d32 = scaled_mm(ta, tb, tsa, tsb, torch.float32).cpu().numpy()
        d16 = scaled_mm(ta, tb, tsa, tsb, torch.float16).cpu().numpy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), a=a, b=b, sfa=sfa, sfb=sfb, d32=d32, d16=d16,
                            M=M, N=N, K=K)
        meta["cases"].append({"name": name, "M": M, "N": N, "K": K, "scale_codes": [lo, hi], "seed": seed,
                              "d32_absmax": float(np.abs(d32).max())})
        print(name, "absmax", float(np.abs(d32).max()))
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
