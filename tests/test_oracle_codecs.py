"""CPU: the oracle's codecs, scale layout and quantizer specification.

Pins: e4m3 against torch's float8_e4m3fn (exhaustive decode, randomized encode);
e2m1 against the format's value table and hand-derived round-to-nearest-even
ties; the blocked scale layout against the reference's own reshape/permute
(matmul/sm100_nvfp4/main.py:16-22); the quantizer against known answers and a
second, pure-Python statement of the same specification.
"""
import math

import numpy as np
import pytest
import torch

E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def test_e2m1_decode_table(oracle):
    for c in range(16):
        v = oracle.e2m1_decode(c)
        mag = E2M1[c & 7]
        assert v == (-mag if c & 8 else mag)
        assert math.copysign(1.0, v) == (-1.0 if c & 8 else 1.0)


@pytest.mark.parametrize("x,code", [
    (0.0, 0), (0.24, 0), (0.25, 0), (0.26, 1), (0.5, 1), (0.74, 1), (0.75, 2), (1.0, 2), (1.25, 2),
    (1.26, 3), (1.5, 3), (1.75, 4), (2.0, 4), (2.5, 4), (2.6, 5), (3.0, 5), (3.5, 6), (4.0, 6),
    (5.0, 6), (5.01, 7), (6.0, 7), (7.0, 7), (1e30, 7), (float("inf"), 7),
    (-0.0, 8), (-0.1, 8), (-0.75, 10), (-5.0, 14), (-6.5, 15), (float("-inf"), 15),
])
def test_e2m1_encode_kat(oracle, x, code):
    assert oracle.e2m1_encode(x) == code


def test_e2m1_encode_is_nearest(oracle):
    xs = np.linspace(-8, 8, 20001, dtype=np.float32)
    for x in xs:
        c = oracle.e2m1_encode(float(x))
        v = oracle.e2m1_decode(c)
        if abs(x) >= 6:
            assert v == math.copysign(6.0, x)
            continue
        best = min(abs(abs(x) - m) for m in E2M1)
        assert abs(abs(x) - abs(v)) == pytest.approx(best, abs=1e-7)


def test_e4m3_decode_exhaustive_vs_torch(oracle):
    codes = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    got = np.array([oracle.e4m3_decode(int(c)) for c in codes], dtype=np.float32)
    assert np.array_equal(np.isnan(ref), np.isnan(got))
    ok = ~np.isnan(ref)
    assert np.array_equal(ref[ok].view(np.uint32), got[ok].view(np.uint32))


def test_e4m3_encode_vs_torch(oracle):
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(50000).astype(np.float32) * 40,
        (2.0 ** rng.uniform(-12, 8.9, 50000)).astype(np.float32),
        np.float32(2.0) ** np.arange(-12, 9, 0.125, dtype=np.float32),
        np.array([0.0, -0.0, 447.9, 448.0, -448.0, 2.0 ** -10, 2.0 ** -9 * 1.5, 2.0 ** -9 * 2.5], np.float32),
    ])
    # torch's CPU cast gives NaN above 448 (no saturation), so compare inside the range
    x = np.clip(x, -448.0, 448.0)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([oracle.e4m3_encode(float(v)) for v in x], dtype=np.uint8)
    assert np.array_equal(ref, got)


@pytest.mark.parametrize("x,code", [(448.0, 0x7E), (1e9, 0x7E), (-1e9, 0xFE), (float("inf"), 0x7E),
                                    (float("nan"), 0x7F), (464.0, 0x7E)])
def test_e4m3_encode_saturates(oracle, x, code):
    assert oracle.e4m3_encode(x) == code


def test_bf16_roundtrip(oracle):
    x = np.random.default_rng(2).standard_normal(10000).astype(np.float32)
    ours = oracle.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)
    back = oracle.bf16_bits_to_f32(ours)
    assert np.array_equal(back, torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def _reference_permute(sf_rowmajor: np.ndarray, rows: int, K: int) -> np.ndarray:
    """matmul/sm100_nvfp4/main.py:16-22, restated with torch on the CPU."""
    t = torch.from_numpy(sf_rowmajor.astype(np.int8).reshape(rows, K // 16))
    t = t.reshape(rows // 128, 4, 32, K // 64, 4).permute(0, 3, 2, 1, 4)
    return t.contiguous().flatten().numpy().view(np.uint8)


@pytest.mark.parametrize("rows,K", [(128, 64), (256, 256), (384, 1024)])
def test_sf_layout_matches_reference_permute(oracle, rows, K):
    sf = np.random.default_rng(rows + K).integers(0, 256, (rows, K // 16)).astype(np.uint8)
    ref = _reference_permute(sf, rows, K)
    assert np.array_equal(oracle.sf_pack(sf, rows, K), ref)
    assert np.array_equal(oracle.sf_unpack(ref, rows, K), sf)
    import nvfp4_b200.layout as lay
    blocked = lay.to_blocked(torch.from_numpy(sf))
    assert np.array_equal(blocked.numpy(), ref)
    assert np.array_equal(lay.from_blocked(blocked, rows, K).numpy(), sf)
    for r, k in [(0, 0), (rows - 1, K // 16 - 1), (37, 3)]:
        off = oracle.sf_offset(r, k, K)
        assert off == lay.sf_offset(r, k, K)
        assert ref[off] == sf[r, k]


def test_sf_layout_pads_ragged_rows(oracle):
    rows, K = 200, 128
    sf = np.random.default_rng(3).integers(1, 256, (rows, K // 16)).astype(np.uint8)
    packed = oracle.sf_pack(sf, rows, K)
    assert packed.size == 256 * K // 16
    padded = np.zeros((256, K // 16), np.uint8)
    padded[:rows] = sf
    assert np.array_equal(packed, _reference_permute(padded, 256, K))


# ---- quantizer -------------------------------------------------------------
def py_quantize_block(xs, gs):
    """Pure-Python statement of the quantizer specification (small cases only)."""
    f = np.float32
    v = [f(x) for x in xs]
    amax = f(0)
    for x in v:
        if abs(x) > amax:
            amax = f(abs(x))
    gs = f(gs)
    code, inv = 0, f(0)
    if f(2.0 ** -100) <= gs <= f(np.finfo(np.float32).max):
        sfv = f(f(amax / f(6)) / gs)
        code = int(torch.tensor([min(float(sfv), 448.0)]).to(torch.float8_e4m3fn).view(torch.uint8))
        s = float(torch.tensor([code], dtype=torch.uint8).view(torch.float8_e4m3fn).float())
        denom = f(f(s) * gs)
        inv = f(0) if denom == 0 else f(f(1) / denom)
    qs = []
    for x in v:
        y = f(x * inv)
        sign = 8 if math.copysign(1.0, float(y)) < 0 else 0
        a = abs(float(y))
        mags = E2M1
        if a >= 6:
            c = 7
        else:
            best = min(range(8), key=lambda i: (abs(a - mags[i]), i % 2))
            c = best
        qs.append(sign | c)
    return code, qs


def _bf16(vals):
    return np.array([np.float32(v) for v in vals], np.float32)


def _run_block(oracle, vals, gs):
    x = oracle.f32_to_bf16_bits(_bf16(vals)).reshape(1, 16)
    x = np.concatenate([x, np.zeros((1, 48), np.uint16)], 1)  # K = 64
    q, sf = oracle.quantize(x, gs)
    codes = []
    for byte in q[0, :8]:
        codes += [int(byte) & 15, int(byte) >> 4]
    return int(sf[oracle.sf_offset(0, 0, 64)]), codes


KATS = [
    # (block values, gs, expected scale code, expected e2m1 codes)
    ([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -5.0, -6.0, 0.0, 0.5, 1.0, -0.1], 1.0,
     0x38, [0, 2, 2, 4, 4, 6, 6, 7, 8, 10, 14, 15, 0, 1, 2, 8]),
    ([0.0] * 16, 1.0, 0x00, [0] * 16),
    ([6.0, 1.0] + [0.0] * 14, 2.0 ** -10, 0x7E, [7, 4] + [0] * 14),          # scale saturates at 448
    ([0.01, -0.004] + [0.0] * 14, 1.0, 0x01, [7, 12] + [0] * 14),            # subnormal scale 2^-9
    ([1.0, -2.0] + [0.0] * 14, 0.0, 0x00, [0, 8] + [0] * 14),               # unusable gs -> zeros
    ([1.0, -2.0] + [0.0] * 14, float("nan"), 0x00, [0, 8] + [0] * 14),
    ([3.0] * 16, 0.5, 0x38, [7] * 16),                                        # (3/6)/0.5 = 1.0
]


@pytest.mark.parametrize("vals,gs,sf_code,codes", KATS)
def test_quantize_kat(oracle, vals, gs, sf_code, codes):
    got_sf, got_q = _run_block(oracle, vals, gs)
    assert got_sf == sf_code
    assert got_q == codes
    ref_sf, ref_q = py_quantize_block(oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(_bf16(vals))), gs)
    assert (ref_sf, ref_q) == (sf_code, codes)


def test_quantize_matches_python_statement(oracle):
    rng = np.random.default_rng(7)
    for trial in range(40):
        scale = 10.0 ** rng.uniform(-3, 3)
        vals = rng.standard_t(3, 16) * scale
        gs = float(np.float32(np.abs(vals).max() * rng.uniform(0.5, 3) / 2688.0))
        xb = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(vals.astype(np.float32)))
        got = _run_block(oracle, xb, gs)
        assert got == py_quantize_block(xb, gs)


def test_quantize_shapes_and_padding(oracle):
    M, K = 130, 192
    x = oracle.normal_bf16((M, K), seed=5)
    gs = oracle.global_scale_for(oracle.amax_bf16(x))
    q, sf = oracle.quantize(x, gs)
    assert q.shape == (M, K // 2) and sf.size == 256 * K // 16
    un = oracle.sf_unpack(sf, 256, K)
    assert np.all(un[M:] == 0)
    deq = oracle.dequant(q, sf, M, K)
    xf = oracle.bf16_bits_to_f32(x).reshape(M, K)
    err = np.abs(deq * gs - xf).max() / np.abs(xf).max()
    assert err < 0.2  # 4-bit mantissa-free codes: coarse, but bounded


def test_generators_deterministic(oracle):
    a = oracle.normal_bf16((64, 64), seed=11)
    b = oracle.normal_bf16((64, 64), seed=11)
    c = oracle.normal_bf16((64, 64), seed=12)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    xf = oracle.bf16_bits_to_f32(oracle.normal_bf16((512, 512), seed=3))
    assert abs(xf.mean()) < 0.02 and abs(xf.std() - 1) < 0.02
    t = oracle.bf16_bits_to_f32(oracle.student_t3_bf16(256, 1024, seed=4, n_outlier_cols=4, gain=50.0))
    col_max = np.abs(t.reshape(256, 1024)).max(0)
    assert (col_max > 200).sum() >= 3  # the four x50 outlier channels dominate
