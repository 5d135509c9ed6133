"""CPU tests of the oracle itself: fp8 rounding against torch and ml_dtypes,
the quantize recipe's edge cases, and the golden vectors recorded on a B200."""
import os

import numpy as np
import pytest
import torch

import fp8_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "cast_golden.npz")
TORCH_FP8 = {O.E4M3: torch.float8_e4m3fn, O.E5M2: torch.float8_e5m2}


@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2])
def test_rne_matches_torch_on_random_and_ties(fmt):
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * np.float32(s)
                        for s in (1e-5, 1e-3, 0.1, 1, 20, 300, 5e4)])
    t = O.DECODE[fmt]
    fin = np.unique(t[np.isfinite(t)])
    mids = ((fin[:-1] + fin[1:]) / 2).astype(np.float32)
    x = np.concatenate([x, fin.astype(np.float32), mids, np.nextafter(mids, np.float32(np.inf)),
                        np.nextafter(mids, np.float32(-np.inf))])
    m = O.FMAX[fmt]
    y = np.fmin(np.fmax(x, -m), m)
    ours = O.f32_to_fp8_bits(y, fmt)
    ref = torch.from_numpy(y).to(TORCH_FP8[fmt]).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)


def test_rne_matches_ml_dtypes():
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(300_000) * 50).astype(np.float32)
    for fmt, mt in ((O.E4M3, ml.float8_e4m3fn), (O.E5M2, ml.float8_e5m2)):
        y = np.fmin(np.fmax(x, -O.FMAX[fmt]), O.FMAX[fmt])
        assert np.array_equal(O.f32_to_fp8_bits(y, fmt), y.astype(mt).view(np.uint8))


def test_saturation_and_specials():
    x = np.array([1e9, -1e9, np.inf, -np.inf, 449.0, 470.0, 0.0, -0.0], np.float32)
    q = O.f32_to_fp8_bits(x, O.E4M3)
    assert list(q) == [0x7E, 0xFE, 0x7E, 0xFE, 0x7E, 0x7E, 0x00, 0x80]
    q = O.f32_to_fp8_bits(np.array([1e9, 61440.0, 61439.0, -np.inf], np.float32), O.E5M2)
    assert list(q) == [0x7B, 0x7B, 0x7B, 0xFB]


def test_decode_roundtrip():
    for fmt in (O.E4M3, O.E5M2):
        codes = np.arange(256, dtype=np.uint8)
        v = O.fp8_bits_to_f64(codes, fmt)
        ok = np.isfinite(v)
        back = O.f32_to_fp8_bits(v[ok].astype(np.float32), fmt)
        # -0 and +0 are distinct codes; everything finite round-trips exactly
        assert np.array_equal(back, codes[ok])


def test_quantize_recipe_edge_cases():
    # all-zero group: scale 0 -> inv 0 -> zeros
    q, s = O.quantize(np.zeros((2, 256), np.float32), "block1x128", O.E4M3)
    assert np.all(q == 0) and np.all(s == 0)
    # NaN is ignored by amax and becomes +FMAX through the NaN-ignoring clamp
    x = np.ones((1, 128), np.float32)
    x[0, 5] = np.nan
    x[0, 6] = -np.nan
    q, s = O.quantize(x, "block1x128", O.E4M3)
    assert s[0, 0] == np.float32(1.0) / np.float32(448.0)
    assert q[0, 5] == 0x7E and q[0, 6] == 0x7E and q[0, 0] == 0x7E  # scaled: NaN is canonical (+)
    q, _ = O.quantize(x, "none", O.E4M3)
    assert q[0, 5] == 0x7E and q[0, 6] == 0xFE  # unscaled: the NaN's sign bit survives
    # Inf in the group: scale Inf, inv 0, finite -> +-0, Inf*0 = NaN -> +FMAX
    x = np.array([[1.0, -2.0, np.inf, -np.inf] + [0.5] * 124], np.float32)
    q, s = O.quantize(x, "block1x128", O.E5M2)
    assert np.isinf(s[0, 0])
    assert q[0, 0] == 0x00 and q[0, 1] == 0x80 and q[0, 2] == 0x7B and q[0, 3] == 0x7B
    # MX: RCEIL to a power of two, E8M0 byte
    x = np.full((1, 32), 448.0 * 4, np.float32)
    q, s = O.quantize(x, "mx1x32", O.E4M3)
    assert s[0, 0] == 127 + 2 and np.all(q == 0x7E)
    x = np.full((1, 32), 448.0 * 4 * 1.01, np.float32)
    q, s = O.quantize(x, "mx1x32", O.E4M3)
    assert s[0, 0] == 127 + 3


def test_block128x128_matches_per_tile_tensor_mode():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((300, 260)).astype(np.float32)
    q, s = O.quantize(x, "block128x128", O.E4M3)
    assert s.shape == (3, 3)
    for i in range(3):
        for j in range(3):
            tile = x[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128]
            qt, st = O.quantize(tile, "tensor", O.E4M3)
            assert st == s[i, j]
            assert np.array_equal(qt, q[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128])


def test_gemm_oracle_block_matches_tensor_when_uniform():
    rng = np.random.default_rng(0)
    a = O.f32_to_fp8_bits(rng.standard_normal((64, 384)).astype(np.float32), O.E4M3)
    b = O.f32_to_fp8_bits(rng.standard_normal((384, 256)).astype(np.float32), O.E4M3)
    ct = O.gemm(a, b, scale_mode="tensor", scale_a=0.5, scale_b=0.25)
    cb = O.gemm(a, b, scale_mode="block", scale_a=np.full((64, 3), 0.5), scale_b=np.full((3, 2), 0.25))
    assert np.allclose(ct, cb, rtol=1e-12, atol=1e-9)


def test_cast_input_distribution():
    x = O.cast_input(1 << 20, seed=0)
    n = x.size
    assert abs(np.isnan(x).sum() - n * 5e-5) <= 1
    assert abs(np.isinf(x).sum() - n * 5e-5) <= 1
    big = np.abs(x[np.isfinite(x)]) >= 500
    assert abs(big.sum() - int(n * 0.01)) < n * 0.001


# ----------------------------------------------------------------------------
# Golden vectors recorded on a B200 by tests/golden/make_golden_triton.py


def _golden():
    if not os.path.exists(GOLDEN):
        pytest.fail(f"golden vectors missing: {GOLDEN} (run tests/golden/make_golden_triton.py on a GPU)")
    return np.load(GOLDEN)


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2])
@pytest.mark.parametrize("mode", ["none", "mx1x32", "block1x128", "tensor", "tensor_noinf"])
def test_oracle_matches_golden(src, fmt, mode):
    g = _golden()
    noinf = mode == "tensor_noinf"
    if src == "f32":
        x = g["x_f32_noinf" if noinf else "x_f32"]
    else:
        x = O.bf16_bits_to_f32(g["x_bf16_noinf_bits" if noinf else "x_bf16_bits"])
    key = f"{src}_{fmt}_{mode}"
    omode = "tensor" if noinf else mode
    q, s = O.quantize(x, omode, fmt)
    exp_q = g[f"q_{key}"]
    bad = np.nonzero(q != exp_q)
    assert bad[0].size == 0, (
        f"{bad[0].size} mismatches, first at {bad[0][0]},{bad[1][0]}: x={x[bad][0]!r} "
        f"ours=0x{q[bad][0]:02x} golden=0x{exp_q[bad][0]:02x}")
    if mode != "none":
        exp_s = g[f"s_{key}"].reshape(-1)
        assert np.array_equal(np.asarray(s).reshape(-1).view(np.uint8), exp_s.view(np.uint8))


def test_stoch_round_oracle_rules():
    """Representable values never move; r = 0 truncates toward zero; the
    largest r rounds any inexact value up; saturation; unbiasedness."""
    import fp8_oracle as O
    x = np.array([1.0, 1.0625, -1.0625, 1.2, 500.0, -np.inf, 0.0], np.float32)
    assert list(O.stoch_round(x, np.zeros(7, np.uint32), "e4m3")) == [0x38, 0x38, 0xB8, 0x39, 0x7E, 0xFE, 0x00]
    assert list(O.stoch_round(x, np.full(7, 0xFFFFFFFF, np.uint32), "e4m3")) == [0x38, 0x39, 0xB9, 0x3A, 0x7E, 0xFE,
                                                                                  0x00]
    rng = np.random.default_rng(0)
    n = 100000
    v = np.full(n, 1.0001, np.float32)
    r = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    h = O.stoch_round(v, r, "f16").view(np.float16).astype(np.float64)
    assert abs(h.mean() - np.float64(np.float32(1.0001))) < 6 * 2 ** -10 / np.sqrt(n)
    b = O.stoch_round(np.array([3.0e38, 5e-41], np.float32), np.array([0xFFFFFFFF, 0], np.uint32), "bf16")
    assert b[0] == 0x7F62 and b[1] == 0x0000  # next bf16 up from 3.0e38; 5e-41 < 2^-133 truncates to 0 at r = 0


def test_mx_gemm_oracle_matches_reference_formula():
    """The MX GEMM oracle equals the formula of the reference's
    test_async_dot_scaled (test_tlx.py:2298-2444): each operand's 32-wide K
    slices multiplied by 2^(scale - 127), then one matmul (float64 here)."""
    import torch
    import fp8_oracle as O
    rng = np.random.default_rng(5)
    M, N, K = 16, 24, 128
    qa, sa = O.quantize(rng.standard_normal((M, K), dtype=np.float32) * 30, "mx1x32", O.E4M3)
    qb, sb = O.quantize(rng.standard_normal((N, K), dtype=np.float32) / 7, "mx1x32", O.E5M2)
    a = torch.from_numpy(O.fp8_bits_to_f64(qa, O.E4M3))
    b = torch.from_numpy(O.fp8_bits_to_f64(qb, O.E5M2))
    fa = torch.pow(2.0, torch.from_numpy(sa.astype(np.float64) - 127)).repeat_interleave(32, dim=1)
    fb = torch.pow(2.0, torch.from_numpy(sb.astype(np.float64) - 127)).repeat_interleave(32, dim=1)
    want = ((a * fa) @ (b * fb).T).numpy()
    got = O.gemm(qa, qb.T, O.E4M3, O.E5M2, "mx", sa, sb)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "f16", "bf16"])
def test_stoch_round_c_and_numpy_oracles_agree(fmt):
    """Two restatements of the stochastic-rounding rule -- integer (numpy) and
    floating-point (C) -- agree bit for bit, specials included."""
    import fp8_oracle as O
    import oracle_c as OC
    rng = np.random.default_rng(11)
    n = 200000
    x = rng.standard_normal(n).astype(np.float32) * np.exp2(rng.integers(-140, 120, n)).astype(np.float32)
    x[:16] = [0.0, -0.0, np.inf, -np.inf, np.nan, 448.0, 464.0, 57344.0, 65504.0, 65520.0, 3.0e38, 1e-45,
              -1e-40, 2.0 ** -126, 1.0625, -1.0625]
    r = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    r[:4] = [0, 0xFFFFFFFF, 0x80000000, 1]
    a = O.stoch_round(x, r, fmt)
    b = OC.stoch_round(x, r, fmt)
    bad = np.nonzero(a != b)[0]
    assert bad.size == 0, (fmt, bad[:5], x[bad[:5]], r[bad[:5]], a[bad[:5]], b[bad[:5]])
