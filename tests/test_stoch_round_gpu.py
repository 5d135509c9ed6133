"""GPU checks of the stochastic-rounding cast in both roundings.

rounding="exact32" (C ABI b2x_stoch_round): bit-exact against the integer CPU
oracle (fp8_oracle.stoch_round) for every element, including signed zeros,
subnormals, values beyond the target range, +-Inf and NaN.
rounding="rs" (b2x_stoch_round_rs, the hardware cvt.rs.satfinite that the
reference lowers to): the properties the reference's tests check
(test_stoch_round, test_stoch_round_partial_pack, test_stoch_round_entropy_quality;
extensions/utlx/test/test_tlx.py:5126-5368), plus: each result is one of the
two neighbours of the input, the rounding-up frequency follows the input's
position between them, and a pack reads only its first element's word.
Both: unbiasedness."""
import zlib

import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu

TARGETS = [(torch.float8_e4m3fn, "e4m3"), (torch.float8_e5m2, "e5m2"), (torch.float16, "f16"),
           (torch.bfloat16, "bf16")]


def _bits(t):
    return t.view(torch.uint8 if t.element_size() == 1 else torch.int16).cpu().numpy().view(
        np.uint8 if t.element_size() == 1 else np.uint16)


def _inputs(shape, seed):
    rng = np.random.default_rng(seed)
    n = int(np.prod(shape))
    x = rng.standard_normal(n).astype(np.float32) * np.exp2(rng.integers(-40, 40, n)).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0, 448.0, 449.0, 464.0, 57344.0, 60000.0,
                        65504.0, 65520.0, 3.0e38, -3.4e38, 1e-45, -1e-45, 2.0 ** -9, 2.0 ** -10, 2.0 ** -126,
                        1.0 + 2.0 ** -23, 1.0625, -1.0625], np.float32)
    k = min(n, special.size)
    x[:k] = special[:k]
    r = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    r[:4] = [0, 0xFFFFFFFF, 0x80000000, 0x7FFFFFFF][:min(4, n)]
    return x.reshape(shape), r.reshape(shape)


@pytest.mark.parametrize("dtype,fmt", TARGETS)
@pytest.mark.parametrize("shape", [(256, 1024), (1000, 37), (4099,), (3, 8)])
def test_stoch_round_bit_exact(dtype, fmt, shape):
    import b2x
    x, r = _inputs(shape, seed=zlib.crc32(repr((fmt, shape)).encode()) & 0xFFFF)
    before = b2x.launch_count()
    y = b2x.stoch_round(torch.from_numpy(x).cuda(), dtype, torch.from_numpy(r.view(np.int32)).cuda(),
                        rounding="exact32")
    torch.cuda.synchronize()
    assert b2x.launch_count() > before, "no libb2x kernel ran"
    got = _bits(y).reshape(-1)
    want = O.stoch_round(x.reshape(-1), r.reshape(-1), fmt)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (f"{fmt} {shape}: {bad.size} mismatches, first at {bad[:5]}: x={x.reshape(-1)[bad[:5]]} "
                           f"r={r.reshape(-1)[bad[:5]]} got={got[bad[:5]]} want={want[bad[:5]]}")


def test_stoch_round_strided_rows():
    import b2x
    x, r = _inputs((64, 160), seed=9)
    xt = torch.from_numpy(x).cuda()[:, 16:144]
    rt = torch.from_numpy(r.view(np.int32)).cuda()[:, 16:144]
    y = b2x.stoch_round(xt, torch.float8_e4m3fn, rt, rounding="exact32")
    want = O.stoch_round(x[:, 16:144].reshape(-1), r[:, 16:144].reshape(-1), "e4m3")
    assert np.array_equal(_bits(y).reshape(-1), want)


@pytest.mark.parametrize("rounding", ["rs", "exact32"])
@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_stoch_round_reference_properties(dtype, fmt, rounding):
    """The checks of the reference's test_stoch_round on 256 randn values."""
    import b2x
    torch.manual_seed(0)
    a = torch.randn(256, dtype=torch.float32, device="cuda")
    rbits = torch.randint(0, 2 ** 31 - 1, (256,), device="cuda", dtype=torch.int32) * 2 + 1
    b = b2x.stoch_round(a, dtype, rbits, rounding=rounding)
    bf = b.float()
    assert not torch.isnan(bf).any() and not torch.isinf(bf).any()
    exact = bf == a
    assert torch.equal(b[exact].float(), a[exact].to(dtype).float())
    lo = a.to(dtype).float()
    # each result is one of the two neighbours of a
    assert (torch.abs(bf - a) <= torch.abs(lo - a) * 2 + 1e-30 + torch.abs(a) * 0.25).all()


@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_stoch_round_is_unbiased(dtype, fmt):
    """exact32: the mean of SR(x) over random words equals x to sampling
    precision."""
    import b2x
    n = 1 << 22
    vals = {"e4m3": 1.03, "e5m2": 1.1, "f16": 1.0001, "bf16": 1.001}
    x = torch.full((n,), vals[fmt], dtype=torch.float32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    r = torch.randint(-2 ** 31, 2 ** 31 - 1, (n,), device="cuda", dtype=torch.int32, generator=g)
    mean = b2x.stoch_round(x, dtype, r, rounding="exact32").double().mean().item()
    lo = torch.tensor(vals[fmt]).to(dtype).double().item()
    ulp = abs(torch.tensor(vals[fmt] * 1.5).to(dtype).double().item() - lo) or 1.0
    assert abs(mean - float(np.float32(vals[fmt]))) < 6 * ulp / np.sqrt(n) + 1e-9, mean


def test_stoch_round_rejects_bad_input():
    import b2x
    x = torch.zeros(8, device="cuda")
    with pytest.raises(ValueError):
        b2x.stoch_round(x, torch.bfloat16, torch.zeros(4, dtype=torch.int32, device="cuda"))
    with pytest.raises(TypeError):
        b2x.stoch_round(x.half(), torch.bfloat16, torch.zeros(8, dtype=torch.int32, device="cuda"))
    assert b2x.stoch_round(x, torch.float32, torch.zeros(8, dtype=torch.int32, device="cuda")) is x


def _neighbours(a, dtype):
    """(lower, upper) representable neighbours of float32 values a (finite,
    inside the target range): round toward zero, and one quantum further."""
    fmt = {torch.float8_e4m3fn: "e4m3", torch.float8_e5m2: "e5m2", torch.float16: "f16", torch.bfloat16: "bf16"}[dtype]
    x = a.cpu().numpy()
    lo = O.stoch_round_value(x, np.zeros(x.shape, np.uint32), fmt)
    hi = O.stoch_round_value(x, np.full(x.shape, 0xFFFFFFFF, np.uint32), fmt)
    return lo, hi


@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_rs_results_are_neighbours(dtype, fmt):
    """rs on 1M values of mixed magnitude: every result is the truncation of
    x or the next value away from zero, and representable values stay."""
    import b2x
    g = torch.Generator(device="cuda").manual_seed(7)
    n = 1 << 20
    fmax = {"e4m3": 440.0, "e5m2": 57000.0, "f16": 65000.0, "bf16": 3e38}[fmt]
    a = torch.randn(n, device="cuda", generator=g) * torch.exp2(torch.randint(-12, 8, (n,), device="cuda",
                                                                               generator=g).float())
    a = a.clamp(-fmax, fmax)
    a[:64] = a[:64].to(dtype).float()  # exactly representable
    r = torch.randint(-2 ** 31, 2 ** 31 - 1, (n,), device="cuda", dtype=torch.int32, generator=g)
    y = b2x.stoch_round(a, dtype, r, rounding="rs").float().cpu().numpy()
    lo, hi = _neighbours(a, dtype)
    ok = (y == lo) | (y == hi)
    assert ok.all(), f"{(~ok).sum()} results are not neighbours; first x={a.cpu().numpy()[~ok][:4]} y={y[~ok][:4]}"
    assert np.array_equal(y[:64], a[:64].cpu().numpy())


@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_rs_round_up_frequency(dtype, fmt):
    """P(round up) follows the position f of x between its neighbours."""
    import b2x
    n = 1 << 18
    base = torch.tensor(1.0)
    q = {"e4m3": 2.0 ** -3, "e5m2": 2.0 ** -2, "f16": 2.0 ** -10, "bf16": 2.0 ** -7}[fmt]
    g = torch.Generator(device="cuda").manual_seed(11)
    for f in (0.125, 0.25, 0.5, 0.75, 0.875):
        x = torch.full((n,), float(base + f * q), device="cuda")
        r = torch.randint(-2 ** 31, 2 ** 31 - 1, (n,), device="cuda", dtype=torch.int32, generator=g)
        up = (b2x.stoch_round(x, dtype, r, rounding="rs").float() > 1.0).double().mean().item()
        assert abs(up - f) < 0.02, f"{fmt}: x = 1 + {f} quantum rounds up with frequency {up}"


@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_rs_pack_reads_first_word(dtype, fmt):
    """Changing the words of a pack's other elements changes nothing."""
    import b2x
    P = 4 if fmt in ("e4m3", "e5m2") else 2
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn((64, 256), device="cuda", generator=g)
    r1 = torch.randint(-2 ** 31, 2 ** 31 - 1, (64, 256), device="cuda", dtype=torch.int32, generator=g)
    r2 = torch.randint(-2 ** 31, 2 ** 31 - 1, (64, 256), device="cuda", dtype=torch.int32, generator=g)
    r2[:, ::P] = r1[:, ::P]
    y1 = b2x.stoch_round(a, dtype, r1, rounding="rs")
    y2 = b2x.stoch_round(a, dtype, r2, rounding="rs")
    assert torch.equal(y1.view(torch.uint8), y2.view(torch.uint8))


@pytest.mark.parametrize("dtype,fmt", TARGETS)
@pytest.mark.parametrize("size", [130, 65, 17])
def test_rs_partial_pack(dtype, fmt, size):
    """The reference's test_stoch_round_partial_pack sizes; ragged packs give
    the same values as the full-pack (vectorised) path does."""
    import b2x
    g = torch.Generator(device="cuda").manual_seed(size)
    a = torch.randn(size + 3, device="cuda", generator=g)
    r = torch.randint(-2 ** 31, 2 ** 31 - 1, (size + 3,), device="cuda", dtype=torch.int32, generator=g)
    y = b2x.stoch_round(a[:size], dtype, r[:size], rounding="rs").float()
    assert not torch.isnan(y).any() and not torch.isinf(y).any()
    full = b2x.stoch_round(a[:8 * (size // 8)], dtype, r[:8 * (size // 8)], rounding="rs").float()
    assert torch.equal(y[: full.numel()], full)
    # the tail element by element in a strided (unvectorised) layout
    a2 = torch.zeros((1, 2 * size), device="cuda")[:, 1:size + 1]
    a2.copy_(a[:size][None])
    r2 = torch.zeros((1, 2 * size), device="cuda", dtype=torch.int32)[:, 1:size + 1]
    r2.copy_(r[:size][None])
    assert torch.equal(b2x.stoch_round(a2, dtype, r2, rounding="rs").float()[0], y)


def test_rs_entropy_quality():
    """The reference's test_stoch_round_entropy_quality: different random
    words give different roundings for values that need rounding."""
    import b2x
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(256, device="cuda", generator=g) * 10.0
    r1 = torch.randint(-2 ** 31, 2 ** 31 - 1, (256,), device="cuda", dtype=torch.int32, generator=g)
    r2 = torch.randint(-2 ** 31, 2 ** 31 - 1, (256,), device="cuda", dtype=torch.int32, generator=g)
    b1 = b2x.stoch_round(a, torch.float8_e5m2, r1, rounding="rs").float()
    b2 = b2x.stoch_round(a, torch.float8_e5m2, r2, rounding="rs").float()
    assert (b1 != b2).sum().item() > 256 * 0.1
