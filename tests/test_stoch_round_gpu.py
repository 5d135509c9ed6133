"""GPU parity of the stochastic-rounding cast (b2x.stoch_round, C ABI
b2x_stoch_round) against the integer CPU oracle (fp8_oracle.stoch_round):
bit-exact for every element, including signed zeros, subnormals, values
beyond the target range, +-Inf and NaN.  Also the properties the reference's
test_stoch_round (test_tlx.py:5126-5213) checks, and unbiasedness."""
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
    x, r = _inputs(shape, seed=hash((fmt, shape)) & 0xFFFF)
    before = b2x.launch_count()
    y = b2x.stoch_round(torch.from_numpy(x).cuda(), dtype, torch.from_numpy(r.view(np.int32)).cuda())
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
    y = b2x.stoch_round(xt, torch.float8_e4m3fn, rt)
    want = O.stoch_round(x[:, 16:144].reshape(-1), r[:, 16:144].reshape(-1), "e4m3")
    assert np.array_equal(_bits(y).reshape(-1), want)


@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_stoch_round_reference_properties(dtype, fmt):
    """The checks of the reference's test_stoch_round on 256 randn values."""
    import b2x
    torch.manual_seed(0)
    a = torch.randn(256, dtype=torch.float32, device="cuda")
    rbits = torch.randint(0, 2 ** 31 - 1, (256,), device="cuda", dtype=torch.int32) * 2 + 1
    b = b2x.stoch_round(a, dtype, rbits)
    bf = b.float()
    assert not torch.isnan(bf).any() and not torch.isinf(bf).any()
    exact = bf == a
    assert torch.equal(b[exact].float(), a[exact].to(dtype).float())
    lo = a.to(dtype).float()
    # each result is one of the two neighbours of a
    assert (torch.abs(bf - a) <= torch.abs(lo - a) * 2 + 1e-30 + torch.abs(a) * 0.25).all()


@pytest.mark.parametrize("dtype,fmt", TARGETS)
def test_stoch_round_is_unbiased(dtype, fmt):
    import b2x
    n = 1 << 22
    vals = {"e4m3": 1.03, "e5m2": 1.1, "f16": 1.0001, "bf16": 1.001}
    x = torch.full((n,), vals[fmt], dtype=torch.float32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    r = torch.randint(-2 ** 31, 2 ** 31 - 1, (n,), device="cuda", dtype=torch.int32, generator=g)
    mean = b2x.stoch_round(x, dtype, r).double().mean().item()
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
