"""GPU parity of the fp8 cast kernels (libb2x) against the CPU oracle and the
B200 golden vectors.  Bit-exact: every byte of q and every scale."""
import os

import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "cast_golden.npz")
FP8 = {O.E4M3: torch.float8_e4m3fn, O.E5M2: torch.float8_e5m2}


def _b2x():
    import b2x
    return b2x


def _run(x_np, src, fmt, mode, scale=None):
    b2x = _b2x()
    xt = torch.from_numpy(np.ascontiguousarray(x_np))
    if src == "bf16":
        xt = xt.to(torch.bfloat16)
    xt = xt.cuda()
    before = b2x.launch_count()
    q, s = b2x.quantize(xt, mode, FP8[fmt], None if scale is None else torch.tensor([scale], device="cuda"))
    torch.cuda.synchronize()
    assert b2x.launch_count() > before, "no libb2x kernel ran"
    return q.view(torch.uint8).cpu().numpy(), (None if s is None else s.cpu().numpy())


def _oracle_input(x_np, src):
    if src == "bf16":
        return torch.from_numpy(x_np).to(torch.bfloat16).float().numpy()
    return x_np


def _assert_bytes_equal(q, ref, x):
    bad = np.nonzero(q != ref)
    assert bad[0].size == 0, (f"{bad[0].size} byte mismatches; first at {tuple(b[0] for b in bad)}: "
                              f"x={x[tuple(b[0] for b in bad)]!r} got=0x{q[tuple(b[0] for b in bad)]:02x} "
                              f"want=0x{ref[tuple(b[0] for b in bad)]:02x}")


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2])
@pytest.mark.parametrize("mode", ["none", "mx1x32", "block1x128", "tensor", "tensor_noinf"])
def test_cast_matches_golden(src, fmt, mode):
    g = np.load(GOLDEN)
    noinf = mode == "tensor_noinf"
    if src == "f32":
        x = g["x_f32_noinf" if noinf else "x_f32"]
    else:
        x = O.bf16_bits_to_f32(g["x_bf16_noinf_bits" if noinf else "x_bf16_bits"])
    q, s = _run(x, "f32" if src == "f32" else "bf16", fmt, "tensor" if noinf else mode)
    key = f"{src}_{fmt}_{mode}"
    _assert_bytes_equal(q.reshape(x.shape), g[f"q_{key}"], x)
    if mode != "none":
        assert np.array_equal(np.asarray(s).reshape(-1).view(np.uint8),
                              g[f"s_{key}"].reshape(-1).view(np.uint8))


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2])
@pytest.mark.parametrize("mode", ["none", "tensor", "block1x128", "block128x128", "mx1x32"])
@pytest.mark.parametrize("shape", [(1024, 1024), (333, 1000), (1, 4100), (257, 129), (2, 3)])
def test_cast_matches_oracle(src, fmt, mode, shape):
    x = O.cast_input(shape[0] * shape[1], seed=hash((src, fmt, mode, shape)) % 1000).reshape(shape)
    q, s = _run(x, src, fmt, mode)
    xo = _oracle_input(x, src)
    rq, rs = O.quantize(xo, mode, fmt)
    _assert_bytes_equal(q.reshape(shape), rq, xo)
    if mode != "none":
        assert np.array_equal(np.asarray(s).reshape(-1).view(np.uint8), np.asarray(rs).reshape(-1).view(np.uint8))


def test_cast_given_scale_and_strided_rows():
    b2x = _b2x()
    x = O.cast_input(300 * 512, seed=11, special_frac=0).reshape(300, 512)
    xt = torch.from_numpy(x).cuda()[:, :384]  # row stride 512, 384 columns
    q, s = b2x.quantize(xt, "given", torch.float8_e4m3fn, torch.tensor([0.37], device="cuda"))
    rq, _ = O.quantize(x[:, :384], "given", O.E4M3, scale=np.float32(0.37))
    _assert_bytes_equal(q.view(torch.uint8).cpu().numpy(), rq, x[:, :384])
    q, s = b2x.quantize(xt, "block1x128", torch.float8_e5m2)
    rq, rs = O.quantize(x[:, :384], "block1x128", O.E5M2)
    _assert_bytes_equal(q.view(torch.uint8).cpu().numpy(), rq, x[:, :384])
    assert np.array_equal(s.cpu().numpy(), rs)


def test_amax_nan_ignoring():
    b2x = _b2x()
    x = O.cast_input(1 << 20, seed=2, special_frac=0)
    x[::1000] = np.nan
    a = b2x.amax(torch.from_numpy(x).cuda()).item()
    assert np.float32(a) == O.nan_ignoring_absmax(x)


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("mode", ["tensor", "block1x128"])
def test_cast_full_size_64M(src, mode):
    """The cast benchmark configuration at full size (64M elements, 1% outliers, 0.01%
    NaN/Inf): every byte equal to an independent torch restatement of the
    recipe on the GPU, with NaN inputs checked against the pinned +FMAX code."""
    b2x = _b2x()
    n = 64 * 1024 * 1024
    R, C = 8192, n // 8192
    x = torch.from_numpy(O.cast_input(n, seed=0)).reshape(R, C).cuda()
    if src == "bf16":
        x = x.to(torch.bfloat16)
    for fmt in (O.E4M3, O.E5M2):
        fm = float(O.FMAX[fmt])
        q, s = b2x.quantize(x, mode, FP8[fmt])
        # fp32 divisions / products evaluated in float64 and rounded once to
        # float32 are the IEEE-rounded fp32 results (torch's tensor/scalar
        # division multiplies by a reciprocal, which is not).
        xf = x.float()
        absx = torch.where(torch.isnan(xf), torch.zeros_like(xf), xf.abs())
        if mode == "tensor":
            sc = (absx.max().double() / fm).float().reshape(1, 1)
        else:
            sc = (absx.reshape(R, C // 128, 128).amax(-1).double() / fm).float()
        assert torch.equal(s.reshape(sc.shape).view(torch.int32), sc.view(torch.int32))
        inv = torch.where(sc == 0, torch.zeros_like(sc), (1.0 / sc.double()).float())
        if mode == "tensor":
            y = (xf.double() * inv.double()).float()
        else:
            y = (xf.reshape(R, C // 128, 128).double() * inv[..., None].double()).float().reshape(R, C)
        y = torch.where(torch.isnan(y), torch.full_like(y, fm), y.clamp(-fm, fm))  # scaled: NaN -> +FMAX
        ref = y.to(FP8[fmt]).view(torch.uint8)
        got = q.view(torch.uint8)
        nbad = (ref != got).sum().item()
        assert nbad == 0, f"{nbad} mismatching bytes ({src}, {mode}, {fmt})"
