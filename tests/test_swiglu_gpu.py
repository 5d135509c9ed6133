"""GPU check of the gate+up GEMM fused with SwiGLU and fp8 quantization
(b2x.gemm_swiglu, C ABI b2x_fp8_gemm_swiglu) against the float64 oracle:
h_ref = silu(g) * u from the oracle GEMMs of the gate and up halves.
Tolerances.  h differs from the float64 h_ref only by the fp32 accumulation
order of the GEMM and the fast exp / division of silu (a few 1e-6 relative):
  scales (1x128 block scales, and the amax of the given-scale mode):
      |s - s_ref| <= 1e-5 * s_ref
  fp8 codes: q must equal the oracle's quantization of h_ref with the kernel's
      own scale, byte for byte, except that a neighbouring code (one step) is
      accepted where h_ref * inv lies within 1e-3 relative of the rounding
      boundary between the two codes."""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu


def _operands(M, I, K, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    wg = rng.standard_normal((I, K), dtype=np.float32)
    wu = rng.standard_normal((I, K), dtype=np.float32)
    qx, sx = O.quantize(x, "tensor", O.E4M3)
    qg, sg = O.quantize(wg, "tensor", O.E4M3)
    qu, su = O.quantize(wu, "tensor", O.E4M3)
    return qx, np.float32(sx), qg, np.float32(sg), qu, np.float32(su)


def _h_ref(qx, sx, qg, sg, qu, su):
    g = O.gemm(qx, qg.T, O.E4M3, O.E4M3, "tensor", sx, sg)
    u = O.gemm(qx, qu.T, O.E4M3, O.E4M3, "tensor", sx, su)
    return g / (1.0 + np.exp(-g)) * u


def _check_codes(q, y):
    """q: the kernel's e4m3 bytes; y: h_ref times the kernel's inverse scale."""
    yc = np.clip(y, -448.0, 448.0)
    want = O.f32_to_fp8_bits(yc.astype(np.float32), O.E4M3)
    diff = q != want
    if not diff.any():
        return
    vq = O.fp8_bits_to_f64(q[diff], O.E4M3)
    vw = O.fp8_bits_to_f64(want[diff], O.E4M3)
    yd = yc[diff]
    # neighbouring codes: same sign, magnitudes one code apart
    one_step = ((q[diff] & 0x80) == (want[diff] & 0x80)) & (np.abs((q[diff] & 0x7F).astype(int) -
                                                                      (want[diff] & 0x7F).astype(int)) == 1)
    near = np.abs((vq + vw) / 2 - yd) <= 1e-3 * np.abs(yd)
    bad = ~(one_step & near)
    assert not bad.any(), (f"{bad.sum()} of {q.size} codes differ beyond a boundary case; first: "
                           f"got {vq[bad][0]} want {vw[bad][0]} y {yd[bad][0]}")


def _run(M, I, K, mode, seed=0):
    import b2x
    qx, sx, qg, sg, qu, su = _operands(M, I, K, seed)
    # one weight scale for the interleaved tensor: re-quantize gate and up with a common scale
    wg = O.fp8_bits_to_f64(qg, O.E4M3) * sg
    wu = O.fp8_bits_to_f64(qu, O.E4M3) * su
    w = np.concatenate([wg, wu]).astype(np.float32)
    qw, sw = O.quantize(w, "tensor", O.E4M3)
    qg, qu, sg, su = qw[:I], qw[I:], np.float32(sw), np.float32(sw)
    X = torch.from_numpy(qx).cuda().view(torch.float8_e4m3fn)
    Wg = torch.from_numpy(qg).cuda().view(torch.float8_e4m3fn)
    Wu = torch.from_numpy(qu).cuda().view(torch.float8_e4m3fn)
    W = b2x.interleave_gate_up(Wg, Wu)
    tsx, tsw = torch.tensor([sx], device="cuda"), torch.tensor([sw], device="cuda")
    href = _h_ref(qx, sx, qg, sg, qu, su)
    before = b2x.launch_count()
    if mode == "block1x128":
        h, s = b2x.gemm_swiglu(X, W, tsx, tsw)
        torch.cuda.synchronize()
        s = s.cpu().numpy()
        sref = np.abs(href).reshape(M, I // 128, 128).max(axis=2) / 448.0
        assert np.all(np.abs(s - sref) <= 1e-5 * sref + 1e-30), (np.abs(s - sref) / sref).max()
        inv = np.where(s == 0, 0.0, 1.0 / s.astype(np.float64))
        _check_codes(h.view(torch.uint8).cpu().numpy(), href * np.repeat(inv, 128, axis=1))
    elif mode == "mx1x32":
        h, s = b2x.gemm_swiglu(X, W, tsx, tsw, mode="mx1x32")
        torch.cuda.synchronize()
        s = s.cpu().numpy()
        # the E8M0 byte of each 32-column group from the oracle's h: it may sit
        # one step off only where amax / 448 lies within 1e-5 of a power of two
        gm = np.abs(href).reshape(M, I // 32, 32).max(axis=2) / 448.0
        want = np.where(gm > 0, np.ceil(np.log2(np.maximum(gm, 1e-300))) + 127, 0).astype(np.int64)
        diff = s.astype(np.int64) - want
        near = np.abs(np.log2(np.maximum(gm, 1e-300)) - np.round(np.log2(np.maximum(gm, 1e-300)))) < 1e-5
        assert np.all((diff == 0) | (near & (np.abs(diff) == 1))), np.abs(diff).max()
        inv = np.where(s == 0, 0.0, np.exp2(127.0 - s.astype(np.float64)))
        _check_codes(h.view(torch.uint8).cpu().numpy(), href * np.repeat(inv, 32, axis=1))
    else:
        given = float(np.abs(href).max() / 448.0 * 1.25)
        amax = torch.zeros(1, device="cuda")
        h, _ = b2x.gemm_swiglu(X, W, tsx, tsw, mode="given", h_scale=torch.tensor([given], device="cuda"),
                               h_amax=amax)
        torch.cuda.synchronize()
        assert abs(amax.item() - np.abs(href).max()) <= 1e-5 * np.abs(href).max()
        inv = 1.0 / np.float64(np.float32(given))
        _check_codes(h.view(torch.uint8).cpu().numpy(), href * inv)
    assert b2x.launch_count() == before + 1, "expected one fused kernel launch"



@pytest.mark.parametrize("M,I,K", [(256, 256, 512), (512, 384, 1024), (200, 128, 256), (64, 256, 384)])
def test_swiglu_block_scales(M, I, K):
    _run(M, I, K, "block1x128")


@pytest.mark.parametrize("M,I,K", [(256, 256, 512), (200, 384, 256)])
def test_swiglu_mx_scales(M, I, K):
    """The E8M0 1x32 recipe of _to_mxfp8_block (mxfp8_utils.py:89-128) in the
    epilogue: scale bytes and h codes against the oracle's h."""
    _run(M, I, K, "mx1x32", seed=2)


@pytest.mark.parametrize("M,I,K", [(256, 256, 512), (384, 512, 256)])
def test_swiglu_given_scale(M, I, K):
    _run(M, I, K, "given", seed=4)


def test_swiglu_rejects_bad_shapes():
    import b2x
    x = torch.zeros((128, 128), device="cuda", dtype=torch.float8_e4m3fn)
    w = torch.zeros((384, 128), device="cuda", dtype=torch.float8_e4m3fn)  # 2I = 384 is not a multiple of 256
    with pytest.raises(Exception):
        b2x.gemm_swiglu(x, w)


def test_swiglu_mx_feeds_mx_down_projection():
    """gate+up -> SwiGLU -> fp8 h with E8M0 1x32 scales, consumed as-is by the
    MX (block-scale tensor-core) down GEMM: the chain without a re-quantize
    pass, checked against the oracle's MX GEMM on the kernel's own h."""
    import b2x
    M, I, K, N = 256, 512, 512, 384
    qx, sx, qg, sg, qu, su = _operands(M, I, K, 7)
    X = torch.from_numpy(qx).cuda().view(torch.float8_e4m3fn)
    W = b2x.interleave_gate_up(torch.from_numpy(qg).cuda().view(torch.float8_e4m3fn),
                               torch.from_numpy(qu).cuda().view(torch.float8_e4m3fn))
    tsx = torch.tensor([sx], device="cuda")
    tsw = torch.tensor([sg], device="cuda")  # gate and up share a scale only approximately: fine here
    h, hs = b2x.gemm_swiglu(X, W, tsx, tsw, mode="mx1x32")
    g = torch.Generator(device="cuda").manual_seed(3)
    wd, wds = b2x.quantize(torch.randn((N, I), device="cuda", generator=g), "mx1x32", torch.float8_e4m3fn)
    out = b2x.matmul(h, wd.t(), {}, scale_a=hs, scale_b=wds)
    torch.cuda.synchronize()
    hb, hsb = h.view(torch.uint8).cpu().numpy(), hs.cpu().numpy()
    wb, wsb = wd.view(torch.uint8).cpu().numpy(), wds.cpu().numpy()
    ref = O.gemm(hb, wb.T, O.E4M3, O.E4M3, "mx", hsb, wsb)
    ad = O.fp8_bits_to_f64(hb, O.E4M3) * np.exp2(np.repeat(hsb.astype(np.float64) - 127, 32, axis=1))
    bd = (O.fp8_bits_to_f64(wb, O.E4M3) * np.exp2(np.repeat(wsb.astype(np.float64) - 127, 32, axis=1))).T
    err, tol = O.gemm_error(out.float().cpu().numpy(), ref, ad, bd)
    assert err <= tol, f"{err} > {tol}"
