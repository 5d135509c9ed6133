"""GPU check of the gate+up GEMM fused with SwiGLU and fp8 quantization
(b2x.gemm_swiglu, C ABI b2x_fp8_gemm_swiglu) against the float64 oracle:
h_ref = silu(g) * u from the oracle GEMMs of the gate and up halves.
Floating-point tolerances (h passes through exp and an fp8 rounding):
  block 1x128 scales:  |s - amax_ref / 448| <= 1e-2 * s_ref + tiny
  dequantized h:       |q * s - h_ref| <= 2^-3 |h_ref| + 2e-2 * amax_row(|h_ref|)
(half an e4m3 ulp is 2^-4 |h|; the rest covers the GEMM's own error bound
and the fast exp)."""
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
    amax_row = np.abs(href).max(axis=1, keepdims=True)
    before = b2x.launch_count()
    if mode == "block1x128":
        h, s = b2x.gemm_swiglu(X, W, tsx, tsw)
        torch.cuda.synchronize()
        s = s.cpu().numpy()
        sref = np.abs(href).reshape(M, I // 128, 128).max(axis=2) / 448.0
        assert np.all(np.abs(s - sref) <= 1e-2 * sref + 1e-30), np.abs(s - sref).max()
        deq = O.fp8_bits_to_f64(h.view(torch.uint8).cpu().numpy(), O.E4M3) * np.repeat(s, 128, axis=1)
    else:
        given = float(np.abs(href).max() / 448.0 * 1.25)
        amax = torch.zeros(1, device="cuda")
        h, _ = b2x.gemm_swiglu(X, W, tsx, tsw, mode="given", h_scale=torch.tensor([given], device="cuda"),
                               h_amax=amax)
        torch.cuda.synchronize()
        assert abs(amax.item() - np.abs(href).max()) <= 1e-2 * np.abs(href).max()
        deq = O.fp8_bits_to_f64(h.view(torch.uint8).cpu().numpy(), O.E4M3) * np.float64(np.float32(given))
    assert b2x.launch_count() == before + 1, "expected one fused kernel launch"
    err = np.abs(deq - href) - (2.0 ** -3) * np.abs(href) - 2e-2 * amax_row
    assert err.max() <= 0, f"{M}x{I}x{K} {mode}: worst excess {err.max():.4g}"


@pytest.mark.parametrize("M,I,K", [(256, 256, 512), (512, 384, 1024), (200, 128, 256), (64, 256, 384)])
def test_swiglu_block_scales(M, I, K):
    _run(M, I, K, "block1x128")


@pytest.mark.parametrize("M,I,K", [(256, 256, 512), (384, 512, 256)])
def test_swiglu_given_scale(M, I, K):
    _run(M, I, K, "given", seed=4)


def test_swiglu_rejects_bad_shapes():
    import b2x
    x = torch.zeros((128, 128), device="cuda", dtype=torch.float8_e4m3fn)
    w = torch.zeros((384, 128), device="cuda", dtype=torch.float8_e4m3fn)  # 2I = 384 is not a multiple of 256
    with pytest.raises(Exception):
        b2x.gemm_swiglu(x, w)
