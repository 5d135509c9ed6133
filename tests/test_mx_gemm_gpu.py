"""GPU parity of the MX (E8M0 1x32) block-scaled fp8 GEMM (tcgen05
kind::mxf8f6f4.block_scale) against the float64 CPU oracle.

C[m, n] = sum_j 2^(sA[m, j] - 127) * 2^(sB[n, j] - 127) * (A[m, 32j:32j+32] . B[32j:32j+32, n]),
the formula of the reference's test_async_dot_scaled (test_tlx.py:2298-2444).
Tolerance: the module-wide GEMM bound on the dequantized operands
(fp8_oracle.gemm_error: 1e-2 * ||A|| * ||B|| / sqrt(K) beyond the bf16
rounding of C).  Inputs span many binades per 32-element group so that the
scales, not just the fp8 mantissas, are exercised.
"""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu

FP8 = {O.E4M3: torch.float8_e4m3fn, O.E5M2: torch.float8_e5m2}


def _mx_operand(rows, K, fmt, seed, spread=12):
    """[rows, K] fp32 whose 32-element groups sit at random binades, quantized
    to fp8 bits + E8M0 scales by the oracle (the reference recipe)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K), dtype=np.float32)
    mag = np.ldexp(1.0, rng.integers(-spread, spread + 1, size=(rows, K // 32))).astype(np.float32)
    x *= np.repeat(mag, 32, axis=1)
    q, s = O.quantize(x, "mx1x32", fmt)
    return q, s


def _deq(q, s, fmt):
    return O.fp8_bits_to_f64(q, fmt) * np.ldexp(1.0, np.repeat(s.astype(np.int64) - 127, 32, axis=1))


def _run(M, N, K, fa=O.E4M3, fb=O.E4M3, config=None, seed=0):
    import b2x
    qa, sa = _mx_operand(M, K, fa, seed)
    qw, sw = _mx_operand(N, K, fb, seed + 1)
    A = torch.from_numpy(qa).cuda().view(FP8[fa])
    W = torch.from_numpy(qw).cuda().view(FP8[fb])
    SA = torch.from_numpy(np.ascontiguousarray(sa)).cuda()
    SW = torch.from_numpy(np.ascontiguousarray(sw)).cuda()
    before = b2x.launch_count()
    C = b2x.matmul(A, W.t(), config, scale_a=SA, scale_b=SW)
    torch.cuda.synchronize()
    assert b2x.launch_count() > before, "no libb2x kernel ran"
    ref = O.gemm(qa, qw.T, fa, fb, "mx", sa, sw)
    err, tol = O.gemm_error(C.float().cpu().numpy(), ref, _deq(qa, sa, fa), _deq(qw, sw, fb).T)
    assert err <= tol, f"MX {M}x{N}x{K} {fa}x{fb} {config}: error {err:.4g} > tol {tol:.4g}"
    return C


@pytest.mark.parametrize("M,N,K", [(128, 192, 128), (256, 384, 512), (200, 300, 256), (1, 64, 128),
                                   (384, 1000, 1024)])
def test_mx_gemm_shapes(M, N, K):
    _run(M, N, K)


@pytest.mark.parametrize("bn", [128, 192])
def test_mx_gemm_tile_widths(bn):
    _run(320, 640, 768, config={"BLOCK_SIZE_N": bn}, seed=3)


@pytest.mark.parametrize("fa,fb", [(O.E5M2, O.E4M3), (O.E4M3, O.E5M2), (O.E5M2, O.E5M2)])
def test_mx_gemm_mixed_formats(fa, fb):
    _run(256, 512, 512, fa, fb, seed=5)


def test_mx_gemm_matches_gpu_cast_scales():
    """End to end on the device: b2x.quantize(..., 'mx1x32') then the MX GEMM,
    against the oracle run on the same quantized bytes."""
    import b2x
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(512, 1024, device="cuda", generator=g)
    w = torch.randn(768, 1024, device="cuda", generator=g) * 3.0
    qx, sx = b2x.quantize(x, "mx1x32", torch.float8_e4m3fn)
    qw, sw = b2x.quantize(w, "mx1x32", torch.float8_e4m3fn)
    C = b2x.matmul(qx, qw.t(), scale_a=sx, scale_b=sw)
    torch.cuda.synchronize()
    bx, bw = qx.view(torch.uint8).cpu().numpy(), qw.view(torch.uint8).cpu().numpy()
    nsx, nsw = sx.cpu().numpy(), sw.cpu().numpy()
    ref = O.gemm(bx, bw.T, O.E4M3, O.E4M3, "mx", nsx, nsw)
    err, tol = O.gemm_error(C.float().cpu().numpy(), ref, _deq(bx, nsx, O.E4M3), _deq(bw, nsw, O.E4M3).T)
    assert err <= tol, (err, tol)
    # and close to the unquantized product (fp8 quantization error only)
    exact = (x.double() @ w.double().t()).cpu().numpy()
    rel = np.abs(C.float().cpu().numpy() - exact).max() / np.abs(exact).max()
    assert rel < 0.05, rel


def test_mx_gemm_large_sampled():
    """4096 x 7168 x 7168 (the block-scaled benchmark shape) in MX form, checked
    on a sample of rows against the oracle."""
    import b2x
    M, N, K = 4096, 7168, 7168
    qa, sa = _mx_operand(M, K, O.E4M3, 11, spread=4)
    qw, sw = _mx_operand(N, K, O.E4M3, 12, spread=4)
    C = b2x.matmul(torch.from_numpy(qa).cuda().view(torch.float8_e4m3fn),
                   torch.from_numpy(qw).cuda().view(torch.float8_e4m3fn).t(),
                   scale_a=torch.from_numpy(sa).cuda(), scale_b=torch.from_numpy(sw).cuda())
    torch.cuda.synchronize()
    rows = np.random.default_rng(0).choice(M, 48, replace=False)
    ref = O.gemm(qa[rows], qw.T, O.E4M3, O.E4M3, "mx", sa[rows], sw)
    err, tol = O.gemm_error(C.float().cpu().numpy()[rows], ref, _deq(qa[rows], sa[rows], O.E4M3),
                            _deq(qw, sw, O.E4M3).T)
    assert err <= tol, (err, tol)


def test_mx_gemm_rejects_ragged_k():
    import b2x
    a = torch.zeros(128, 96, device="cuda", dtype=torch.float8_e4m3fn)
    w = torch.zeros(128, 96, device="cuda", dtype=torch.float8_e4m3fn)
    s = torch.full((128, 3), 127, device="cuda", dtype=torch.uint8)
    with pytest.raises(Exception):
        b2x.matmul(a, w.t(), {"BLOCK_SIZE_N": 128}, scale_a=s, scale_b=s)
        torch.cuda.synchronize()
