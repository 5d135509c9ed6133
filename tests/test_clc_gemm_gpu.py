"""GPU parity of the cluster-launch-control GEMM (b2x.blackwell_gemm_clc.matmul,
C ABI b2x_fp8_gemm_clc) against the float64 oracle, within the path's
tolerance (fp8_oracle.gemm_error).  The grid has one CTA per output tile, so
every shape with more tiles than resident CTAs exercises the hand-over of
tiles through clusterlaunchcontrol.try_cancel; split-K units are scheduled
the same way."""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    import b2x
    g = torch.Generator(device="cuda").manual_seed(seed)
    A, sa = b2x.quantize(torch.randn((M, K), device="cuda", generator=g), "tensor", torch.float8_e4m3fn)
    W, sw = b2x.quantize(torch.randn((N, K), device="cuda", generator=g), "tensor", torch.float8_e4m3fn)
    return A, sa, W, sw


def _check(C, A, sa, W, sw, rows=None, cols=None):
    a_bits = A.view(torch.uint8).cpu().numpy()
    w_bits = W.view(torch.uint8).cpu().numpy()
    c = C.float().cpu().numpy()
    if rows is not None:
        a_bits, c = a_bits[rows], c[rows]
    if cols is not None:
        w_bits, c = w_bits[cols], c[:, cols]
    ref = O.gemm(a_bits, w_bits.T, scale_mode="tensor", scale_a=sa.item(), scale_b=sw.item())
    err, tol = O.gemm_error(c, ref, O.fp8_bits_to_f64(a_bits, O.E4M3) * sa.item(),
                            O.fp8_bits_to_f64(w_bits.T, O.E4M3) * sw.item())
    assert err <= tol, f"{err} > {tol}"


@pytest.mark.parametrize("M,N,K,cfg", [
    (512, 512, 512, None),                        # 16 tiles: fewer than the SMs
    (2048, 4096, 1024, None),                     # 256 tiles of 128x256: tiles handed over
    (4096, 4096, 512, {"BLOCK_SIZE_N": 128}),     # 1024 tiles: many hand-overs per CTA
    (384, 1000, 640, {"BLOCK_SIZE_N": 64}),       # ragged N, 64-wide tiles
    (256, 2048, 4096, {"SPLIT_K": 4, "BLOCK_SIZE_N": 128}),   # split-K units
])
def test_clc_gemm_matches_oracle(M, N, K, cfg):
    import b2x
    from b2x import blackwell_gemm_clc
    A, sa, W, sw = _operands(M, N, K, seed=M + N + K)
    before = b2x.launch_count()
    C = blackwell_gemm_clc.matmul(A, W.t(), cfg, scale_a=sa, scale_b=sw)
    torch.cuda.synchronize()
    assert b2x.launch_count() == before + 1
    b2x.check_device()
    if M * N > 2048 * 2048:
        g = torch.Generator(device="cpu").manual_seed(1)
        rows = np.sort(torch.randperm(M, generator=g)[:256].numpy())
        cols = np.sort(torch.randperm(N, generator=g)[:256].numpy())
        _check(C, A, sa, W, sw, rows, cols)
    else:
        _check(C, A, sa, W, sw)


def test_clc_equals_persistent_schedule():
    """Same tiles, same K order per tile: the CLC schedule gives the persistent
    kernel's bits."""
    import b2x
    from b2x import blackwell_gemm_clc
    A, sa, W, sw = _operands(2048, 2048, 1024, seed=5)
    c1 = blackwell_gemm_clc.matmul(A, W.t(), {"BLOCK_SIZE_N": 256}, scale_a=sa, scale_b=sw)
    c2 = b2x.matmul(A, W.t(), {"BLOCK_SIZE_N": 256, "NUM_CTAS": 1}, scale_a=sa, scale_b=sw)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)


def test_clc_rejects_block_scales():
    from b2x import blackwell_gemm_clc
    A = torch.zeros((256, 256), device="cuda", dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError):
        blackwell_gemm_clc.matmul(A, A.t(), None, scale_a=torch.ones((256, 2), device="cuda"),
                                  scale_b=torch.ones((2, 2), device="cuda"))
