"""GPU test of b2x_fp8_gemm_splitk_noalloc, the split-K GEMM entry point for
callers that may not allocate device memory (memory reserved up front by a
serving loop, a foreign framework's pool, a C host without an allocator).

It is called through the C ABI with no workspace, twice in a row on the same
inputs, and each result is compared with the regular entry point
(b2x_fp8_gemm with a caller-provided workspace) within the GEMM tolerance
used by the other tests (fp8_oracle.gemm_error).  This file is collected last
so that a run stopping at the first failure has run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    qa, sa = O.quantize(rng.standard_normal((M, K), dtype=np.float32), "tensor", O.E4M3)
    qw, sw = O.quantize(rng.standard_normal((N, K), dtype=np.float32), "tensor", O.E4M3)
    return qa, np.float32(sa), qw, np.float32(sw)


def _call_noalloc(A, W, sa, sb, split_k):
    from b2x import _lib as L
    from b2x import ops
    C = torch.full((A.shape[0], W.shape[0]), float("nan"), dtype=torch.bfloat16, device="cuda")
    cfg = [0] * len(ops.CONFIG_FIELDS)
    cfg[ops.CONFIG_FIELDS.index("split_k")] = split_k
    g = ops._gemm_args(A, W.t(), C, "tensor", sa, sb, cfg)
    st = L.lib().b2x_fp8_gemm_splitk_noalloc(ctypes.byref(g), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == L.OK, L.lib().b2x_last_error().decode()
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("shape,split_k", [((64, 8192, 28672), 8), ((200, 1024, 4096), 4), ((128, 512, 1024), 2)])
def test_noalloc_matches_workspace_entry_point(shape, split_k):
    import b2x
    M, N, K = shape
    qa, sa, qw, sw = _inputs(M, N, K, seed=M + N)
    A = torch.from_numpy(qa).cuda().view(torch.float8_e4m3fn)
    W = torch.from_numpy(qw).cuda().view(torch.float8_e4m3fn)
    sa_t = torch.tensor([sa], device="cuda")
    sw_t = torch.tensor([sw], device="cuda")
    ref = b2x.matmul(A, W.t(), {"SPLIT_K": split_k}, scale_a=sa_t, scale_b=sw_t).float().cpu().numpy()
    ad = O.fp8_bits_to_f64(qa, O.E4M3) * sa
    bd = O.fp8_bits_to_f64(qw, O.E4M3).T * sw
    for call in range(2):  # the second call finds the scratch as the first one left it
        c = _call_noalloc(A, W, sa_t, sw_t, split_k).float().cpu().numpy()
        assert np.isfinite(c).all()
        err, tol = O.gemm_error(c, ref.astype(np.float64), ad, bd)
        assert err <= tol, f"call {call}: {err} > {tol}"


def test_noalloc_rejects_problems_beyond_its_scratch():
    from b2x import _lib as L
    from b2x import ops
    M, N, K = 1024, 4096, 4096  # split-K sum would need 16 MiB
    A = torch.zeros((M, K), dtype=torch.float8_e4m3fn, device="cuda")
    W = torch.zeros((N, K), dtype=torch.float8_e4m3fn, device="cuda")
    C = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    cfg = [0] * len(ops.CONFIG_FIELDS)
    cfg[ops.CONFIG_FIELDS.index("split_k")] = 2
    g = ops._gemm_args(A, W.t(), C, "none", None, None, cfg)
    assert L.lib().b2x_fp8_gemm_splitk_noalloc(ctypes.byref(g), None) == L.ERR_WORKSPACE
    assert b"scratch" in L.lib().b2x_last_error()
