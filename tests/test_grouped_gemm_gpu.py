"""GPU parity of the grouped fp8 GEMM (b2x.grouped_gemm, C ABI
b2x_fp8_grouped_gemm) against the float64 CPU oracle, group by group, with the
module-wide GEMM tolerance (fp8_oracle.gemm_error).  Shapes: the reference's
test_op groups (blackwell-grouped-gemm_test.py:787-815: square 1024/512/256/128)
and ragged mixture-of-experts groups, including empty and one-row groups."""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu


def _group(M, N, K, seed, scaled=True):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32)
    mode = "tensor" if scaled else "none"
    qa, sa = O.quantize(a, mode, O.E4M3)
    qw, sw = O.quantize(w * (1.0 if scaled else 0.25), mode, O.E4M3)
    return qa, qw, (np.float32(sa) if scaled else None), (np.float32(sw) if scaled else None)


def _run(shapes, scaled=True, block_n=0):
    import b2x
    groups = [_group(M, N, K, 100 + i, scaled) for i, (M, N, K) in enumerate(shapes)]
    A = [torch.from_numpy(g[0]).cuda().view(torch.float8_e4m3fn) for g in groups]
    B = [torch.from_numpy(g[1]).cuda().view(torch.float8_e4m3fn) for g in groups]
    SA = [torch.tensor([g[2]], device="cuda") for g in groups] if scaled else None
    SB = [torch.tensor([g[3]], device="cuda") for g in groups] if scaled else None
    before = b2x.launch_count()
    C = b2x.grouped_gemm(A, B, SA, SB, block_n=block_n)
    torch.cuda.synchronize()
    if any(M * N for (M, N, _) in shapes):
        assert b2x.launch_count() == before + 1, "expected exactly one grouped kernel launch"
    for i, ((M, N, K), g) in enumerate(zip(shapes, groups)):
        assert tuple(C[i].shape) == (M, N)
        if M * N == 0:
            continue
        ref = O.gemm(g[0], g[1].T, O.E4M3, O.E4M3, "tensor" if scaled else "none", g[2], g[3])
        a_deq = O.fp8_bits_to_f64(g[0], O.E4M3) * (float(g[2]) if scaled else 1.0)
        b_deq = O.fp8_bits_to_f64(g[1].T, O.E4M3) * (float(g[3]) if scaled else 1.0)
        err, tol = O.gemm_error(C[i].float().cpu().numpy(), ref, a_deq, b_deq)
        assert err <= tol, f"group {i} {M}x{N}x{K}: error {err:.4g} > tol {tol:.4g}"


def test_grouped_reference_shapes():
    _run([(1024, 1024, 1024), (512, 512, 512), (256, 256, 256), (128, 128, 128)])


@pytest.mark.parametrize("block_n", [0, 128, 256])
def test_grouped_ragged_experts(block_n):
    _run([(37, 768, 512), (0, 768, 512), (300, 768, 512), (1, 768, 512), (129, 768, 512), (513, 200, 384)],
         block_n=block_n)


def test_grouped_unscaled_and_mixed_k():
    _run([(256, 512, 1024), (128, 1000, 96), (64, 64, 2048)], scaled=False)


def test_grouped_many_groups():
    rng = np.random.default_rng(1)
    shapes = [(int(m), 512, 256) for m in rng.integers(0, 300, 24)]
    _run(shapes)


def test_grouped_rejects_bad_groups():
    import b2x
    a = torch.zeros((16, 64), device="cuda", dtype=torch.float8_e4m3fn)
    b = torch.zeros((32, 48), device="cuda", dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError):
        b2x.grouped_gemm([a], [b])
    assert b2x.grouped_gemm([], []) == []
