"""Parity at the GEMM shapes the headline benchmark times.

The Llama-3-70B fp8 linear set at 8192 tokens (QKV 8192x10240x8192, gate+up
8192x57344x8192, down 8192x8192x28672) and the shards those layers become on
2, 4 and 8 GPUs (column-parallel N/g, row-parallel K/g), each with the
default configuration the benchmark uses.  Every shape is checked on 256
random rows x 256 random columns (plus the last row and column) at full K
against the float64 oracle, within the path's tolerance
max|C - C_ref| <= 1e-2 * ||A|| * ||B|| / sqrt(K) on top of bf16 rounding
(fp8_oracle.gemm_error).  Inputs are ~N(0,1), per-tensor e4m3 scales, as in
the benchmark configuration.
"""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = {
    "qkv": (8192, 10240, 8192),
    "gate_up": (8192, 57344, 8192),
    "down": (8192, 8192, 28672),
    "qkv/2": (8192, 5120, 8192), "gate_up/2": (8192, 28672, 8192), "down/2": (8192, 8192, 14336),
    "qkv/4": (8192, 2560, 8192), "gate_up/4": (8192, 14336, 8192), "down/4": (8192, 8192, 7168),
    "qkv/8": (8192, 1280, 8192), "gate_up/8": (8192, 7168, 8192), "down/8": (8192, 8192, 3584),
}


@pytest.mark.parametrize("name", list(SHAPES))
def test_headline_shape_sampled(name):
    import b2x
    M, N, K = SHAPES[name]
    g = torch.Generator(device="cuda").manual_seed(list(SHAPES).index(name))
    A, sa = b2x.quantize(torch.randn((M, K), device="cuda", generator=g), "tensor", torch.float8_e4m3fn)
    W, sb = b2x.quantize(torch.randn((N, K), device="cuda", generator=g), "tensor", torch.float8_e4m3fn)
    before = b2x.launch_count()
    C = b2x.matmul(A, W.t(), {}, scale_a=sa, scale_b=sb)
    torch.cuda.synchronize()
    assert b2x.launch_count() > before
    rows = torch.cat([torch.randperm(M, device="cuda", generator=g)[:256], torch.tensor([M - 1], device="cuda")])
    cols = torch.cat([torch.randperm(N, device="cuda", generator=g)[:256], torch.tensor([N - 1], device="cuda")])
    a_bits = A[rows].view(torch.uint8).cpu().numpy()
    b_bits = W[cols].view(torch.uint8).cpu().numpy().T
    ref = O.gemm(a_bits, b_bits, scale_mode="tensor", scale_a=sa.item(), scale_b=sb.item())
    got = C[rows][:, cols].float().cpu().numpy()
    err, tol = O.gemm_error(got, ref, O.fp8_bits_to_f64(a_bits, O.E4M3) * sa.item(),
                            O.fp8_bits_to_f64(b_bits, O.E4M3) * sb.item())
    assert err <= tol, f"{name} {M}x{N}x{K}: {err:.4g} > {tol:.4g}"
    assert b2x.read_device_status() == 0
    del A, W, C
    torch.cuda.empty_cache()
