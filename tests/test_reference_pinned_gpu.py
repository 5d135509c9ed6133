"""GPU kernels against outputs of the reference's own code.

Fixtures: tests/golden/ref_kernels_golden.npz, made by tests/golden/
make_golden_reference.py from the reference's _compute_scale_and_quantize
(extensions/utlx/tlx/language/tlx/mxfp8_utils.py:13-86) and _reduce_k_kernel
(extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:1033-1056).  Both are
bit-exact requirements: casts are byte work and the reduction is an fp32 sum
in split order followed by one rounding.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FP8 = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2}


@pytest.fixture(scope="module")
def kern():
    return dict(np.load(os.path.join(GOLD, "ref_kernels_golden.npz")))


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_mx_quantize_matches_reference_function(kern, src, fmt):
    import b2x
    if src == "f32":
        x = torch.from_numpy(kern["mx_x_f32"]).cuda()
    else:
        x = torch.from_numpy(kern["mx_x_bf16_bits"].view(np.int16)).cuda().view(torch.bfloat16)
    q, s = b2x.quantize(x, "mx1x32", FP8[fmt])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(s.cpu().numpy(), kern[f"mx_{src}_{fmt}_s"])
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), kern[f"mx_{src}_{fmt}_q"])


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("shape", ["100x200x3", "32x128x8"])
def test_reduce_k_matches_reference_kernel(kern, dt, shape):
    import b2x
    M, N, sk = (int(v) for v in shape.split("x"))
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dt]
    bits = {"f32": torch.int32, "bf16": torch.int16, "f16": torch.int16}[dt]
    ws = torch.from_numpy(kern[f"rk_{dt}_{shape}_ws"]).cuda().view(tdt)
    c = torch.full((M, N), float("nan"), device="cuda", dtype=tdt)
    b2x.reduce_k(ws, c, M, N, sk)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(c.view(bits).cpu().numpy(), kern[f"rk_{dt}_{shape}_c"])
    assert b2x.read_device_status() == 0
