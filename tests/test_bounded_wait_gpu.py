"""The bounded-wait failure path of the GEMM kernels, exercised without a
GPU fault: a test hook (b2x_debug_inject) lowers every mbarrier wait limit to
1 ms and makes the paired GEMM's MMA warp withhold the accumulator-ready
signal of its first tile.  The epilogue's wait then runs out; the kernel must
record 0x103 (epilogue) in the device status word, unwind every role (TMA
producer, MMA issuer, epilogues, TMEM release) and return, so that
b2x_check_device reports B2X_ERR_TIMEOUT and the CUDA context stays usable:
the next GEMM, with the hook off, is correct."""
import ctypes

import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu


def test_withheld_commit_times_out_and_context_survives():
    import b2x
    from b2x import _lib as L
    g = torch.Generator(device="cuda").manual_seed(0)
    A, sa = b2x.quantize(torch.randn((512, 512), device="cuda", generator=g), "tensor", torch.float8_e4m3fn)
    W, sw = b2x.quantize(torch.randn((512, 512), device="cuda", generator=g), "tensor", torch.float8_e4m3fn)
    torch.cuda.synchronize()
    assert b2x.read_device_status() == 0
    try:
        L.check(L.lib().b2x_debug_inject(1, 1_000_000))
        before = b2x.launch_count()
        b2x.matmul(A, W.t(), {"NUM_CTAS": 2}, scale_a=sa, scale_b=sw)
        torch.cuda.synchronize()  # returns: the kernel unwound instead of hanging
        assert b2x.launch_count() == before + 1
        assert L.lib().b2x_check_device() == L.ERR_TIMEOUT
        assert "epilogue" in L.lib().b2x_last_error().decode()
        assert b2x.read_device_status() == 0  # the check cleared the word
    finally:
        L.check(L.lib().b2x_debug_inject(0, 0))
    # same GEMM, hook off: correct result and a clean status word
    C = b2x.matmul(A, W.t(), {"NUM_CTAS": 2}, scale_a=sa, scale_b=sw)
    torch.cuda.synchronize()
    b2x.check_device()
    a_bits = A.view(torch.uint8).cpu().numpy()
    b_bits = W.view(torch.uint8).cpu().numpy().T
    ref = O.gemm(a_bits, b_bits, scale_mode="tensor", scale_a=sa.item(), scale_b=sw.item())
    err, tol = O.gemm_error(C.float().cpu().numpy(), ref, O.fp8_bits_to_f64(a_bits, O.E4M3) * sa.item(),
                            O.fp8_bits_to_f64(b_bits, O.E4M3) * sw.item())
    assert err <= tol


def test_debug_inject_rejects_unknown_switch():
    from b2x import _lib as L
    assert L.lib().b2x_debug_inject(7, 0) == L.ERR_INVALID_ARG
