"""b2x -- B200-native (sm_100a) fp8 GEMM, fp8 cast and split-K.

Host-side mirror of the reference's op-level API for this path
(imperatormk/triton-ext, µTLX tutorials):
    b2x.matmul(a, b, config=None, use_heuristic=False, *, scale_a, scale_b, out_dtype)
    b2x.quantize(x, mode, dtype)            fp32/bf16 -> fp8 with amax scales
    b2x.reduce_k(workspace, c, M, N, SPLIT_K)
    b2x.stoch_round(src, dst_ty, rand_bits)  fp32 -> fp8/fp16/bf16, stochastic rounding
    b2x.grouped_gemm(group_A, group_B)      a list of fp8 GEMMs in one launch
    b2x.gemm_swiglu(x, w_gu, sx, sw)        gate+up GEMM -> SwiGLU -> fp8 h in one kernel
    b2x.blackwell_gemm_ws / b2x.blackwell_gemm_clc / b2x.mxfp8_utils  modules with the reference's names
Every op runs in libb2x.so (hand-written CUDA for sm_100a) through its C ABI
(include/b2x.h); there is no CPU fallback.
"""
from . import _lib
from ._lib import B2XError, build, check_device, launch_count, read_device_status
from .ops import amax, quantize, gemm_config, stoch_round, grouped_gemm, gemm_swiglu, interleave_gate_up
from .blackwell_gemm_ws import matmul, reduce_k, get_heuristic_config
from . import blackwell_gemm_clc, blackwell_gemm_ws, mxfp8_utils

__all__ = ["matmul", "quantize", "reduce_k", "amax", "get_heuristic_config", "gemm_config", "stoch_round", "grouped_gemm", "gemm_swiglu", "interleave_gate_up",
           "blackwell_gemm_ws", "blackwell_gemm_clc", "mxfp8_utils", "B2XError", "build", "check_device", "launch_count", "read_device_status"]
