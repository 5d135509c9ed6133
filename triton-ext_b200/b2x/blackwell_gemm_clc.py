"""Drop-in counterpart of the reference's cluster-launch-control GEMM module
(extensions/utlx/tlx/tutorials/blackwell_gemm_clc.py), for fp8 operands.

    matmul(a, b, config=None)     (:281)

One CTA per output tile (per split with SPLIT_K > 1); a CTA starts with its
own tile and takes over the tiles of CTAs that have not launched yet through
clusterlaunchcontrol.try_cancel, as matmul_kernel_tma_ws_blackwell_clc
(:62-281) does.  The work runs in libb2x's single-CTA warp-specialized
kernel (include/b2x.h, b2x_fp8_gemm_clc).  Differences a caller sees are
those of blackwell_gemm_ws.matmul: fp8 inputs give a bfloat16 (or
`out_dtype`) C, and per-tensor scales are keyword-only arguments.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .blackwell_gemm_ws import _scale_mode, _to_b2x_config


def matmul(a, b, config=None, *, scale_a: Optional[torch.Tensor] = None, scale_b: Optional[torch.Tensor] = None,
           out_dtype: torch.dtype = torch.bfloat16):
    """C = (A . B) * sA * sB with A [M, K] and B [K, N] fp8 (:281-340)."""
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.is_contiguous(), "Matrix A must be contiguous"
    if a.dtype not in ops.FP8_DTYPES or b.dtype not in ops.FP8_DTYPES:
        raise NotImplementedError("b2x's CLC GEMM takes float8 operands (e4m3fn / e5m2)")
    mode = _scale_mode(scale_a, scale_b)
    if mode not in ("none", "tensor"):
        raise ValueError("the CLC-scheduled GEMM takes per-tensor scales or none")
    cfg = dict(config or {})
    cfg["NUM_CTAS"] = 1
    return ops.fp8_gemm_clc(a, b, scale_a, scale_b, mode, out_dtype, tuple(_to_b2x_config(cfg, a.shape[1])))
