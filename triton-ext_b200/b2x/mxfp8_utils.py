"""Counterpart of the reference's fp8 quantize helpers
(extensions/utlx/tlx/language/tlx/mxfp8_utils.py), as host-callable ops that
run libb2x's sm_100a cast kernels on whole tensors.

    _compute_scale_and_quantize(data_block, VEC_SIZE, dtype) -> (scale_e8m0, data_fp8)   (:13-86)
    _to_mxfp8_block(data_input, data_out_tile, scale_out_tile, VEC_SIZE, dtype)          (:89-128)

`dtype` is torch.float8_e4m3fn / torch.float8_e5m2 (the reference's
tl.float8e4nv / tl.float8e5); the strings "e4m3" / "e5m2" are accepted too.
VEC_SIZE is 32 (one E8M0 scale per 1x32 group, rounded up to a power of two).
"""
from __future__ import annotations

import torch

from . import ops

_NAMES = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2,
          "float8e4nv": torch.float8_e4m3fn, "float8e5": torch.float8_e5m2}


def _fp8(dtype):
    if isinstance(dtype, str):
        dtype = _NAMES.get(dtype, dtype)
    if dtype not in (torch.float8_e4m3fn, torch.float8_e5m2):
        raise AssertionError(f"dtype must be float8_e4m3fn or float8_e5m2, got {dtype}")
    return dtype


def get_fp8_format_name(dtype) -> str:
    """'e4m3' or 'e5m2' (tlx.get_fp8_format_name, utility.py:92)."""
    return "e4m3" if _fp8(dtype) == torch.float8_e4m3fn else "e5m2"


def _compute_scale_and_quantize(data_block, VEC_SIZE, dtype):
    """Per-1xVEC_SIZE E8M0 scales (uint8 biased exponents) and fp8 data."""
    if VEC_SIZE != 32:
        raise AssertionError(f"VEC_SIZE must be 32 (MX block size), got {VEC_SIZE}")
    if data_block.dim() != 2:
        raise AssertionError("data_block must be 2-D [BLOCK_M, BLOCK_K]")
    q, sc = ops.quantize(data_block.to(torch.float32) if data_block.dtype not in (torch.float32, torch.bfloat16)
                         else data_block, "mx1x32", _fp8(dtype))
    return sc, q


def _to_mxfp8_block(data_input, data_out_tile, scale_out_tile, VEC_SIZE, dtype):
    """Quantize a [128, 128] tile and store data and scales into the given tensors."""
    if tuple(data_input.shape) != (128, 128) or VEC_SIZE != 32:
        raise AssertionError("_to_mxfp8_block takes a 128x128 tile with VEC_SIZE 32")
    sc, q = _compute_scale_and_quantize(data_input, VEC_SIZE, dtype)
    data_out_tile.copy_(q)
    scale_out_tile.copy_(sc.view(scale_out_tile.dtype) if scale_out_tile.dtype != sc.dtype else sc)
