"""Torch-facing ops over the libb2x C ABI, registered as torch custom ops
(`torch.ops.b2x.quantize`, `torch.ops.b2x.fp8_gemm`, `torch.ops.b2x.reduce_k`).

Torch is used here only for device memory, the current stream and the op
registry.  All arithmetic happens in the sm_100a kernels of libb2x.so.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional, Sequence

import torch

from . import _lib as L

FP8_DTYPES = {torch.float8_e4m3fn: L.E4M3, torch.float8_e5m2: L.E5M2}
IN_DTYPES = {torch.float32: L.F32, torch.bfloat16: L.BF16}
OUT_DTYPES = {torch.bfloat16: L.BF16, torch.float16: L.F16}
CAST_MODES = {
    "none": L.SCALE_NONE,
    "tensor": L.SCALE_TENSOR,
    "given": L.SCALE_TENSOR_GIVEN,
    "block1x128": L.SCALE_BLOCK_1x128,
    "block128x128": L.SCALE_BLOCK_128x128,
    "mx1x32": L.SCALE_MX_1x32,
}
GEMM_SCALE_MODES = {"none": L.SCALE_NONE, "tensor": L.SCALE_TENSOR, "block": L.SCALE_BLOCK_1x128,
                    "mx": L.SCALE_MX_1x32}
CONFIG_FIELDS = ("block_m", "block_n", "block_k", "group_size_m", "num_smem_buffers", "num_tmem_buffers",
                 "num_mma_groups", "epilogue_subtile", "num_ctas", "split_k", "interleave_epilogue", "num_sms")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("b2x ops take CUDA tensors only (there is no CPU path)")


# ----------------------------------------------------------------------------
# Workspaces.  Split-K workspaces must be all-zero before a call and are
# returned all-zero by every successful call, so one zeroed buffer per
# (device, stream) is reused; it is dropped after any failed call and
# whenever the device status word reports a kernel that gave up a wait (its
# partial sums and tile counters may be left nonzero).

_ws_lock = threading.Lock()
_ws_cache: dict = {}


def _workspace(dev: torch.device, nbytes: int, zeroed: bool) -> torch.Tensor:
    key = (dev.index, _stream(dev), zeroed)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
            _ws_cache[key] = buf
        return buf


def _drop_workspaces(_status: int = 0) -> None:
    with _ws_lock:
        _ws_cache.clear()


L._status_hooks.append(_drop_workspaces)


# ----------------------------------------------------------------------------
# quantize


def _scale_shape(mode: str, R: int, C: int):
    if mode in ("tensor", "given"):
        return (1,), torch.float32
    if mode == "block1x128":
        return (R, -(-C // 128)), torch.float32
    if mode == "block128x128":
        return (-(-R // 128), -(-C // 128)), torch.float32
    if mode == "mx1x32":
        return (R, -(-C // 32)), torch.uint8
    return (0,), torch.float32


@torch.library.custom_op("b2x::quantize", mutates_args=())
def quantize_op(x: torch.Tensor, mode: str, fp8_dtype: torch.dtype,
                scale: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32/bf16 [R, C] -> (fp8 [R, C], scales); see include/b2x.h b2x_fp8_cast."""
    _require_cuda(x, scale)
    if mode not in CAST_MODES:
        raise ValueError(f"unknown quantize mode {mode!r}; expected one of {sorted(CAST_MODES)}")
    if x.dtype not in IN_DTYPES:
        raise TypeError(f"quantize input must be float32 or bfloat16, got {x.dtype}")
    if fp8_dtype not in FP8_DTYPES:
        raise TypeError(f"quantize output must be float8_e4m3fn or float8_e5m2, got {fp8_dtype}")
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    if x2.dim() != 2:
        x2 = x2.reshape(-1, x2.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    R, C = x2.shape
    q = torch.empty((R, C), dtype=fp8_dtype, device=x.device)
    sshape, sdt = _scale_shape(mode, R, C)
    if mode == "given":
        if scale is None:
            raise ValueError("mode 'given' needs a scale tensor")
        sc = scale.to(torch.float32).reshape(1).clone()  # a custom op may not return an alias of an input
    else:
        sc = torch.empty(sshape, dtype=sdt, device=x.device)
    a = L.CastArgs()
    a.x, a.x_type, a.rows, a.cols, a.ld_x = x2.data_ptr(), IN_DTYPES[x.dtype], R, C, x2.stride(0)
    a.q, a.q_type, a.ld_q = q.data_ptr(), FP8_DTYPES[fp8_dtype], C
    a.scale = sc.data_ptr() if sc.numel() else None
    a.mode = CAST_MODES[mode]
    a.ld_scale = sc.shape[1] if sc.dim() == 2 else 1
    lib = L.lib()
    nws = lib.b2x_cast_workspace_size(ctypes.byref(a))
    if nws:
        ws = _workspace(x.device, nws, zeroed=False)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(x.device):
        L.check(lib.b2x_fp8_cast(ctypes.byref(a), ctypes.c_void_p(_stream(x.device))))
    return q.reshape(x.shape), sc


@quantize_op.register_fake
def _(x, mode, fp8_dtype, scale=None):
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 1 else x.reshape(1, -1)
    sshape, sdt = _scale_shape(mode, x2.shape[0], x2.shape[1])
    return torch.empty_like(x, dtype=fp8_dtype), x.new_empty(sshape, dtype=sdt)


def amax(x: torch.Tensor) -> torch.Tensor:
    """NaN-ignoring max |x| on the GPU (one fp32 element)."""
    _require_cuda(x)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    a = L.CastArgs()
    a.rows, a.cols, a.ld_x, a.ld_q, a.mode = x2.shape[0], x2.shape[1], x2.stride(0), x2.stride(0), L.SCALE_TENSOR
    lib = L.lib()
    ws = _workspace(x.device, lib.b2x_cast_workspace_size(ctypes.byref(a)), zeroed=False)
    with torch.cuda.device(x.device):
        L.check(lib.b2x_amax(x2.data_ptr(), IN_DTYPES[x.dtype], x2.shape[0], x2.shape[1], x2.stride(0),
                             out.data_ptr(), ws.data_ptr(), ws.numel(), ctypes.c_void_p(_stream(x.device))))
    return out


# ----------------------------------------------------------------------------
# GEMM


def _gemm_args(a, b, c, scale_mode, scale_a, scale_b, config: Sequence[int]) -> L.GemmArgs:
    M, K = a.shape
    K2, N = b.shape
    g = L.GemmArgs()
    g.a, g.b, g.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    g.M, g.N, g.K = M, N, K
    g.lda = a.stride(0)
    sk, sn = b.stride()
    if sk == 1 and (sn != 1 or N == 1):
        g.ldb_k, g.ldb_n = 1, (sn if N > 1 else max(K, 16))
    else:
        g.ldb_k, g.ldb_n = (sk if K > 1 else max(N, 16)), sn
    g.ldc = c.stride(0)
    g.a_type, g.b_type, g.c_type = FP8_DTYPES[a.dtype], FP8_DTYPES[b.dtype], OUT_DTYPES[c.dtype]
    g.scale_mode = GEMM_SCALE_MODES[scale_mode]
    if scale_a is not None:
        g.scale_a = scale_a.data_ptr()
        if scale_a.dim() == 2:
            g.sa_stride_m, g.sa_stride_k = scale_a.stride()
    if scale_b is not None:
        g.scale_b = scale_b.data_ptr()
        if scale_mode == "mx":  # [N, K/32] bytes: row stride along N
            g.sb_stride_n, g.sb_stride_k = scale_b.stride()
        elif scale_b.dim() == 2:
            g.sb_stride_k, g.sb_stride_n = scale_b.stride()
    for name, v in zip(CONFIG_FIELDS, config):
        setattr(g.config, name, int(v))
    return g


def _tma_friendly(a: torch.Tensor, b: torch.Tensor):
    """TMA descriptors need 16-byte aligned bases and row pitches.  Operands
    that miss this (K or N not a multiple of 16, odd views) are copied once
    into zero-padded buffers; the padding adds zero products only."""
    M, K = a.shape
    N = b.shape[1]
    k16 = -(-K // 16) * 16
    a_ok = a.stride(1) == 1 and a.stride(0) % 16 == 0 and a.data_ptr() % 16 == 0 and K % 16 == 0
    if not a_ok:
        ap = torch.zeros((M, k16), dtype=a.dtype, device=a.device)
        ap[:, :K] = a
        a = ap
    sk, sn = b.stride()
    kmajor = sk == 1 and (sn != 1 or N == 1)
    if kmajor:
        b_ok = sn % 16 == 0 and b.data_ptr() % 16 == 0 and K % 16 == 0
    else:
        b_ok = sn == 1 and sk % 16 == 0 and b.data_ptr() % 16 == 0 and K % 16 == 0
    if not b_ok:
        # store as an [N, K16] K-major weight (the layout the kernel streams best)
        bp = torch.zeros((N, k16), dtype=b.dtype, device=b.device)
        bp[:, :K] = b.t()
        b = bp.t()
    return a, b


@torch.library.custom_op("b2x::fp8_gemm", mutates_args=())
def fp8_gemm_op(a: torch.Tensor, b: torch.Tensor, scale_a: Optional[torch.Tensor], scale_b: Optional[torch.Tensor],
                scale_mode: str, out_dtype: torch.dtype, config: list[int]) -> torch.Tensor:
    """C[M,N] = scaled fp8 A[M,K] @ B[K,N]; see include/b2x.h b2x_fp8_gemm."""
    _require_cuda(a, b, scale_a, scale_b)
    if a.dtype not in FP8_DTYPES or b.dtype not in FP8_DTYPES:
        raise TypeError(f"fp8_gemm takes float8 A and B, got {a.dtype} and {b.dtype}")
    if out_dtype not in OUT_DTYPES:
        raise TypeError(f"fp8_gemm output must be bfloat16 or float16, got {out_dtype}")
    M, K = a.shape
    N = b.shape[1]
    if M == 0 or N == 0:
        return torch.empty((M, N), dtype=out_dtype, device=a.device)
    a, b = _tma_friendly(a, b)
    # TMA needs 16-byte row pitches: give C a padded pitch when N % 8 != 0.
    n8 = -(-N // 8) * 8
    c = torch.empty((M, n8), dtype=out_dtype, device=a.device)[:, :N]
    g = _gemm_args(a, b, c, scale_mode, scale_a, scale_b, config)
    lib = L.lib()
    with torch.cuda.device(a.device):
        nws = lib.b2x_gemm_workspace_size(ctypes.byref(g))
        if nws:
            ws = _workspace(a.device, nws, zeroed=scale_mode != "mx")  # MX: scratch for tiled scales
            g.workspace, g.workspace_bytes = ws.data_ptr(), ws.numel()
        st = lib.b2x_fp8_gemm(ctypes.byref(g), ctypes.c_void_p(_stream(a.device)))
        if st != L.OK:
            _drop_workspaces()
        L.check(st)
    return c


# Cached launch plans: the ABI struct, padded C pitch and workspace size per
# call signature, so a repeated GEMM costs one struct copy and one C call on
# the host (the custom-op dispatcher is bypassed outside torch.compile).
_plans: dict = {}


def fp8_gemm_fast(a: torch.Tensor, b: torch.Tensor, scale_a: Optional[torch.Tensor], scale_b: Optional[torch.Tensor],
                  scale_mode: str, out_dtype: torch.dtype, config: tuple) -> torch.Tensor:
    """Same as torch.ops.b2x.fp8_gemm with a per-signature host plan."""
    key = (a.shape, a.stride(), b.shape, b.stride(), a.dtype, b.dtype, a.device, scale_mode, out_dtype, config,
           None if scale_a is None else scale_a.stride(), None if scale_b is None else scale_b.stride(),
           a.data_ptr() % 16, b.data_ptr() % 16)
    plan = _plans.get(key)
    if plan is None:
        if (not a.is_cuda or not b.is_cuda or a.dtype not in FP8_DTYPES or b.dtype not in FP8_DTYPES
                or out_dtype not in OUT_DTYPES or a.shape[0] == 0 or b.shape[1] == 0):
            return fp8_gemm_op(a, b, scale_a, scale_b, scale_mode, out_dtype, list(config))
        a2, b2 = _tma_friendly(a, b)
        if a2 is not a or b2 is not b:  # needs padded copies: not a plain launch
            return fp8_gemm_op(a, b, scale_a, scale_b, scale_mode, out_dtype, list(config))
        M, N = a.shape[0], b.shape[1]
        n8 = -(-N // 8) * 8
        c = torch.empty((M, n8), dtype=out_dtype, device=a.device)[:, :N]
        g = _gemm_args(a, b, c, scale_mode, scale_a, scale_b, config)
        with torch.cuda.device(a.device):
            nws = L.lib().b2x_gemm_workspace_size(ctypes.byref(g))
        plan = (bytes(g), nws, M, N, n8)
        if len(_plans) > 4096:
            _plans.clear()
        _plans[key] = plan
    raw, nws, M, N, n8 = plan
    c = torch.empty((M, n8), dtype=out_dtype, device=a.device)
    if n8 != N:
        c = c[:, :N]
    g = L.GemmArgs.from_buffer_copy(raw)
    g.a, g.b, g.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    if scale_a is not None:
        g.scale_a = scale_a.data_ptr()
    if scale_b is not None:
        g.scale_b = scale_b.data_ptr()
    dev = a.device
    lib = L.lib()
    if dev.index != torch.cuda.current_device():
        with torch.cuda.device(dev):
            return fp8_gemm_fast(a, b, scale_a, scale_b, scale_mode, out_dtype, config)
    if nws:
        ws = _workspace(dev, nws, zeroed=scale_mode != "mx")
        g.workspace, g.workspace_bytes = ws.data_ptr(), ws.numel()
    st = lib.b2x_fp8_gemm(ctypes.byref(g), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    if st != L.OK:
        _drop_workspaces()
        L.check(st)
    return c


def fp8_gemm_clc(a: torch.Tensor, b: torch.Tensor, scale_a: Optional[torch.Tensor], scale_b: Optional[torch.Tensor],
                 scale_mode: str, out_dtype: torch.dtype, config: Sequence[int]) -> torch.Tensor:
    """The same GEMM on single-CTA tiles scheduled by cluster launch control
    (include/b2x.h b2x_fp8_gemm_clc)."""
    _require_cuda(a, b, scale_a, scale_b)
    if a.dtype not in FP8_DTYPES or b.dtype not in FP8_DTYPES:
        raise TypeError(f"fp8_gemm_clc takes float8 A and B, got {a.dtype} and {b.dtype}")
    if scale_mode not in ("none", "tensor"):
        raise ValueError("the CLC-scheduled GEMM takes per-tensor scales or none")
    M, K = a.shape
    N = b.shape[1]
    if M == 0 or N == 0:
        return torch.empty((M, N), dtype=out_dtype, device=a.device)
    a, b = _tma_friendly(a, b)
    n8 = -(-N // 8) * 8
    c = torch.empty((M, n8), dtype=out_dtype, device=a.device)[:, :N]
    g = _gemm_args(a, b, c, scale_mode, scale_a, scale_b, config)
    g.config.num_ctas = 1
    lib = L.lib()
    with torch.cuda.device(a.device):
        nws = lib.b2x_gemm_workspace_size(ctypes.byref(g))
        if nws:
            ws = _workspace(a.device, nws, zeroed=True)
            g.workspace, g.workspace_bytes = ws.data_ptr(), ws.numel()
        st = lib.b2x_fp8_gemm_clc(ctypes.byref(g), ctypes.c_void_p(_stream(a.device)))
        if st != L.OK:
            _drop_workspaces()
        L.check(st)
    return c


@fp8_gemm_op.register_fake
def _(a, b, scale_a, scale_b, scale_mode, out_dtype, config):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype)


def gemm_config(a: torch.Tensor, b: torch.Tensor, scale_mode: str = "tensor",
                config: Sequence[int] = ()) -> dict:
    """The configuration libb2x picks for this problem (all fields filled)."""
    c = torch.empty((1, 1), dtype=torch.bfloat16, device=a.device)
    g = _gemm_args(a, b, c, scale_mode, None, None, tuple(config) + (0,) * (len(CONFIG_FIELDS) - len(config)))
    g.M, g.N = a.shape[0], b.shape[1]
    out = L.GemmConfig()
    L.check(L.lib().b2x_gemm_default_config(ctypes.byref(g), ctypes.byref(out)))
    return {n: getattr(out, n) for n in CONFIG_FIELDS}


@torch.library.custom_op("b2x::reduce_k", mutates_args=("c",))
def reduce_k_op(workspace: torch.Tensor, c: torch.Tensor, M: int, N: int, SPLIT_K: int) -> None:
    """c = cast(sum over SPLIT_K planes of workspace[(SPLIT_K*M), N]) (fp32 sum)."""
    _require_cuda(workspace, c)
    dt = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.float16: L.F16}
    if workspace.dtype not in dt or c.dtype not in dt:
        raise TypeError("reduce_k supports float32 / bfloat16 / float16")
    if workspace.numel() < SPLIT_K * M * N or not workspace.is_contiguous():
        raise ValueError("workspace must be a contiguous (SPLIT_K*M, N) tensor")
    if c.stride(-1) != 1:
        raise ValueError("c must have unit column stride")
    with torch.cuda.device(c.device):
        L.check(L.lib().b2x_splitk_reduce(workspace.data_ptr(), dt[workspace.dtype], c.data_ptr(), dt[c.dtype],
                                          M, N, c.stride(0), SPLIT_K, ctypes.c_void_p(_stream(c.device))))


def quantize(x: torch.Tensor, mode: str = "tensor", dtype: torch.dtype = torch.float8_e4m3fn,
             scale: Optional[torch.Tensor] = None):
    """Quantize fp32/bf16 to fp8. Returns (q, scale) -- scale is None for mode 'none'."""
    q, sc = torch.ops.b2x.quantize(x, mode, dtype, scale)
    return q, (None if mode == "none" else sc)


# ----------------------------------------------------------------------------
# stochastic rounding

SR_DTYPES = {torch.float8_e4m3fn: L.E4M3, torch.float8_e5m2: L.E5M2, torch.float16: L.F16,
             torch.bfloat16: L.BF16}


@torch.library.custom_op("b2x::stoch_round", mutates_args=())
def stoch_round_op(src: torch.Tensor, dst_dtype: torch.dtype, rand_bits: torch.Tensor,
                   rounding: str = "rs") -> torch.Tensor:
    """fp32 -> e4m3 / e5m2 / fp16 / bf16 with caller-given entropy;
    rounding "rs" (b2x_stoch_round_rs) or "exact32" (b2x_stoch_round)."""
    if rounding not in ("rs", "exact32"):
        raise ValueError(f"rounding must be 'rs' or 'exact32', got {rounding!r}")
    _require_cuda(src, rand_bits)
    if src.dtype != torch.float32:
        raise TypeError(f"stoch_round takes a float32 source, got {src.dtype}")
    if dst_dtype not in SR_DTYPES:
        raise TypeError(f"stoch_round targets float8_e4m3fn, float8_e5m2, float16 or bfloat16, got {dst_dtype}")
    if rand_bits.shape != src.shape:
        raise ValueError(f"rand_bits shape {tuple(rand_bits.shape)} must match src shape {tuple(src.shape)}")
    if rand_bits.dtype not in (torch.int32, torch.uint32):
        raise TypeError(f"rand_bits must be a 32-bit integer tensor, got {rand_bits.dtype}")
    shape = src.shape
    x = src.reshape(1, -1) if src.dim() <= 1 else src.reshape(-1, shape[-1])
    r = rand_bits.reshape(1, -1) if rand_bits.dim() <= 1 else rand_bits.reshape(-1, shape[-1])
    if x.stride(-1) != 1:
        x = x.contiguous()
    if r.stride(-1) != 1:
        r = r.contiguous()
    R, C = x.shape
    y = torch.empty((R, C), dtype=dst_dtype, device=src.device)
    if R * C:
        with torch.cuda.device(src.device):
            fn = L.lib().b2x_stoch_round_rs if rounding == "rs" else L.lib().b2x_stoch_round
            L.check(fn(x.data_ptr(), R, C, x.stride(0), r.data_ptr(), r.stride(0), y.data_ptr(), SR_DTYPES[dst_dtype],
                       C, ctypes.c_void_p(_stream(src.device))))
    return y.reshape(shape)


@stoch_round_op.register_fake
def _(src, dst_dtype, rand_bits, rounding="rs"):
    return src.new_empty(src.shape, dtype=dst_dtype)


def stoch_round(src: torch.Tensor, dst_ty: torch.dtype, rand_bits: torch.Tensor, *,
                rounding: str = "rs") -> torch.Tensor:
    """Stochastic rounding of float32 `src` to `dst_ty` (the reference's
    tlx.stoch_round(src, dst_ty, rand_bits), extensions/utlx/tlx/language/
    tlx/utility.py:113-153).  rand_bits has src's shape.

    rounding="rs" (default): the hardware `cvt.rs.satfinite` the reference
    lowers to; packs of 4 (fp8) / 2 (16-bit) consecutive elements of a row
    share the rand_bits word of the pack's first element.
    rounding="exact32": b2x's integer rule, every element rounds up with
    probability frac/2^32 from its own full word (bit-exact CPU oracle).
    Same-dtype requests return `src` unchanged, as the reference does."""
    if dst_ty == src.dtype:
        return src
    return torch.ops.b2x.stoch_round(src, dst_ty, rand_bits, rounding)


# ----------------------------------------------------------------------------
# grouped GEMM

def grouped_gemm(group_A: Sequence[torch.Tensor], group_B: Sequence[torch.Tensor],
                 scales_a: Optional[Sequence[torch.Tensor]] = None, scales_b: Optional[Sequence[torch.Tensor]] = None,
                 out_dtype: torch.dtype = torch.bfloat16, block_n: int = 0) -> list:
    """[A_g (M_g, K_g) fp8] x [B_g (N_g, K_g) fp8 weights] -> [C_g (M_g, N_g)] in one launch
    (include/b2x.h b2x_fp8_grouped_gemm; the reference's group_gemm_tlx_fn,
    blackwell-grouped-gemm_test.py:727-784, takes B as [N, K] the same way).
    Optional per-tensor scales per group: C_g = sA_g * sB_g * A_g . B_g^T."""
    if len(group_A) != len(group_B):
        raise ValueError("group_A and group_B differ in length")
    if (scales_a is None) != (scales_b is None):
        raise ValueError("pass both scale lists or neither")
    n = len(group_A)
    if n == 0:
        return []
    _require_cuda(*group_A, *group_B)
    dev = group_A[0].device
    a_dt, b_dt = group_A[0].dtype, group_B[0].dtype
    if a_dt not in FP8_DTYPES or b_dt not in FP8_DTYPES:
        raise TypeError(f"grouped_gemm takes float8 operands, got {a_dt} x {b_dt}")
    if out_dtype not in OUT_DTYPES:
        raise TypeError(f"grouped_gemm output must be bfloat16 or float16, got {out_dtype}")
    arr = (L.GemmGroup * n)()
    outs, keep = [], []
    for i, (A, B) in enumerate(zip(group_A, group_B)):
        if A.dtype != a_dt or B.dtype != b_dt or A.device != dev or B.device != dev:
            raise TypeError("all groups must share operand dtypes and device")
        if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
            raise ValueError(f"group {i}: A {tuple(A.shape)} and B {tuple(B.shape)} are not [M, K] and [N, K]")
        M, K = A.shape
        N = B.shape[0]
        if A.stride(1) != 1 or A.stride(0) % 16 or A.data_ptr() % 16:
            A = _pad_k(A)
        if B.stride(1) != 1 or B.stride(0) % 16 or B.data_ptr() % 16:
            B = _pad_k(B)
        n8 = -(-N // 8) * 8
        C = torch.empty((M, n8), dtype=out_dtype, device=dev)[:, :N]
        keep += [A, B]
        outs.append(C)
        g = arr[i]
        g.a, g.b, g.c = A.data_ptr(), B.data_ptr(), C.data_ptr()
        g.M, g.N, g.K = M, N, K
        g.lda, g.ldb, g.ldc = A.stride(0), B.stride(0), C.stride(0)
        if scales_a is not None:
            sa = scales_a[i].to(torch.float32).reshape(1)
            sb = scales_b[i].to(torch.float32).reshape(1)
            keep += [sa, sb]
            g.scale_a, g.scale_b = sa.data_ptr(), sb.data_ptr()
    lib = L.lib()
    with torch.cuda.device(dev):
        nws = lib.b2x_grouped_gemm_workspace_size(n)
        ws = _workspace(dev, nws + 64, zeroed=False)
        base = ws.data_ptr()
        off = (-base) % 64
        L.check(lib.b2x_fp8_grouped_gemm(arr, n, FP8_DTYPES[a_dt], FP8_DTYPES[b_dt], OUT_DTYPES[out_dtype], block_n,
                                         base + off, ws.numel() - off, ctypes.c_void_p(_stream(dev))))
    return outs


def _pad_k(t: torch.Tensor) -> torch.Tensor:
    """Copy into a row-major buffer with a 16-element-aligned row pitch."""
    R, K = t.shape
    k16 = -(-K // 16) * 16
    out = torch.zeros((R, k16), dtype=t.dtype, device=t.device)
    out[:, :K] = t
    return out[:, :K]


# ----------------------------------------------------------------------------
# gate+up GEMM fused with SwiGLU and fp8 quantization

def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[I, K] gate and up weights -> the [2I, K] weight gemm_swiglu expects:
    gate rows 128j..128j+127, then up rows 128j..128j+127, for each j."""
    if w_gate.shape != w_up.shape or w_gate.shape[0] % 128:
        raise ValueError("gate and up weights must have the same [I, K] shape with I % 128 == 0")
    I, K = w_gate.shape
    return torch.stack([w_gate.reshape(I // 128, 128, K), w_up.reshape(I // 128, 128, K)], dim=1).reshape(2 * I, K)


def gemm_swiglu(x: torch.Tensor, w_gu: torch.Tensor, scale_x: Optional[torch.Tensor] = None,
                scale_w: Optional[torch.Tensor] = None, mode: str = "block1x128",
                h_scale: Optional[torch.Tensor] = None, h_dtype: torch.dtype = torch.float8_e4m3fn,
                h_amax: Optional[torch.Tensor] = None):
    """h = fp8(silu(x . gate^T) * (x . up^T)) for the interleaved weight w_gu
    [2I, K] (interleave_gate_up); see include/b2x.h b2x_fp8_gemm_swiglu.
    mode "block1x128": returns (h [M, I], scales [M, I/128]);
    mode "mx1x32": returns (h [M, I], E8M0 uint8 scales [M, I/32]) for an MX down projection;
    mode "given": h_scale (one fp32) is used, returns (h, h_scale); if h_amax
    (one fp32, zeroed by the caller) is given, max |h| is accumulated into it."""
    _require_cuda(x, w_gu, scale_x, scale_w, h_scale, h_amax)
    if x.dtype not in FP8_DTYPES or w_gu.dtype not in FP8_DTYPES or h_dtype not in FP8_DTYPES:
        raise TypeError("gemm_swiglu takes float8 operands and produces float8 h")
    if mode not in ("block1x128", "mx1x32", "given"):
        raise ValueError(f"mode must be 'block1x128', 'mx1x32' or 'given', got {mode!r}")
    M, K = x.shape
    N = w_gu.shape[0]
    I = N // 2
    b = w_gu.t()
    x, b = _tma_friendly(x, b)
    h = torch.empty((M, -(-I // 16) * 16), dtype=h_dtype, device=x.device)[:, :I]
    if mode == "block1x128":
        sc = torch.empty((M, I // 128 if I % 128 == 0 else I // 128 + 1), dtype=torch.float32, device=x.device)
        ld_sc, smode = sc.stride(0), L.SCALE_BLOCK_1x128
    elif mode == "mx1x32":
        if I % 128:
            raise ValueError("mode 'mx1x32' needs I = N/2 to be a multiple of 128")
        sc = torch.empty((M, I // 32), dtype=torch.uint8, device=x.device)
        ld_sc, smode = sc.stride(0), L.SCALE_MX_1x32
    else:
        if h_scale is None:
            raise ValueError("mode 'given' needs h_scale")
        sc = h_scale.to(torch.float32).reshape(1)
        ld_sc, smode = 1, L.SCALE_TENSOR_GIVEN
    sm = "none" if scale_x is None else "tensor"
    c = torch.empty((1, 8), dtype=torch.bfloat16, device=x.device)
    g = _gemm_args(x, b, c, sm, scale_x, scale_w, (0,) * len(CONFIG_FIELDS))
    g.c, g.ldc = None, N
    with torch.cuda.device(x.device):
        L.check(L.lib().b2x_fp8_gemm_swiglu(ctypes.byref(g), h.data_ptr(), h.stride(0), FP8_DTYPES[h_dtype], smode,
                                            sc.data_ptr(), ld_sc, None if h_amax is None else h_amax.data_ptr(),
                                            ctypes.c_void_p(_stream(x.device))))
    return h, sc
