"""ctypes binding of libb2x.so (the C ABI declared in include/b2x.h).

The library is built in-tree (`make -C triton-ext_b200/csrc`, or
`b2x.build()`); importing this module when it is missing raises -- there is
no CPU or Python fallback for any op.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb2x.so")
CSRC = os.path.join(os.path.dirname(_HERE), "csrc")

# b2x_status
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_WORKSPACE = range(6)
# b2x_dtype
F32, BF16, F16, E4M3, E5M2, U8 = range(6)
# b2x_scale_mode
SCALE_NONE, SCALE_TENSOR, SCALE_TENSOR_GIVEN, SCALE_BLOCK_1x128, SCALE_BLOCK_128x128, SCALE_MX_1x32 = range(6)

EXPORTED = (
    "b2x_cast_workspace_size", "b2x_fp8_cast", "b2x_amax", "b2x_gemm_default_config",
    "b2x_gemm_workspace_size", "b2x_fp8_gemm", "b2x_fp8_gemm_clc", "b2x_splitk_reduce", "b2x_last_error",
    "b2x_read_device_status", "b2x_check_device", "b2x_debug_inject", "b2x_abi_version", "b2x_launch_count", "b2x_fp8_gemm_splitk_noalloc",
    "b2x_trace_read", "b2x_allreduce_signal_words", "b2x_fp8_gemm_allreduce",
    "b2x_stoch_round", "b2x_stoch_round_rs", "b2x_grouped_gemm_workspace_size", "b2x_fp8_grouped_gemm", "b2x_fp8_gemm_swiglu",
)

AR_MAX_RANKS = 8
TRACE_SLOTS = 16  # counters per CTA returned by b2x_trace_read


class CastArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("x_type", ctypes.c_int),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("ld_x", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("q_type", ctypes.c_int), ("ld_q", ctypes.c_int64),
        ("scale", ctypes.c_void_p), ("mode", ctypes.c_int), ("ld_scale", ctypes.c_int64),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class GemmConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "block_m", "block_n", "block_k", "group_size_m", "num_smem_buffers", "num_tmem_buffers",
        "num_mma_groups", "epilogue_subtile", "num_ctas", "split_k", "interleave_epilogue", "num_sms")]


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p),
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
        ("lda", ctypes.c_int64), ("ldb_k", ctypes.c_int64), ("ldb_n", ctypes.c_int64), ("ldc", ctypes.c_int64),
        ("a_type", ctypes.c_int), ("b_type", ctypes.c_int), ("c_type", ctypes.c_int),
        ("scale_mode", ctypes.c_int),
        ("scale_a", ctypes.c_void_p), ("sa_stride_m", ctypes.c_int64), ("sa_stride_k", ctypes.c_int64),
        ("scale_b", ctypes.c_void_p), ("sb_stride_k", ctypes.c_int64), ("sb_stride_n", ctypes.c_int64),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("config", GemmConfig),
    ]


class AllReduceArgs(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_int), ("world", ctypes.c_int),
        ("c_multicast", ctypes.c_void_p), ("c_peers", ctypes.c_void_p * AR_MAX_RANKS),
        ("signal_multicast", ctypes.c_void_p), ("signal_peers", ctypes.c_void_p * AR_MAX_RANKS),
        ("epoch", ctypes.c_uint32),
    ]


class GemmGroup(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p),
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
        ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64),
        ("scale_a", ctypes.c_void_p), ("scale_b", ctypes.c_void_p),
    ]


class B2XError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b2x status {status}: {msg}")
        self.status = status


_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> str:
    """Compile libb2x.so for sm_100a with nvcc (make in the csrc directory)."""
    cmd = ["make", "-C", CSRC]
    if force:
        cmd.insert(1, "-B")
    subprocess.run(cmd, check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libb2x.so not found at {LIB_PATH}; build it with `make -C {CSRC}` "
                "(b2x has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.b2x_cast_workspace_size.argtypes = [ctypes.POINTER(CastArgs)]
        L.b2x_cast_workspace_size.restype = ctypes.c_size_t
        L.b2x_fp8_cast.argtypes = [ctypes.POINTER(CastArgs), ctypes.c_void_p]
        L.b2x_fp8_cast.restype = ctypes.c_int
        L.b2x_amax.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        L.b2x_amax.restype = ctypes.c_int
        L.b2x_gemm_default_config.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(GemmConfig)]
        L.b2x_gemm_default_config.restype = ctypes.c_int
        L.b2x_gemm_workspace_size.argtypes = [ctypes.POINTER(GemmArgs)]
        L.b2x_gemm_workspace_size.restype = ctypes.c_size_t
        L.b2x_fp8_gemm.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p]
        L.b2x_fp8_gemm.restype = ctypes.c_int
        L.b2x_fp8_gemm_clc.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p]
        L.b2x_fp8_gemm_clc.restype = ctypes.c_int
        L.b2x_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.b2x_trace_read.restype = ctypes.c_int
        L.b2x_fp8_gemm_swiglu.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                          ctypes.c_void_p]
        L.b2x_fp8_gemm_swiglu.restype = ctypes.c_int
        L.b2x_grouped_gemm_workspace_size.argtypes = [ctypes.c_int]
        L.b2x_grouped_gemm_workspace_size.restype = ctypes.c_size_t
        L.b2x_fp8_grouped_gemm.argtypes = [ctypes.POINTER(GemmGroup), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.c_void_p]
        L.b2x_fp8_grouped_gemm.restype = ctypes.c_int
        L.b2x_stoch_round.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p]
        L.b2x_stoch_round.restype = ctypes.c_int
        L.b2x_stoch_round_rs.argtypes = L.b2x_stoch_round.argtypes
        L.b2x_stoch_round_rs.restype = ctypes.c_int
        L.b2x_allreduce_signal_words.argtypes = [ctypes.c_int64, ctypes.c_int64]
        L.b2x_allreduce_signal_words.restype = ctypes.c_size_t
        L.b2x_fp8_gemm_allreduce.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(AllReduceArgs), ctypes.c_void_p]
        L.b2x_fp8_gemm_allreduce.restype = ctypes.c_int
        L.b2x_fp8_gemm_splitk_noalloc.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p]
        L.b2x_fp8_gemm_splitk_noalloc.restype = ctypes.c_int
        L.b2x_splitk_reduce.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                        ctypes.c_void_p]
        L.b2x_splitk_reduce.restype = ctypes.c_int
        L.b2x_last_error.argtypes = []
        L.b2x_last_error.restype = ctypes.c_char_p
        L.b2x_check_device.argtypes = []
        L.b2x_check_device.restype = ctypes.c_int
        L.b2x_debug_inject.argtypes = [ctypes.c_int, ctypes.c_uint64]
        L.b2x_debug_inject.restype = ctypes.c_int
        L.b2x_read_device_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
        L.b2x_read_device_status.restype = ctypes.c_int
        L.b2x_abi_version.argtypes = []
        L.b2x_abi_version.restype = ctypes.c_int
        L.b2x_launch_count.argtypes = []
        L.b2x_launch_count.restype = ctypes.c_uint64
        _lib = L
        return L


def check(status: int) -> None:
    if status != OK:
        msg = lib().b2x_last_error().decode(errors="replace")
        raise B2XError(status, msg)


def launch_count() -> int:
    return int(lib().b2x_launch_count())


def read_trace(max_ctas: int = 148):
    """Per-CTA wait-cycle counters of the GEMM kernels (see b2x_trace_read)."""
    import numpy as np
    buf = np.zeros((max_ctas, TRACE_SLOTS), np.uint64)
    n = ctypes.c_int(0)
    check(lib().b2x_trace_read(buf.ctypes.data, max_ctas, ctypes.byref(n)))
    return buf[: n.value]


# Called with the status whenever read_device_status() finds a kernel that
# gave up a bounded wait: state that such a kernel may have left half-updated
# (the cached split-K workspaces, for one) registers a hook to drop it.
_status_hooks: list = []


def check_device() -> None:
    """Raises B2XError(ERR_TIMEOUT) if a kernel gave up a bounded wait since
    the last read of the device status word (blocking; clears the word)."""
    v = ctypes.c_int(0)
    check(lib().b2x_read_device_status(ctypes.byref(v)))
    if v.value:
        for hook in list(_status_hooks):
            hook(v.value)
        raise B2XError(ERR_TIMEOUT, f"a kernel gave up a bounded wait (device status 0x{v.value:x})")


def read_device_status() -> int:
    """Reads and clears the current device's status word (blocking).  A
    nonzero value means a kernel gave up a bounded wait; the registered
    hooks then drop any state that kernel may have left dirty."""
    v = ctypes.c_int(0)
    check(lib().b2x_read_device_status(ctypes.byref(v)))
    if v.value:
        for hook in list(_status_hooks):
            hook(v.value)
    return v.value
