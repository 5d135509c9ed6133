"""ctypes loader for liboracle.so (the C restatement in fp8_oracle.c).
TEST INFRASTRUCTURE / TIMED CPU REFERENCE ONLY -- see fp8_oracle.py."""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PATH = os.path.join(HERE, "liboracle.so")
MODES = {"none": 0, "tensor": 1, "block1x128": 3, "block128x128": 4, "mx1x32": 5}
FMTS = {"e4m3": 0, "e5m2": 1}
_lib = None


def build():
    subprocess.run(["make", "-C", HERE], check=True, stdout=subprocess.DEVNULL)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(PATH):
            build()
        L = ctypes.CDLL(PATH)
        L.oracle_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.oracle_quantize.restype = ctypes.c_int
        L.oracle_gemm_bf16.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_float, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int]
        L.oracle_gemm_bf16.restype = ctypes.c_double
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_stoch_round.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                         ctypes.c_void_p]
        L.oracle_stoch_round.restype = None
        _lib = L
    return _lib


def quantize(x, mode, fmt, nthreads=0):
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    R, C = x.shape
    q = np.empty((R, C), np.uint8)
    if mode in ("none", "tensor"):
        s = np.zeros(1, np.float32)
    elif mode == "block1x128":
        s = np.zeros((R, -(-C // 128)), np.float32)
    elif mode == "mx1x32":
        s = np.zeros((R, -(-C // 32)), np.uint8)
    else:
        s = np.zeros((-(-R // 128), -(-C // 128)), np.float32)
    rc = lib().oracle_quantize(x.ctypes.data, R, C, FMTS[fmt], MODES[mode], q.ctypes.data, s.ctypes.data, nthreads)
    assert rc == 0
    return q, (None if mode == "none" else (s[0] if mode == "tensor" else s))


def gemm_bf16(a_bits, bt_bits, a_fmt, b_fmt, sa, sb, rows=None, cols=None, nthreads=0):
    """bf16 bits of C = sa*sb*(A . Bt^T) on rows x cols (default: everything)."""
    a_bits = np.ascontiguousarray(a_bits, np.uint8)
    bt_bits = np.ascontiguousarray(bt_bits, np.uint8)
    M, K = a_bits.shape
    N = bt_bits.shape[0]
    m0, m1 = rows if rows else (0, M)
    n0, n1 = cols if cols else (0, N)
    c = np.zeros((M, N), np.uint16)
    flops = lib().oracle_gemm_bf16(a_bits.ctypes.data, K, FMTS[a_fmt], bt_bits.ctypes.data, K, FMTS[b_fmt], K,
                                   float(sa), float(sb), c.ctypes.data, N, m0, m1, n0, n1, nthreads)
    return c, flops


def max_threads():
    return lib().oracle_max_threads()


SR_FMTS = {"e4m3": 0, "e5m2": 1, "f16": 2, "bf16": 3}


def stoch_round(x, r, fmt):
    """Codes of the stochastic rounding of float32 x with uint32 entropy r."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    r = np.ascontiguousarray(r, np.uint32).reshape(-1)
    out = np.empty(x.size, np.uint8 if fmt in ("e4m3", "e5m2") else np.uint16)
    lib().oracle_stoch_round(x.ctypes.data, r.ctypes.data, x.size, SR_FMTS[fmt], out.ctypes.data)
    return out
