"""CPU oracle for the b2x fp8 path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (libb2x.so behind the `b2x` package) never calls
it and fails loudly when its CUDA library is missing.

It restates, in numpy integer/float32 arithmetic, the reference's quantize
recipe and its scaled fp8 GEMM:

* quantize -- `_compute_scale_and_quantize`
  (extensions/utlx/tlx/language/tlx/mxfp8_utils.py:37-84):
    amax  = max |x| per scale group, NaN-ignoring (tl.max, :49-50)
    scale = amax / FMAX                                  (:53)
    MX 1x32 only: scale rounded up to a power of two (RCEIL bit trick, :59-65),
                  stored as the biased exponent byte (:68)
    inv   = 0 if scale == 0 else 1 / scale               (:69)
    q     = fp8(clamp(x * inv, -FMAX, FMAX))             (:72-84)
  where `.to(fp8)` is round-to-nearest-even (Triton's default cast rounding,
  triton/language/semantic.py:809) and the symmetric tl.clamp with
  propagate_nan=NONE is, as a B200 computes it, copysign(fmin(|y|, FMAX), y):
  a NaN becomes +-FMAX by its sign bit; the fp32 multiply before it returns
  the canonical positive NaN, so in scaled modes every NaN (and Inf * 0)
  becomes +FMAX.  Divisions are IEEE fp32
  divisions and the multiply is a single rounded fp32 multiply.  The same
  recipe with one scale per tensor, per 1x128 row block or per 128x128 tile
  gives the other scale modes (the benchmark configurations; no reference test pins them).

* GEMM -- matmul of blackwell_gemm_ws.py:1352 on fp8 inputs with the scaled
  reference formula of test_async_dot_scaled (extensions/utlx/test/
  test_tlx.py:2426-2435): C = (A * sA) @ (B * sB), evaluated here in float64
  from the exactly-decoded fp8 values.

Pinning: the finite-value rounding is checked against torch's and
ml_dtypes' float8 conversions; NaN/Inf/ties/sign-of-zero behaviour of the
whole recipe is pinned by golden vectors produced on a B200 by a plain-Triton
restatement of the recipe (tests/golden/make_golden_triton.py).
"""
from __future__ import annotations

import numpy as np

E4M3 = "e4m3"
E5M2 = "e5m2"
FMAX = {E4M3: np.float32(448.0), E5M2: np.float32(57344.0)}

# ----------------------------------------------------------------------------
# fp32 -> fp8 bit patterns, round-to-nearest-even, saturate to max finite.


def f32_to_fp8_bits(x: np.ndarray, fmt: str) -> np.ndarray:
    """Encode float32 values to fp8 bytes (RNE, satfinite, NaN -> 0x7F|sign).

    Mirrors PTX `cvt.rn.satfinite.{e4m3x2,e5m2x2}.f32`: finite values beyond
    the largest finite fp8 value (and infinities) saturate to it.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    sign = ((u >> np.uint32(24)) & np.uint32(0x80)).astype(np.uint8)
    a = np.abs(x)
    ua = a.view(np.uint32).astype(np.uint64)
    if fmt == E4M3:
        mbits, bias, min_normal_exp, max_code, nan_code = 3, 7, -6, 0x7E, 0x7F
        big = a >= np.float32(448.0)
    elif fmt == E5M2:
        mbits, bias, min_normal_exp, max_code, nan_code = 2, 15, -14, 0x7B, 0x7F
        big = a >= np.float32(57344.0)
    else:
        raise ValueError(fmt)
    drop = 23 - mbits
    lsb = (ua >> np.uint64(drop)) & np.uint64(1)
    r = (ua + np.uint64((1 << (drop - 1)) - 1) + lsb) & ~np.uint64((1 << drop) - 1)
    e = (r >> np.uint64(23)).astype(np.int64) - 127 + bias
    m = ((r >> np.uint64(drop)) & np.uint64((1 << mbits) - 1)).astype(np.int64)
    normal_code = np.minimum((e << mbits) | m, max_code)
    # subnormal range: codes are a linear grid of step 2^(min_normal_exp - mbits)
    with np.errstate(invalid="ignore", over="ignore"):
        sub_val = np.rint(a.astype(np.float64) * float(2.0 ** (mbits - min_normal_exp)))
    sub = a < np.float32(2.0 ** min_normal_exp)
    sub_code = np.where(sub, sub_val, 0).astype(np.int64)
    code = np.where(sub, sub_code, normal_code)
    code = np.where(big, max_code, code)
    code = np.where(np.isnan(x), nan_code, code)
    return (code.astype(np.uint8) | sign).reshape(x.shape)


def _decode_table(fmt: str) -> np.ndarray:
    t = np.zeros(256, np.float64)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        if fmt == E4M3:
            e, m = (c >> 3) & 15, c & 7
            if e == 15 and m == 7:
                v = np.nan
            elif e == 0:
                v = m * 2.0 ** -9
            else:
                v = (1 + m / 8.0) * 2.0 ** (e - 7)
        else:
            e, m = (c >> 2) & 31, c & 3
            if e == 31:
                v = np.inf if m == 0 else np.nan
            elif e == 0:
                v = m * 2.0 ** -16
            else:
                v = (1 + m / 4.0) * 2.0 ** (e - 15)
        t[c] = s * v
    return t


DECODE = {E4M3: _decode_table(E4M3), E5M2: _decode_table(E5M2)}


def fp8_bits_to_f64(bits: np.ndarray, fmt: str) -> np.ndarray:
    return DECODE[fmt][np.asarray(bits, np.uint8)]


# ----------------------------------------------------------------------------
# The quantize recipe.


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def nan_ignoring_absmax(x: np.ndarray, axis=None) -> np.ndarray:
    a = np.abs(np.asarray(x, np.float32))
    a = np.where(np.isnan(a), np.float32(0.0), a)
    return a.max(axis=axis).astype(np.float32) if a.size else np.float32(0.0)


def _inv_scale(scale: np.ndarray) -> np.ndarray:
    scale = np.asarray(scale, np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(scale == 0, np.float32(0.0), np.float32(1.0) / scale)
    return inv.astype(np.float32)


def clamp_sym(y: np.ndarray, m) -> np.ndarray:
    """tl.clamp(y, -m, m) as a B200 computes it: NaN-ignoring min on |y|, sign
    bit of y kept -- so a NaN becomes +m or -m according to its sign bit."""
    return np.copysign(np.fmin(np.abs(y), m), y).astype(np.float32)


def _scaled_cast(x: np.ndarray, inv, fmt: str) -> np.ndarray:
    """clamp(x * inv) -> fp8.  inv=None means no multiply (mode "none").  The
    GPU's fp32 multiply returns the canonical positive NaN for every NaN
    result (x86 may return a negative one), so NaNs are made positive here."""
    m = FMAX[fmt]
    y = x.astype(np.float32)
    if inv is not None:
        with np.errstate(invalid="ignore", over="ignore"):
            y = (y * np.asarray(inv, np.float32)).astype(np.float32)
        y = np.where(np.isnan(y), np.float32(np.nan), y)
    return f32_to_fp8_bits(clamp_sym(y, m), fmt)


def quantize(x: np.ndarray, mode: str, fmt: str, scale: np.ndarray | float | None = None):
    """Quantize a 2-D float32 array.  Returns (q_bits uint8, scale).

    mode: "none" (scale 1), "tensor" (amax/FMAX), "given" (caller's scale),
    "block1x128", "block128x128" (fp32 scales), "mx1x32" (E8M0 bytes, RCEIL).
    """
    x = np.asarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    R, C = x.shape
    fm = FMAX[fmt]
    if mode == "none":
        return _scaled_cast(x, None, fmt), None
    if mode == "given":
        sc = np.float32(scale)
        return _scaled_cast(x, _inv_scale(sc), fmt), sc
    if mode == "tensor":
        sc = np.float32(nan_ignoring_absmax(x) / fm)
        return _scaled_cast(x, _inv_scale(sc), fmt), sc
    if mode in ("block1x128", "mx1x32"):
        G = 128 if mode == "block1x128" else 32
        nb = -(-C // G)
        pad = np.zeros((R, nb * G), np.float32)
        pad[:, :C] = x
        blocks = pad.reshape(R, nb, G)
        amax = nan_ignoring_absmax(blocks, axis=2)
        with np.errstate(over="ignore"):
            sc = (amax / fm).astype(np.float32)
        if mode == "mx1x32":
            e = (sc.view(np.uint32).astype(np.uint64) + 0x7FFFFF) & 0x7F800000
            rounded = e.astype(np.uint32).view(np.float32)
            inv = _inv_scale(rounded)
            out_scale = (e >> 23).astype(np.uint8)
        else:
            inv = _inv_scale(sc)
            out_scale = sc
        q = _scaled_cast(blocks, inv[:, :, None], fmt).reshape(R, nb * G)[:, :C]
        return np.ascontiguousarray(q), out_scale
    if mode == "block128x128":
        nr, nc = -(-R // 128), -(-C // 128)
        pad = np.zeros((nr * 128, nc * 128), np.float32)
        pad[:R, :C] = x
        t = pad.reshape(nr, 128, nc, 128).transpose(0, 2, 1, 3)
        amax = nan_ignoring_absmax(t.reshape(nr, nc, -1), axis=2)
        sc = (amax / fm).astype(np.float32)
        inv = _inv_scale(sc)
        q = _scaled_cast(t, inv[:, :, None, None], fmt).transpose(0, 2, 1, 3).reshape(nr * 128, nc * 128)
        return np.ascontiguousarray(q[:R, :C]), sc
    raise ValueError(mode)


# ----------------------------------------------------------------------------
# Scaled fp8 GEMM.


def gemm(a_bits, b_bits_kn, a_fmt=E4M3, b_fmt=E4M3, scale_mode="tensor", scale_a=None, scale_b=None):
    """float64 C[M,N] for fp8 A[M,K] and B[K,N] (bytes) with the given scales.

    scale_mode "none" | "tensor" (scalars) | "block" (sA[M, KB], sB[KB, NB],
    one scale per 128-deep K block; sB per 128x128 tile of the logical [K, N])
    | "mx" (uint8 E8M0 sA[M, K/32], sB[N, K/32]: each 32-deep K slice of a row
    of A / column of B is multiplied by 2^(s - 127) -- the formula of the
    reference's test_async_dot_scaled, test_tlx.py:2298-2444).
    """
    A = fp8_bits_to_f64(a_bits, a_fmt)
    B = fp8_bits_to_f64(b_bits_kn, b_fmt)
    if scale_mode == "none":
        return A @ B
    if scale_mode == "tensor":
        return (A @ B) * float(np.float32(scale_a)) * float(np.float32(scale_b))
    if scale_mode == "mx":
        sa = np.asarray(scale_a, np.int64)
        sb = np.asarray(scale_b, np.int64)
        K = A.shape[1]
        fa = np.ldexp(1.0, np.repeat(sa - 127, 32, axis=1)[:, :K])      # [M, K]
        fb = np.ldexp(1.0, np.repeat(sb - 127, 32, axis=1)[:, :K]).T    # [K, N]
        return (A * fa) @ (B * fb)
    if scale_mode == "block":
        M, K = A.shape
        N = B.shape[1]
        sa = np.asarray(scale_a, np.float64)
        sb = np.asarray(scale_b, np.float64)
        C = np.zeros((M, N))
        for kb in range(-(-K // 128)):
            ks = slice(kb * 128, min(K, kb * 128 + 128))
            part = A[:, ks] @ B[ks, :]
            col_scale = np.repeat(sb[kb], 128)[:N]
            C += part * sa[:, kb][:, None] * col_scale[None, :]
        return C
    raise ValueError(scale_mode)


def gemm_tolerance(a_deq: np.ndarray, b_deq_kn: np.ndarray) -> float:
    """max-abs-error bound 1e-2 * ||A|| * ||B|| / sqrt(K).

    ||A|| is the largest row 2-norm of the dequantized A and ||B|| the largest
    column 2-norm of the dequantized B, so ||A||*||B|| bounds every |C[m,n]|
    (Cauchy-Schwarz) and the bound is about 1% of the typical output size for
    random operands.
    """
    K = a_deq.shape[1]
    na = np.sqrt((a_deq.astype(np.float64) ** 2).sum(axis=1)).max()
    nb = np.sqrt((b_deq_kn.astype(np.float64) ** 2).sum(axis=0)).max()
    return 1e-2 * na * nb / np.sqrt(K)


OUTPUT_ROUNDING = 2.0 ** -8  # bf16 output: half an ulp is 2^-9 of |C|; budget 2^-8


def gemm_error(c: np.ndarray, ref: np.ndarray, a_deq: np.ndarray, b_deq_kn: np.ndarray):
    """(worst excess, tolerance) for a GEMM result against the oracle.

    The bound 1e-2 * ||A|| * ||B|| / sqrt(K) is about the GEMM's arithmetic;
    rounding the result to bf16 adds up to half an ulp of each element on top,
    budgeted as 2^-8 * |C_ref|.  Passing means  max(|C - C_ref| - 2^-8 |C_ref|) <= tol.
    """
    tol = gemm_tolerance(a_deq, b_deq_kn)
    ref = np.asarray(ref, np.float64)
    excess = (np.abs(np.asarray(c, np.float64) - ref) - OUTPUT_ROUNDING * np.abs(ref)).max()
    return float(excess), float(tol)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 (RNE) -> float32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(np.float32)


# ----------------------------------------------------------------------------
# Seeded synthetic inputs with the benchmark configurations' distributions.


def cast_input(n: int, seed: int = 0, sigma: float = 2.0, outlier_frac: float = 0.01,
               special_frac: float = 1e-4) -> np.ndarray:
    """~N(0, sigma) float32 with `outlier_frac` of positions set to +-U[500, 1e5]
    and `special_frac` set to NaN / +-Inf (half NaN, half Inf)."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n, dtype=np.float32) * np.float32(sigma)).astype(np.float32)
    k = int(n * outlier_frac)
    if k:
        idx = rng.choice(n, k, replace=False)
        x[idx] = (rng.uniform(500.0, 1e5, k) * rng.choice([-1.0, 1.0], k)).astype(np.float32)
    k = int(n * special_frac)
    if k:
        idx = rng.choice(n, k, replace=False)
        half = k // 2
        x[idx[:half]] = np.nan
        x[idx[half:]] = (np.inf * rng.choice([-1.0, 1.0], k - half)).astype(np.float32)
    return x


# ----------------------------------------------------------------------------
# Stochastic rounding (tlx.stoch_round, extensions/utlx/tlx/language/tlx/
# utility.py:113-153; the rounding rule is stated in include/b2x.h,
# b2x_stoch_round).  Integer restatement, one uint32 of entropy per element.

SR_FORMATS = {"e4m3": (3, -6), "e5m2": (2, -14), "f16": (10, -14), "bf16": (7, -126)}


def stoch_round_value(x: np.ndarray, r: np.ndarray, fmt: str) -> np.ndarray:
    """float32 result of the stochastic truncation, before saturation/encoding."""
    p, emin = SR_FORMATS[fmt]
    x = np.asarray(x, np.float32)
    bits = x.view(np.uint32).astype(np.int64)
    r = np.asarray(r).astype(np.uint32).astype(np.int64)
    sign = bits & 0x80000000
    a = bits & 0x7FFFFFFF
    E = a >> 23
    F = a & 0x7FFFFF
    sub = E == 0
    M = np.where(sub, F, F | 0x800000)
    e2 = np.where(sub, -149, E - 150)
    with np.errstate(divide="ignore"):
        lg = np.floor(np.log2(np.maximum(F, 1))).astype(np.int64)
    eb = np.where(sub, -149 + lg, E - 127)
    u = np.maximum(eb, emin) - p
    s = u - e2
    out = a.copy()  # s <= 0: representable already
    need = (s > 0) & (a != 0) & (a < 0x7F800000)
    ss = np.clip(s, 0, 63)
    q = np.where(ss >= 56, 0, M >> np.minimum(ss, 55))
    rem = np.where(ss >= 56, 0, M & ((np.int64(1) << np.minimum(ss, 55)) - 1))
    frac32 = np.where(ss <= 32, (rem << np.clip(32 - ss, 0, 32)) & 0xFFFFFFFF, rem >> np.clip(ss - 32, 0, 63))
    q = q + ((frac32 + r) >> 32)
    val = q.astype(np.float64) * np.exp2(u.astype(np.float64))
    with np.errstate(over="ignore"):
        vbits = val.astype(np.float32).view(np.uint32).astype(np.int64)
    out = np.where(need, vbits, out)
    res = (out | sign).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, res)


def stoch_round(x: np.ndarray, r: np.ndarray, fmt: str) -> np.ndarray:
    """Encoded bits: uint8 for e4m3/e5m2, uint16 for f16/bf16 (saturating;
    NaN -> the target's canonical NaN as the GPU's satfinite converts give it)."""
    y = stoch_round_value(x, r, fmt)
    if fmt in (E4M3, E5M2):
        return f32_to_fp8_bits(y, fmt)
    if fmt == "f16":
        fmax = np.float32(65504.0)
        with np.errstate(invalid="ignore"):
            c = np.where(np.isnan(y), np.float32(np.nan), np.clip(y, -fmax, fmax)).astype(np.float32)
        h = c.astype(np.float16).view(np.uint16)
        return np.where(np.isnan(y), np.uint16(0x7FFF), h).astype(np.uint16)
    # bf16: the value is exact in bf16 unless it overflowed; saturate to +-max
    yb = y.view(np.uint32)
    absb = yb & 0x7FFFFFFF
    sat = (absb >= 0x7F800000) & ~np.isnan(y)
    hi = (yb >> 16).astype(np.uint16)
    hi = np.where(sat, ((yb >> 16) & 0x8000) | 0x7F7F, hi)
    return np.where(np.isnan(y), np.uint16(0x7FFF), hi).astype(np.uint16)


# ----------------------------------------------------------------------------
# Split-K reduction of a reference-layout workspace.


def reduce_k(ws: np.ndarray, M: int, N: int, split_k: int, out: str = "f32") -> np.ndarray:
    """c[m, n] = sum over s = 0..SPLIT_K-1, in that order, of ws[s*M + m, n],
    accumulated in fp32 and stored in `out` ("f32", "bf16" bits as uint16,
    "f16" bits as uint16) with round-to-nearest-even -- the reference's
    `_reduce_k_kernel` (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:
    1033-1056: acc = 0; acc += partial.to(fp32) per split; acc.to(OUTPUT_DTYPE)).
    `ws` holds float32 values (already widened from the workspace dtype)."""
    w = np.asarray(ws, np.float32).reshape(split_k, M, N)
    acc = np.zeros((M, N), np.float32)
    for s in range(split_k):
        acc = (acc + w[s]).astype(np.float32)
    if out == "f32":
        return acc
    if out == "bf16":
        return (bf16_round(acc).view(np.uint32) >> 16).astype(np.uint16)
    if out == "f16":
        return acc.astype(np.float16).view(np.uint16)
    raise ValueError(out)
