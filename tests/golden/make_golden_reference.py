"""Generate golden fixtures by running the REFERENCE's own Python code.

Runs in a checkout that has the reference tree (it reads
extensions/utlx/tlx/... from REFERENCE_ROOT, default /root/reference); the
GPU box and the test suite only read the committed outputs:

  heuristic_golden.json
      blackwell_gemm_ws.get_heuristic_config(M, N, K)          (:24-341)
      blackwell_gemm_ws.preprocess_configs(space, {M,N,K})      (:442-637)
      over a fixed shape list plus seeded random shapes.  Pure Python: the
      reference module is imported as-is (a stub stands in for its unused
      `triton.language.extra.tlx` import, and triton.Config accepts the
      `ctas_per_cga` keyword of the reference's newer Triton).

  ref_kernels_golden.npz
      mxfp8_utils._compute_scale_and_quantize (:13-86) and
      blackwell_gemm_ws._reduce_k_kernel (:1033-1056), the reference's own
      @triton.jit functions, executed by Triton's interpreter
      (TRITON_INTERPRET=1) on the CPU.  The interpreter emulates the
      reference's arithmetic op by op in numpy (fp32 division, uint32 bit
      tricks, multiply, clamp, fp32 accumulation) but its float narrowing
      (`_convert_float`) truncates the mantissa without carry and does not
      saturate.  That one function is replaced here by round-to-nearest-even
      conversions from torch (fp32 -> e4m3fn / e5m2 / bf16 / fp16), which is
      what Triton's NVIDIA lowering emits (cvt.rn[.satfinite]).  Inputs are
      finite: NaN and Inf handling is hardware-specific and is pinned by the
      B200 golden run of make_golden_triton.py instead.

Usage:  python tests/golden/make_golden_reference.py
"""
import importlib.util
import json
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("REFERENCE_ROOT", "/root/reference")
TLX = os.path.join(REF, "extensions", "utlx", "tlx")

# --- environment shims (no reference code is changed) ----------------------
_stub = types.ModuleType("triton.language.extra.tlx")
sys.modules["triton.language.extra.tlx"] = _stub
import triton.language.extra as _extra  # noqa: E402
_extra.tlx = _stub

_Config = triton.Config


class _ConfigWithCga(_Config):
    def __init__(self, kwargs, *a, ctas_per_cga=None, **kw):
        super().__init__(kwargs, *a, **kw)
        self.ctas_per_cga = ctas_per_cga


triton.Config = _ConfigWithCga

_TORCH_OF = {tl.float8e4nv: torch.float8_e4m3fn, tl.float8e5: torch.float8_e5m2,
             tl.bfloat16: torch.bfloat16, tl.float16: torch.float16, tl.float32: torch.float32}


def _convert_float_rne(inp, in_dtype, out_dtype, rounding_mode):
    """fp -> fp with round-to-nearest-even (torch), returned as the raw bits
    the interpreter stores (uint8 for fp8, uint16 for bf16/fp16)."""
    if in_dtype == tl.bfloat16:
        src = torch.from_numpy(np.ascontiguousarray(inp).view(np.int16)).view(torch.bfloat16)
    elif in_dtype in (tl.float8e4nv, tl.float8e5):
        src = torch.from_numpy(np.ascontiguousarray(inp).view(np.uint8)).view(_TORCH_OF[in_dtype])
    else:
        src = torch.from_numpy(np.ascontiguousarray(inp))
    out = src.to(_TORCH_OF[out_dtype])
    bits = {1: torch.uint8, 2: torch.int16, 4: torch.int32}[out.element_size()]
    arr = out.view(bits).numpy()
    ubits = {1: np.uint8, 2: np.uint16, 4: np.uint32}[out.element_size()]
    return arr.view(ubits).reshape(np.shape(inp))


_interp._convert_float = _convert_float_rne


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


ref_ws = _load(os.path.join(TLX, "tutorials", "blackwell_gemm_ws.py"), "ref_blackwell_gemm_ws")
ref_ws._get_num_sms = lambda: 148
ref_mx = _load(os.path.join(TLX, "language", "tlx", "mxfp8_utils.py"), "ref_mxfp8_utils")
_compute_scale_and_quantize = ref_mx._compute_scale_and_quantize


# --- heuristics ------------------------------------------------------------

FIXED_SHAPES = [
    (512, 512, 512), (8192, 8192, 8192), (4096, 7168, 7168), (64, 8192, 28672),
    (8192, 10240, 8192), (8192, 57344, 8192), (8192, 8192, 28672),
    (8192, 1280, 8192), (8192, 7168, 8192), (8192, 8192, 3584), (8192, 2560, 8192), (8192, 14336, 8192),
    (8192, 8192, 7168), (8192, 5120, 8192), (8192, 28672, 8192), (8192, 8192, 14336),
    (3159809, 384, 384), (1024, 2048, 16384), (3000, 300, 64), (1500, 100, 256), (200, 20000, 64),
    (1, 4096, 4096), (16, 8192, 8192), (128, 128, 128), (256, 384, 512), (2048, 2048, 2048),
    (4096, 4096, 4096), (16384, 16384, 1024), (100000, 1000, 128), (1024, 65536, 128),
]
PREPROCESS_SHAPES = [(8192, 8192, 8192), (64, 8192, 28672), (4096, 7168, 7168), (1024, 2048, 16384),
                     (100000, 1000, 128), (512, 512, 512), (8192, 1280, 8192), (256, 65536, 4096)]


def _clean(cfg):
    if cfg is None:
        return None
    out = {}
    for k, v in cfg.items():
        if k == "pre_hook":
            continue
        out[k] = list(v) if isinstance(v, tuple) else v
    return out


def heuristics():
    rng = np.random.default_rng(2024)
    shapes = list(FIXED_SHAPES)
    for _ in range(300):
        M = int(2 ** rng.uniform(0, 16)) + int(rng.integers(0, 3))
        N = int(2 ** rng.uniform(4, 16)) // 16 * 16 + 16
        K = int(2 ** rng.uniform(5, 15.5)) // 16 * 16 + 16
        shapes.append((M, N, K))
    heur = []
    for M, N, K in shapes:
        heur.append({"M": M, "N": N, "K": K, "config": _clean(ref_ws.get_heuristic_config(M, N, K))})
    space = ref_ws.get_cuda_autotune_config()
    keys = sorted(space[0].kwargs.keys())
    pre = []
    for M, N, K in PREPROCESS_SHAPES:
        kept = ref_ws.preprocess_configs(space, {"M": M, "N": N, "K": K})
        pre.append({"M": M, "N": N, "K": K,
                    "kept": sorted([[c.kwargs[k] for k in keys] for c in kept])})
    with open(os.path.join(HERE, "heuristic_golden.json"), "w") as f:
        json.dump({"generator": "reference blackwell_gemm_ws.py via make_golden_reference.py",
                   "space_size": len(space), "space_keys": keys, "heuristic": heur, "preprocess": pre},
                  f, separators=(",", ":"))
    print(f"heuristics: {len(heur)} shapes, preprocess over {len(space)} configs for {len(pre)} shapes")


# --- reference kernels under the interpreter -------------------------------


@triton.jit
def _mx_driver(x_ptr, q_ptr, s_ptr, C: tl.constexpr, BM: tl.constexpr, BK: tl.constexpr,
               DTYPE: tl.constexpr):
    # one [BM, BK] block per program; calls the reference function verbatim
    pm = tl.program_id(0)
    pk = tl.program_id(1)
    rows = pm * BM + tl.arange(0, BM)
    cols = pk * BK + tl.arange(0, BK)
    x = tl.load(x_ptr + rows[:, None] * C + cols[None, :])
    scale, q = _compute_scale_and_quantize(x, 32, DTYPE)
    tl.store(q_ptr + rows[:, None] * C + cols[None, :], q)
    NS: tl.constexpr = BK // 32
    scols = pk * NS + tl.arange(0, NS)
    tl.store(s_ptr + rows[:, None] * (C // 32) + scols[None, :], scale)


def mx_input(rows, cols, seed):
    """Finite fp32 rows that exercise the recipe: N(0,1) and N(0,2) with
    outliers, tiny and subnormal values, all-zero groups, groups whose amax
    is exactly 448*2^k / 57344*2^k or a power of two, single-spike groups,
    huge values near fp32 max, and values that land on RNE ties."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[1::8] *= 2.0
    out = rng.random((rows, cols)) < 0.01
    x[out] = (np.sign(rng.standard_normal(out.sum())) * rng.uniform(500, 1e5, out.sum())).astype(np.float32)
    g = x.reshape(rows, cols // 32, 32)
    g[2::16, ::3] = 0.0                                                  # all-zero groups
    g[3::16, ::2] *= np.float32(1e-30)                                   # tiny
    g[4::16, 1::2] = (rng.standard_normal(g[4::16, 1::2].shape) * 1e-40).astype(np.float32)  # subnormal
    g[5::16, :, 0] = np.float32(448.0) * np.exp2(rng.integers(-20, 20, g[5::16, :, 0].shape)).astype(np.float32)
    g[6::16, :, 7] = np.float32(57344.0) * np.exp2(rng.integers(-20, 20, g[6::16, :, 7].shape)).astype(np.float32)
    g[7::16, :, 3] = np.exp2(rng.integers(-60, 60, g[7::16, :, 3].shape)).astype(np.float32)
    g[8::16, :, :] = 0.0
    g[8::16, :, 5] = rng.uniform(-1e3, 1e3, g[8::16, :, 5].shape).astype(np.float32)   # single spike
    g[9::16] = np.clip(g[9::16], -2e5, 2e5) * np.float32(1e33)          # near fp32 max
    # ties: amax 448 makes the scale exactly 1; mantissas halfway between e4m3 / e5m2 codes
    t = g[10::16]
    t[:] = (rng.integers(-15, 16, t.shape) * 2 + 1).astype(np.float32) * np.float32(2.0 ** -4)
    t[:, :, 0] = 448.0
    t = g[11::16]
    t[:] = (rng.integers(-7, 8, t.shape) * 2 + 1).astype(np.float32) * np.float32(2.0 ** -3)
    t[:, :, 0] = 57344.0
    return np.ascontiguousarray(x)


def run_mx(x, tl_dtype):
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.uint8)
    s = np.zeros((rows, cols // 32), np.uint8)
    xt = torch.from_numpy(x)
    qt = torch.from_numpy(q).view(_TORCH_OF[tl_dtype])
    st = torch.from_numpy(s)
    BM, BK = 16, 128
    _mx_driver[(rows // BM, cols // BK)](xt, qt, st, cols, BM, BK, tl_dtype)
    return qt.view(torch.uint8).numpy().copy(), st.numpy().copy()


def run_reduce_k(ws, M, N, split_k):
    c = torch.empty((M, N), dtype=ws.dtype)
    grid = (triton.cdiv(M, 128), triton.cdiv(N, 128))
    ref_ws._reduce_k_kernel[grid](ws, c, M, N, SPLIT_K=split_k, BLOCK_SIZE_M=128, BLOCK_SIZE_N=128,
                                  OUTPUT_DTYPE={torch.bfloat16: tl.bfloat16, torch.float16: tl.float16,
                                                torch.float32: tl.float32}[ws.dtype])
    return c


def kernels():
    out = {}
    x = mx_input(128, 512, seed=11)
    xb = torch.from_numpy(mx_input(64, 512, seed=12)).to(torch.bfloat16).float().numpy()  # bf16-exact
    out["mx_x_f32"] = x
    out["mx_x_bf16_bits"] = torch.from_numpy(xb).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    for name, dt in (("e4m3", tl.float8e4nv), ("e5m2", tl.float8e5)):
        q, s = run_mx(x, dt)
        out[f"mx_f32_{name}_q"], out[f"mx_f32_{name}_s"] = q, s
        q, s = run_mx(xb, dt)
        out[f"mx_bf16_{name}_q"], out[f"mx_bf16_{name}_s"] = q, s
    rng = np.random.default_rng(13)
    for dtn, dt in (("f32", torch.float32), ("bf16", torch.bfloat16), ("f16", torch.float16)):
        for (M, N, sk) in ((100, 200, 3), (32, 128, 8)):
            ws = torch.from_numpy((rng.standard_normal((sk * M, N)) * 40).astype(np.float32)).to(dt)
            c = run_reduce_k(ws, M, N, sk)
            key = f"rk_{dtn}_{M}x{N}x{sk}"
            bits = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}[dt]
            out[key + "_ws"] = ws.view(bits).numpy().copy()
            out[key + "_c"] = c.view(bits).numpy().copy()
    for k, v in out.items():
        assert k.endswith("_q") or k.endswith("_s") or np.all(np.isfinite(v.view(np.float32))) or v.dtype != np.float32, k
    np.savez_compressed(os.path.join(HERE, "ref_kernels_golden.npz"), **out)
    print("kernels:", ", ".join(sorted(k for k in out)))


if __name__ == "__main__":
    heuristics()
    kernels()
