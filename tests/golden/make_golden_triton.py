"""Generate the fp8 cast golden vectors on a GPU with upstream Triton.

The reference's quantize recipe (extensions/utlx/tlx/language/tlx/
mxfp8_utils.py:37-84) is a Triton kernel body; its cast semantics (tl.max,
tl.clamp, `.to(fp8)` with round-to-nearest-even) are whatever Triton's NVIDIA
lowering makes of them.  The reference itself cannot run here (its TLX plugin
needs a patched Triton), so this script restates the recipe as a plain-Triton
kernel -- the same operations in the same order -- and records what a B200
computes, including NaN, +-Inf, +-0, ties and saturation.  These vectors pin
the CPU oracle (oracle/fp8_oracle.py) and the b2x kernels.

Modes:
  mx1x32      the reference recipe verbatim (E8M0 RCEIL scales, `/` division)
  block1x128  fp32 scale per 1x128 group, IEEE divisions (tl.math.div_rn)
  tensor      fp32 scale for the whole tensor, IEEE divisions
  none        clamp + cast only
for fp32 and bf16 inputs and e4m3fn / e5m2 outputs.

Usage (on a machine with a CUDA GPU):
    python tests/golden/make_golden_triton.py [out.npz]
"""
import os
import sys

import numpy as np
import torch
import triton
import triton.language as tl

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
import fp8_oracle as O  # noqa: E402  (input generator only)


@triton.jit
def _group_kernel(x_ptr, q_ptr, s_ptr, C, NG, G: tl.constexpr, FMAX: tl.constexpr, MX: tl.constexpr):
    row = tl.program_id(0)
    g = tl.program_id(1)
    offs = g * G + tl.arange(0, G)
    mask = offs < C
    x = tl.load(x_ptr + row * C + offs, mask=mask, other=0.0).to(tl.float32)
    amax = tl.max(tl.abs(x), axis=0)
    if MX:
        descale = amax / FMAX
        e = (descale.to(tl.uint32, bitcast=True) + 0x007FFFFF) & 0x7F800000
        d = e.to(tl.float32, bitcast=True)
        tl.store(s_ptr + row * NG + g, (e >> 23).to(tl.uint8))
        inv = tl.where(d == 0, 0.0, 1.0 / d)
    else:
        descale = tl.math.div_rn(amax, FMAX)
        tl.store(s_ptr + row * NG + g, descale)
        inv = tl.where(descale == 0, 0.0, tl.math.div_rn(1.0, descale))
    y = tl.clamp(x * inv, -FMAX, FMAX)
    tl.store(q_ptr + row * C + offs, y.to(q_ptr.dtype.element_ty), mask=mask)


@triton.jit
def _none_kernel(x_ptr, q_ptr, n, BLOCK: tl.constexpr, FMAX: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    mask = offs < n
    x = tl.load(x_ptr + offs, mask=mask, other=0.0).to(tl.float32)
    y = tl.clamp(x, -FMAX, FMAX)
    tl.store(q_ptr + offs, y.to(q_ptr.dtype.element_ty), mask=mask)


def special_rows(C: int) -> np.ndarray:
    """Rows of hand-picked values: NaN/Inf/zeros/ties/saturation/subnormals."""
    rows = []
    vals = [0.0, -0.0, np.nan, -np.nan, np.inf, -np.inf, 448.0, -448.0, 449.0, 464.0, 465.0, 480.0, 500.0,
            57344.0, 61440.0, 61441.0, 65536.0, 1e30, -1e30, 1e-40, -1e-40, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10,
            2.0 ** -16, 2.0 ** -17, 3 * 2.0 ** -17, 1.0625, 1.1875, -1.0625, 1.125, 0.4946, 7.5, 240.0, 232.0]
    for fmt in (O.E4M3, O.E5M2):
        t = O.DECODE[fmt]
        fin = np.unique(np.abs(t[np.isfinite(t)]))
        mids = (fin[:-1] + fin[1:]) / 2
        vals += list(fin[::7]) + list(mids[::5]) + list(-mids[::11])
    vals = np.array(vals, np.float32)
    # row A: specials as-is; row B: specials in a group whose amax is 448*2^k exactly
    for shift in (0, 3):
        r = np.zeros(C, np.float32)
        v = vals[: C]
        r[: v.size] = v * np.float32(2.0 ** shift)
        rows.append(r)
    # groups whose amax is exactly FMAX * 2^k (IEEE quotient is a power of two)
    r = np.zeros(C, np.float32)
    for g in range(C // 32):
        k = (g % 9) - 4
        r[g * 32: g * 32 + 32] = np.linspace(-1, 1, 32, dtype=np.float32) * np.float32(448.0 * 2.0 ** k)
    rows.append(r)
    r = np.zeros(C, np.float32)
    for g in range(C // 32):
        k = (g % 9) - 4
        r[g * 32: g * 32 + 32] = np.linspace(-1, 1, 32, dtype=np.float32) * np.float32(57344.0 * 2.0 ** k)
    rows.append(r)
    rows.append(np.zeros(C, np.float32))  # all-zero row: scale 0 -> inv 0
    return np.stack(rows)


def main(out_path: str) -> None:
    dev = "cuda"
    R, C = 64, 256
    x = O.cast_input(R * C, seed=1234, sigma=2.0, outlier_frac=0.01, special_frac=0.002).reshape(R, C)
    sp = special_rows(C)
    x[: sp.shape[0]] = sp
    x_nan_only = O.cast_input(R * C, seed=99, special_frac=0.0).reshape(R, C)
    x_nan_only.reshape(-1)[::997] = np.nan
    out = {"x_f32": x, "x_f32_noinf": x_nan_only}
    bf = torch.from_numpy(x).to(torch.bfloat16)
    bf_noinf = torch.from_numpy(x_nan_only).to(torch.bfloat16)
    out["x_bf16_bits"] = bf.view(torch.int16).numpy().view(np.uint16)
    out["x_bf16_noinf_bits"] = bf_noinf.view(torch.int16).numpy().view(np.uint16)
    fp8 = {"e4m3": (torch.float8_e4m3fn, 448.0), "e5m2": (torch.float8_e5m2, 57344.0)}
    srcs = {"f32": (torch.from_numpy(x), torch.from_numpy(x_nan_only)), "bf16": (bf, bf_noinf)}
    for sname, (xt, xt_noinf) in srcs.items():
        for fname, (fdt, fmax) in fp8.items():
            for mode in ("none", "mx1x32", "block1x128", "tensor", "tensor_noinf"):
                src = (xt_noinf if mode == "tensor_noinf" else xt).to(dev)
                q = torch.empty(src.shape, dtype=fdt, device=dev)
                if mode == "none":
                    n = src.numel()
                    _none_kernel[(triton.cdiv(n, 1024),)](src, q, n, BLOCK=1024, FMAX=fmax)
                    s = torch.zeros(1)
                else:
                    if mode.startswith("tensor"):
                        src = src.reshape(1, -1)
                        q = q.reshape(1, -1)
                        G = src.shape[1]
                    else:
                        G = 32 if mode == "mx1x32" else 128
                    rr, cc = src.shape
                    ng = triton.cdiv(cc, G)
                    s = torch.empty((rr, ng), dtype=torch.uint8 if mode == "mx1x32" else torch.float32, device=dev)
                    _group_kernel[(rr, ng)](src, q, s, cc, ng, G=G, FMAX=fmax, MX=(mode == "mx1x32"))
                torch.cuda.synchronize()
                key = f"{sname}_{fname}_{mode}"
                out[f"q_{key}"] = q.view(torch.uint8).cpu().numpy().reshape(R, C)
                out[f"s_{key}"] = s.cpu().numpy()
    out["device"] = np.array(torch.cuda.get_device_name())
    out["triton_version"] = np.array(triton.__version__)
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, "keys", len(out))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "cast_golden.npz"))
