"""CPU tests pinned by the reference's own code.

The fixtures in tests/golden/ were produced by tests/golden/
make_golden_reference.py, which imports the reference's modules and runs
them unchanged:
  * heuristic_golden.json -- get_heuristic_config / preprocess_configs
    (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:24-341, :442-637);
  * ref_kernels_golden.npz -- _compute_scale_and_quantize (extensions/utlx/
    tlx/language/tlx/mxfp8_utils.py:13-86) and _reduce_k_kernel
    (blackwell_gemm_ws.py:1033-1056) executed by Triton's interpreter with
    round-to-nearest-even narrowing.
Here the CPU oracle and the host-side mirror are checked against them; the
GPU kernels are checked against the same fixtures in tests/test_reference_pinned_gpu.py.
"""
import json
import os

import numpy as np
import pytest

import fp8_oracle as O
from b2x import blackwell_gemm_ws as G

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def heur():
    with open(os.path.join(GOLD, "heuristic_golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def kern():
    return dict(np.load(os.path.join(GOLD, "ref_kernels_golden.npz")))


def _norm(cfg):
    if cfg is None:
        return None
    out = {k: (list(v) if isinstance(v, tuple) else v) for k, v in cfg.items() if k != "pre_hook"}
    return out


def test_heuristic_config_matches_reference(heur):
    bad = []
    for e in heur["heuristic"]:
        got = _norm(G.get_heuristic_config(e["M"], e["N"], e["K"]))
        if got != e["config"]:
            bad.append((e["M"], e["N"], e["K"], got, e["config"]))
    assert not bad, f"{len(bad)} of {len(heur['heuristic'])} shapes differ, first: {bad[0]}"


def test_preprocess_configs_matches_reference(heur):
    keys = heur["space_keys"]
    space = G.get_cuda_autotune_config()
    assert len(space) == heur["space_size"]
    for e in heur["preprocess"]:
        kept = G.preprocess_configs(space, {"M": e["M"], "N": e["N"], "K": e["K"]}, num_sms=148)
        got = sorted([[(list(c[k]) if isinstance(c[k], tuple) else c[k]) for k in keys] for c in kept])
        assert got == e["kept"], (e["M"], e["N"], e["K"], len(got), len(e["kept"]))


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2])
def test_oracle_mx_matches_reference_function(kern, src, fmt):
    if src == "f32":
        x = kern["mx_x_f32"]
    else:
        x = O.bf16_bits_to_f32(kern["mx_x_bf16_bits"])
    q, s = O.quantize(x, "mx1x32", fmt)
    np.testing.assert_array_equal(s, kern[f"mx_{src}_{fmt}_s"])
    np.testing.assert_array_equal(q, kern[f"mx_{src}_{fmt}_q"])


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("shape", ["100x200x3", "32x128x8"])
def test_oracle_reduce_k_matches_reference_kernel(kern, dt, shape):
    M, N, sk = (int(v) for v in shape.split("x"))
    ws_bits = kern[f"rk_{dt}_{shape}_ws"]
    if dt == "f32":
        ws = ws_bits.view(np.float32)
    elif dt == "bf16":
        ws = O.bf16_bits_to_f32(ws_bits.view(np.uint16))
    else:
        ws = ws_bits.view(np.float16).astype(np.float32)
    got = O.reduce_k(ws, M, N, sk, dt)
    want = kern[f"rk_{dt}_{shape}_c"]
    np.testing.assert_array_equal(got.view(np.uint32 if dt == "f32" else np.uint16),
                                  want.view(np.uint32 if dt == "f32" else np.uint16))
