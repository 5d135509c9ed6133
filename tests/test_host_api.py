"""CPU tests of the host-side mirror of the reference API (blackwell_gemm_ws /
mxfp8_utils names, heuristics, config mapping) and of the no-CPU-fallback
rule.  Expected configs follow the rules of the reference's
get_heuristic_config (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:24-341)."""
import math

import numpy as np
import pytest
import torch

import b2x
from b2x import blackwell_gemm_ws as G
from b2x import mxfp8_utils


def test_module_exposes_reference_names():
    for name in ("matmul", "get_heuristic_config", "_select_group_size_m", "get_cuda_autotune_config",
                 "matmul_tma_set_block_size_hook", "preprocess_configs", "_reduce_k_kernel", "reduce_k"):
        assert hasattr(G, name), name
    for name in ("_compute_scale_and_quantize", "_to_mxfp8_block", "get_fp8_format_name"):
        assert hasattr(mxfp8_utils, name), name


def test_select_group_size_m():
    assert G._select_group_size_m(100000, 1000, 128) == 1          # M >> N: sweep M
    assert G._select_group_size_m(64, 8192, 128) == 1              # one M tile
    assert G._select_group_size_m(1024, 65536, 128) == 8           # N >> M: min(64, tiles)
    assert G._select_group_size_m(8192, 8192, 256) == 8


def test_heuristic_saturated_square():
    c = G.get_heuristic_config(8192, 8192, 8192)
    assert (c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"], c["SPLIT_K"], c["NUM_CTAS"]) == (256, 256, 64, 1, 1)
    assert c["GROUP_SIZE_M"] == 8 and c["NUM_SMEM_BUFFERS"] == 3


def test_heuristic_tall_m_low_intensity_pairs_ctas():
    c = G.get_heuristic_config(3159809, 384, 384)
    assert (c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"], c["NUM_CTAS"]) == (256, 128, 128, 2)
    assert c["ctas_per_cga"] == (2, 1, 1) and c["GROUP_SIZE_M"] == 1


def test_heuristic_decode_uses_split_k():
    c = G.get_heuristic_config(64, 8192, 28672)
    # small output (M*N < 1e6): 128x64x128 tiles; 224 K tiles -> first of (4, 2, 8) keeping >= 4 per split
    assert (c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"], c["SPLIT_K"]) == (128, 64, 128, 4)
    assert c["NUM_TMEM_BUFFERS"] == 3


def test_heuristic_large_output_undersaturated():
    c = G.get_heuristic_config(1024, 2048, 16384)
    assert (c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"]) == (256, 128, 64)
    assert c["SPLIT_K"] == 4 and c["EPILOGUE_SUBTILE"] == 8


def test_heuristic_fallback_returns_a_fitting_config():
    for M, N, K in ((3000, 300, 64), (1500, 100, 256), (200, 20000, 64)):
        c = G.get_heuristic_config(M, N, K)
        assert c is not None
        assert c["BLOCK_SIZE_M"] // c["NUM_MMA_GROUPS"] <= 128


def test_preprocess_configs_rules():
    space = [c for c in G.get_cuda_autotune_config() if c["BLOCK_SIZE_K"] == 128 and c["NUM_CTAS"] == 1][:20000]
    kept = G.preprocess_configs(space, {"M": 8192, "N": 8192, "K": 8192}, num_sms=148)
    assert kept
    for c in kept:
        assert c["SPLIT_K"] == 1                      # saturated: split-K pruned
        assert c["GROUP_SIZE_M"] == 8                 # balanced: moderate group size
        smem = c["BLOCK_SIZE_M"] * 128 * 2 * c["NUM_SMEM_BUFFERS"] + 128 * c["BLOCK_SIZE_N"] * 2 * c["NUM_SMEM_BUFFERS"]
        assert smem <= 232 * 1024
    kept = G.preprocess_configs(space, {"M": 64, "N": 8192, "K": 28672}, num_sms=148)
    assert kept and all(c["GROUP_SIZE_M"] >= 32 for c in kept)   # N >> M
    for c in kept:
        assert c["SPLIT_K"] == 1 or math.ceil(28672 / 128) // c["SPLIT_K"] >= 4


def test_config_dict_mapping():
    f = G._to_b2x_config({"BLOCK_SIZE_M": 256, "BLOCK_SIZE_N": 256, "GROUP_SIZE_M": 8, "SPLIT_K": 1}, 8192)
    assert f[0] == 128 and f[1] == 256 and f[2] == 128 and f[3] == 16  # 256-row groups of 8 -> 16 x 128 rows
    with pytest.warns(UserWarning):
        f = G._to_b2x_config({"BLOCK_SIZE_N": 128, "SPLIT_K": 24}, 1024)  # 8 K blocks cannot feed 24 splits
    assert f[9] <= 8


def test_no_cpu_fallback():
    x = torch.randn(4, 128)
    with pytest.raises(ValueError, match="CUDA"):
        b2x.quantize(x, "tensor", torch.float8_e4m3fn)
    a = torch.zeros(4, 16, dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="CUDA"):
        b2x.matmul(a, a.t(), {})


def test_new_ops_have_no_cpu_fallback():
    a = torch.zeros(4, 16, dtype=torch.float8_e4m3fn)
    w = torch.zeros(256, 16, dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="CUDA"):
        b2x.grouped_gemm([a], [a])
    with pytest.raises(ValueError, match="CUDA"):
        b2x.gemm_swiglu(a, w)
    with pytest.raises(ValueError, match="CUDA"):
        b2x.stoch_round(torch.zeros(8), torch.bfloat16, torch.zeros(8, dtype=torch.int32))


def test_mx_scale_mode_and_config_mapping():
    sa = torch.zeros(4, 4, dtype=torch.uint8)
    assert G._scale_mode(sa, sa) == "mx"
    with pytest.raises(ValueError):
        G._scale_mode(sa, torch.zeros(4, 4))  # MX scales must both be uint8
    assert G._to_b2x_config({"BLOCK_SIZE_N": 192}, 1024)[1] == 192  # the MX tile width is kept
    assert G._to_b2x_config({"BLOCK_SIZE_N": 200}, 1024)[1] == 256  # other widths snap to 64/128/256


def test_matmul_reference_asserts():
    a = torch.zeros(4, 16, dtype=torch.float8_e4m3fn)
    with pytest.raises(AssertionError, match="Incompatible dimensions"):
        b2x.matmul(a, torch.zeros(8, 4, dtype=torch.float8_e4m3fn))
    with pytest.raises(AssertionError, match="contiguous"):
        b2x.matmul(torch.zeros(16, 8, dtype=torch.float8_e4m3fn).t(), torch.zeros(16, 4, dtype=torch.float8_e4m3fn))
    with pytest.raises(NotImplementedError):
        b2x.matmul(torch.zeros(4, 16), torch.zeros(16, 4))


def test_mxfp8_utils_argument_checks():
    with pytest.raises(AssertionError):
        mxfp8_utils._compute_scale_and_quantize(torch.zeros(128, 128), 16, torch.float8_e4m3fn)
    with pytest.raises(AssertionError):
        mxfp8_utils._compute_scale_and_quantize(torch.zeros(128, 128), 32, torch.float16)
    assert mxfp8_utils.get_fp8_format_name(torch.float8_e5m2) == "e5m2"
    assert mxfp8_utils.get_fp8_format_name("e4m3") == "e4m3"


def test_oracle_c_matches_numpy_oracle():
    import fp8_oracle as O
    import oracle_c as OC
    x = O.cast_input(300 * 520, seed=4).reshape(300, 520)
    for fmt in (O.E4M3, O.E5M2):
        for mode in ("none", "tensor", "block1x128", "block128x128", "mx1x32"):
            q1, s1 = O.quantize(x, mode, fmt)
            q2, s2 = OC.quantize(x, mode, fmt)
            assert np.array_equal(q1, q2), (fmt, mode)
            if s1 is not None:
                assert np.array_equal(np.asarray(s1).reshape(-1).view(np.uint8), np.asarray(s2).reshape(-1).view(np.uint8))
    rng = np.random.default_rng(0)
    a = O.f32_to_fp8_bits(rng.standard_normal((96, 640)).astype(np.float32), O.E4M3)
    bt = O.f32_to_fp8_bits(rng.standard_normal((200, 640)).astype(np.float32), O.E5M2)
    c, flops = OC.gemm_bf16(a, bt, O.E4M3, O.E5M2, 0.5, 2.0)
    assert flops == 2 * 96 * 200 * 640
    ref = O.gemm(a, bt.T, O.E4M3, O.E5M2, scale_mode="tensor", scale_a=0.5, scale_b=2.0)
    err, tol = O.gemm_error(O.bf16_bits_to_f32(c), ref, O.fp8_bits_to_f64(a, O.E4M3) * 0.5,
                            O.fp8_bits_to_f64(bt, O.E5M2).T * 2.0)
    assert err <= tol
