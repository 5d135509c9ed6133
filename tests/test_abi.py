"""CPU tests of the C ABI boundary: libb2x.so loads, exports every symbol that
include/b2x.h declares, and rejects bad requests with status codes and
messages before touching a GPU.  No kernel is launched here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b2x.h")


def _lib():
    from b2x import _lib as L
    return L


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"B2X_API\s+[\w\s\*]+?\b(b2x_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("b2x_fp8_gemm", "b2x_fp8_cast", "b2x_splitk_reduce", "b2x_gemm_workspace_size",
              "b2x_cast_workspace_size", "b2x_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = _lib()
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"declared in b2x.h but not exported: {missing}"
    assert set(declared_symbols()) == set(L.EXPORTED)


def test_abi_version_matches_header():
    L = _lib()
    v = int(re.search(r"#define B2X_ABI_VERSION (\d+)", open(HEADER).read()).group(1))
    assert L.lib().b2x_abi_version() == v


def test_struct_layouts_match_header():
    """The ctypes mirrors of the ABI structs have the C sizes."""
    import shutil
    import subprocess
    import tempfile
    L = _lib()
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = '#include <stdio.h>\n#include "b2x.h"\nint main(){printf("%zu %zu %zu\\n", sizeof(b2x_cast_args),' \
          ' sizeof(b2x_gemm_config), sizeof(b2x_gemm_args)); printf("%zu\\n", sizeof(b2x_allreduce_args));' \
          ' return 0;}\n'
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "p.c"), "w") as f:
            f.write(src)
        exe = os.path.join(d, "p")
        subprocess.run([cc, "-I", os.path.join(ROOT, "include"), os.path.join(d, "p.c"), "-o", exe], check=True)
        sizes = [int(v) for v in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert sizes == [ctypes.sizeof(L.CastArgs), ctypes.sizeof(L.GemmConfig), ctypes.sizeof(L.GemmArgs),
                     ctypes.sizeof(L.AllReduceArgs)]


def _gemm_args(**kw):
    L = _lib()
    g = L.GemmArgs()
    g.a, g.b, g.c = 0x10000, 0x20000, 0x30000
    g.M, g.N, g.K = 256, 256, 256
    g.lda, g.ldb_k, g.ldb_n, g.ldc = 256, 1, 256, 256
    g.a_type = g.b_type = L.E4M3
    g.c_type = L.BF16
    g.scale_mode = L.SCALE_NONE
    for k, v in kw.items():
        setattr(g, k, v)
    return g


@pytest.mark.parametrize("field,value,status", [
    ("a_type", 1, "ERR_UNSUPPORTED"),          # bf16 A: not this library's path
    ("c_type", 3, "ERR_UNSUPPORTED"),          # fp8 C
    ("lda", 200, "ERR_INVALID_ARG"),           # lda < K
    ("lda", 264, "ERR_INVALID_ARG"),           # lda % 16 != 0
    ("a", 0, "ERR_INVALID_ARG"),               # NULL A
    ("a", 0x10008, "ERR_INVALID_ARG"),         # misaligned A
    ("ldb_k", 3, "ERR_INVALID_ARG"),           # neither K-major nor row-major
    ("ldc", 100, "ERR_INVALID_ARG"),           # ldc < N
    ("K", 0, "ERR_UNSUPPORTED"),
    ("M", -1, "ERR_INVALID_ARG"),
])
def test_gemm_rejects_bad_arguments(field, value, status):
    L = _lib()
    g = _gemm_args(**{field: value})
    st = L.lib().b2x_fp8_gemm(ctypes.byref(g), None)
    assert st == getattr(L, status), L.lib().b2x_last_error()
    assert L.lib().b2x_last_error()


def test_gemm_split_k_needs_workspace():
    L = _lib()
    g = _gemm_args()
    g.config.split_k = 2
    assert L.lib().b2x_gemm_workspace_size(ctypes.byref(g)) == 256 * 256 * 4 + 256
    assert L.lib().b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_WORKSPACE
    g.config.split_k = 3  # 2 K blocks of 128 cannot feed 3 splits
    assert L.lib().b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_INVALID_ARG


def test_gemm_zero_sized_is_a_no_op():
    L = _lib()
    g = _gemm_args(M=0)
    assert L.lib().b2x_fp8_gemm(ctypes.byref(g), None) == L.OK


def test_block_scaled_requires_kmajor_b():
    L = _lib()
    g = _gemm_args(ldb_k=256, ldb_n=1, scale_mode=L.SCALE_BLOCK_1x128, scale_a=0x40000, scale_b=0x50000)
    assert L.lib().b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_UNSUPPORTED


def _ar_args(**kw):
    L = _lib()
    r = L.AllReduceArgs()
    r.rank, r.world, r.epoch = 0, 2, 1
    r.c_peers[0], r.c_peers[1] = 0x30000, 0x70000
    r.signal_peers[0], r.signal_peers[1] = 0x90000, 0xA0000
    for k, v in kw.items():
        setattr(r, k, v)
    return r


def test_allreduce_signal_words():
    lib = _lib().lib()
    assert lib.b2x_allreduce_signal_words(8192, 8192) == 64 + 64 * 32
    assert lib.b2x_allreduce_signal_words(256, 256) == 64 + 2


@pytest.mark.parametrize("gemm_kw,ar_kw,status", [
    ({}, {"world": 9}, "ERR_INVALID_ARG"),
    ({}, {"rank": 2}, "ERR_INVALID_ARG"),
    ({"M": 384}, {}, "ERR_UNSUPPORTED"),                      # M not a multiple of 256
    ({"c_type": 2}, {}, "ERR_UNSUPPORTED"),                   # fp16 output
    ({"ldb_k": 256, "ldb_n": 1}, {}, "ERR_UNSUPPORTED"),      # row-major B
    ({"c": 0x50000}, {}, "ERR_INVALID_ARG"),                  # C is not this rank's buffer
    ({}, {"c_multicast": 0x100000}, "ERR_INVALID_ARG"),      # multicast C without multicast signals
    ({}, {"signal_peers": None}, "ERR_INVALID_ARG"),
])
def test_fused_allreduce_rejects_bad_arguments(gemm_kw, ar_kw, status):
    L = _lib()
    g = _gemm_args(**gemm_kw)
    if ar_kw.get("signal_peers", 1) is None:
        r = _ar_args()
        r.signal_peers[1] = 0
    else:
        r = _ar_args(**ar_kw)
    st = L.lib().b2x_fp8_gemm_allreduce(ctypes.byref(g), ctypes.byref(r), None)
    assert st == getattr(L, status), L.lib().b2x_last_error()
    assert L.lib().b2x_last_error()


def _cast_args(**kw):
    L = _lib()
    a = L.CastArgs()
    a.x, a.x_type, a.rows, a.cols, a.ld_x = 0x10000, L.F32, 64, 256, 256
    a.q, a.q_type, a.ld_q = 0x20000, L.E4M3, 256
    a.scale, a.mode, a.ld_scale = 0x30000, L.SCALE_BLOCK_1x128, 2
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("field,value,status", [
    ("x_type", 2, "ERR_UNSUPPORTED"),   # fp16 input
    ("q_type", 1, "ERR_UNSUPPORTED"),   # bf16 output
    ("x", 0, "ERR_INVALID_ARG"),
    ("ld_x", 100, "ERR_INVALID_ARG"),
    ("ld_scale", 1, "ERR_INVALID_ARG"),
    ("mode", 42, "ERR_INVALID_ARG"),
    ("scale", 0, "ERR_INVALID_ARG"),
])
def test_cast_rejects_bad_arguments(field, value, status):
    L = _lib()
    a = _cast_args(**{field: value})
    assert L.lib().b2x_fp8_cast(ctypes.byref(a), None) == getattr(L, status)


def test_cast_per_tensor_needs_workspace():
    L = _lib()
    a = _cast_args(mode=L.SCALE_TENSOR)
    assert L.lib().b2x_cast_workspace_size(ctypes.byref(a)) > 0
    assert L.lib().b2x_fp8_cast(ctypes.byref(a), None) == L.ERR_WORKSPACE


def test_splitk_reduce_rejects_bad_arguments():
    L = _lib()
    lib = L.lib()
    assert lib.b2x_splitk_reduce(None, L.F32, 0x1000, L.BF16, 4, 4, 4, 2, None) == L.ERR_INVALID_ARG
    assert lib.b2x_splitk_reduce(0x1000, L.E4M3, 0x2000, L.BF16, 4, 4, 4, 2, None) == L.ERR_UNSUPPORTED
    assert lib.b2x_splitk_reduce(0x1000, L.F32, 0x2000, L.BF16, 4, 4, 2, 2, None) == L.ERR_INVALID_ARG


def _default_config(M, N, K, kmajor=True, **cfg):
    L = _lib()
    g = _gemm_args(M=M, N=N, K=K, lda=K, ldc=N)
    if kmajor:
        g.ldb_k, g.ldb_n = 1, K
    else:
        g.ldb_k, g.ldb_n = N, 1
    for k, v in cfg.items():
        setattr(g.config, k, v)
    out = L.GemmConfig()
    assert L.lib().b2x_gemm_default_config(ctypes.byref(g), ctypes.byref(out)) == L.OK
    return out


def test_default_config_large_square_uses_wide_tiles_no_split():
    c = _default_config(8192, 8192, 8192)
    assert (c.block_m, c.block_n, c.block_k, c.split_k) == (128, 256, 128, 1)
    assert c.group_size_m == 8


def test_default_config_decode_uses_split_k():
    c = _default_config(64, 8192, 28672)
    assert c.split_k > 1
    assert (28672 // 128) // c.split_k >= 4
    assert c.group_size_m == 1  # one M tile


def test_default_config_keeps_caller_fields():
    c = _default_config(64, 8192, 28672, split_k=8, block_n=128)
    assert (c.split_k, c.block_n) == (8, 128)
    c = _default_config(4096, 4096, 4096, kmajor=False)
    assert c.block_n >= 128  # row-major B is streamed in 128-column slabs


def test_mx_gemm_rejects_bad_arguments():
    L = _lib()
    lib = L.lib()
    ok = dict(scale_mode=L.SCALE_MX_1x32, scale_a=0x40000, scale_b=0x50000, sa_stride_m=8, sb_stride_n=8)
    g = _gemm_args(**dict(ok, K=192, lda=256))  # K % 128 != 0
    assert lib.b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_UNSUPPORTED
    g = _gemm_args(**dict(ok, sa_stride_m=6))  # scale rows not 4-byte aligned / too short
    assert lib.b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_INVALID_ARG
    g = _gemm_args(**dict(ok, ldb_k=256, ldb_n=1))  # row-major B
    assert lib.b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_UNSUPPORTED
    g = _gemm_args(**ok)
    assert lib.b2x_gemm_workspace_size(ctypes.byref(g)) > 0
    assert lib.b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_WORKSPACE  # scale tiles need a workspace
    g.config.block_n = 256  # MX tiles are 128 or 192 wide
    assert lib.b2x_fp8_gemm(ctypes.byref(g), None) == L.ERR_UNSUPPORTED
    assert b"MX" in lib.b2x_last_error()


def test_mx_default_config_picks_an_mx_tile():
    L = _lib()
    g = _gemm_args(M=8192, N=8192, K=8192, lda=8192, ldc=8192, ldb_n=8192, scale_mode=L.SCALE_MX_1x32)
    out = L.GemmConfig()
    assert L.lib().b2x_gemm_default_config(ctypes.byref(g), ctypes.byref(out)) == L.OK
    assert out.block_n in (128, 192) and out.num_ctas == 1 and out.split_k == 1


def test_grouped_gemm_rejects_bad_arguments():
    L = _lib()
    lib = L.lib()
    assert lib.b2x_grouped_gemm_workspace_size(0) == 0
    ws = lib.b2x_grouped_gemm_workspace_size(2)
    assert ws >= 2 * 3 * 128
    arr = (L.GemmGroup * 2)()
    for g in arr:
        g.a, g.b, g.c = 0x10000, 0x20000, 0x30000
        g.M, g.N, g.K, g.lda, g.ldb, g.ldc = 128, 128, 128, 128, 128, 128
    call = lambda groups, n, bn=0, w=0x40000, wb=ws: lib.b2x_fp8_grouped_gemm(groups, n, L.E4M3, L.E4M3, L.BF16,  # noqa: E731
                                                                            bn, w, wb, None)
    assert call(arr, 0) == L.OK
    assert call(arr, 2, w=0) == L.ERR_WORKSPACE
    assert call(arr, 2, bn=64) == L.ERR_UNSUPPORTED
    arr[1].lda = 100
    assert call(arr, 2) == L.ERR_INVALID_ARG
    arr[1].lda = 128
    arr[0].K = 0
    assert call(arr, 2) == L.ERR_UNSUPPORTED
    assert lib.b2x_fp8_grouped_gemm(arr, 2, L.BF16, L.E4M3, L.BF16, 0, 0x40000, ws, None) == L.ERR_UNSUPPORTED


def test_swiglu_rejects_bad_arguments():
    L = _lib()
    lib = L.lib()
    g = _gemm_args()
    call = lambda g, h=0x60000, ld=128, ht=L.E4M3, m=L.SCALE_BLOCK_1x128, s=0x70000, lds=1: lib.b2x_fp8_gemm_swiglu(  # noqa: E731
        ctypes.byref(g), h, ld, ht, m, s, lds, None, None)
    assert call(g, ht=L.BF16) == L.ERR_UNSUPPORTED
    assert call(g, m=L.SCALE_TENSOR) == L.ERR_UNSUPPORTED
    assert call(_gemm_args(N=384, ldc=384)) == L.ERR_UNSUPPORTED  # 2I not a multiple of 256
    assert call(g, ld=100) == L.ERR_INVALID_ARG
    assert call(g, s=0) == L.ERR_INVALID_ARG
    assert call(_gemm_args(ldb_k=256, ldb_n=1)) == L.ERR_UNSUPPORTED  # row-major B


def test_interleave_gate_up_layout():
    import torch
    from b2x import ops
    wg = torch.arange(256 * 2, dtype=torch.float32).reshape(256, 2)
    wu = -wg
    w = ops.interleave_gate_up(wg, wu)
    assert torch.equal(w[:128], wg[:128]) and torch.equal(w[128:256], wu[:128])
    assert torch.equal(w[256:384], wg[128:]) and torch.equal(w[384:], wu[128:])
