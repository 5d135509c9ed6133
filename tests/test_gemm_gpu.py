"""GPU parity of the tcgen05 fp8 GEMM (libb2x) against the float64 CPU oracle.

Tolerance (the accuracy target of this path): max |C - C_ref| <= 1e-2 * ||A|| * ||B|| / sqrt(K),
with ||A|| the largest row 2-norm of the dequantized A and ||B|| the largest
column 2-norm of the dequantized B, on top of the rounding of C to bf16
(2^-8 * |C_ref| per element; fp8_oracle.gemm_error).  Split-K must agree with
the non-split result within the same bound.
"""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu

FP8 = {O.E4M3: torch.float8_e4m3fn, O.E5M2: torch.float8_e5m2}


def _b2x():
    import b2x
    return b2x


def _quant(shape, fmt, seed, scale_mode="tensor"):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape, dtype=np.float32)
    if scale_mode == "tensor":
        q, s = O.quantize(x, "tensor", fmt)
    else:
        q, s = O.quantize(x, "none", fmt)
        s = np.float32(1.0)
    return q, np.float32(s)


def _dev_fp8(bits, fmt):
    return torch.from_numpy(np.ascontiguousarray(bits)).cuda().view(FP8[fmt])


def _check(c, ref, a_deq, b_deq, what=""):
    err, tol = O.gemm_error(c, ref, a_deq, b_deq)
    assert err <= tol, f"{what}: error beyond bf16 output rounding {err:.4g} > tol {tol:.4g}"
    return err, tol


def _gemm(a_bits, b_bits_kn, a_fmt, b_fmt, sa, sb, b_layout="kmajor", config=None, out_dtype=torch.bfloat16):
    b2x = _b2x()
    A = _dev_fp8(a_bits, a_fmt)
    if b_layout == "kmajor":
        B = _dev_fp8(np.ascontiguousarray(b_bits_kn.T), b_fmt).t()  # [K, N] view of an [N, K] weight
    else:
        B = _dev_fp8(b_bits_kn, b_fmt)  # row-major [K, N]
    before = b2x.launch_count()
    C = b2x.matmul(A, B, config, scale_a=torch.tensor([sa], device="cuda"),
                   scale_b=torch.tensor([sb], device="cuda"), out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert b2x.launch_count() > before, "no libb2x kernel ran"
    return C.float().cpu().numpy()


SHAPES = [(128, 256, 128), (256, 512, 1024), (384, 768, 512), (1, 64, 128), (200, 304, 272), (64, 256, 16),
          (130, 136, 4096), (512, 512, 512)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("b_layout", ["kmajor", "rowmajor"])
def test_gemm_e4m3_vs_oracle(shape, b_layout):
    M, N, K = shape
    a, sa = _quant((M, K), O.E4M3, 1)
    b, sb = _quant((K, N), O.E4M3, 2)
    ref = O.gemm(a, b, scale_mode="tensor", scale_a=sa, scale_b=sb)
    c = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, b_layout, config={})
    _check(c, ref, O.fp8_bits_to_f64(a, O.E4M3) * sa, O.fp8_bits_to_f64(b, O.E4M3) * sb, f"{shape} {b_layout}")


@pytest.mark.parametrize("fa,fb", [(O.E5M2, O.E4M3), (O.E4M3, O.E5M2), (O.E5M2, O.E5M2)])
def test_gemm_mixed_formats(fa, fb):
    M, N, K = 256, 512, 640
    a, sa = _quant((M, K), fa, 3)
    b, sb = _quant((K, N), fb, 4)
    ref = O.gemm(a, b, fa, fb, scale_mode="tensor", scale_a=sa, scale_b=sb)
    c = _gemm(a, b, fa, fb, sa, sb, "kmajor", config={})
    _check(c, ref, O.fp8_bits_to_f64(a, fa) * sa, O.fp8_bits_to_f64(b, fb) * sb, f"{fa}x{fb}")


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_block_n_variants_and_fp16_out(bn):
    M, N, K = 300, 520, 1024
    a, sa = _quant((M, K), O.E4M3, 5)
    b, sb = _quant((K, N), O.E4M3, 6)
    ref = O.gemm(a, b, scale_mode="tensor", scale_a=sa, scale_b=sb)
    for out in (torch.bfloat16, torch.float16):
        c = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, "kmajor", config={"BLOCK_SIZE_N": bn}, out_dtype=out)
        _check(c, ref, O.fp8_bits_to_f64(a, O.E4M3) * sa, O.fp8_bits_to_f64(b, O.E4M3) * sb, f"bn={bn} {out}")


@pytest.mark.parametrize("split_k", [2, 3, 4, 8])
@pytest.mark.parametrize("b_layout", ["kmajor", "rowmajor"])
def test_splitk_matches_oracle_and_nonsplit(split_k, b_layout):
    M, N, K = 64, 1024, 4096
    a, sa = _quant((M, K), O.E4M3, 7)
    b, sb = _quant((K, N), O.E4M3, 8)
    ref = O.gemm(a, b, scale_mode="tensor", scale_a=sa, scale_b=sb)
    ad, bd = O.fp8_bits_to_f64(a, O.E4M3) * sa, O.fp8_bits_to_f64(b, O.E4M3) * sb
    c1 = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, b_layout, config={"SPLIT_K": 1, "BLOCK_SIZE_N": 128})
    for rep in range(2):  # second call re-uses the (self-cleaning) workspace
        cs = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, b_layout, config={"SPLIT_K": split_k, "BLOCK_SIZE_N": 128})
        _check(cs, ref, ad, bd, f"split_k={split_k} rep={rep}")
        _check(cs, c1.astype(np.float64), ad, bd, "split vs non-split")
    from b2x import ops
    for key, buf in ops._ws_cache.items():
        if key[2]:  # the zero-invariant split-K workspaces (not the amax partials)
            assert int(buf.count_nonzero().item()) == 0, "split-K workspace not left zeroed"


@pytest.mark.parametrize("shape", [(256, 256, 256), (384, 520, 1024), (129, 1000, 640), (1000, 256, 4096)])
@pytest.mark.parametrize("b_layout", ["kmajor", "rowmajor"])
def test_paired_cta_matches_single_cta_and_oracle(shape, b_layout):
    """NUM_CTAS=2 (cta_group::2 256x256 tiles over two SMs) against NUM_CTAS=1 and the oracle."""
    M, N, K = shape
    a, sa = _quant((M, K), O.E4M3, 21)
    b, sb = _quant((K, N), O.E4M3, 22)
    ref = O.gemm(a, b, scale_mode="tensor", scale_a=sa, scale_b=sb)
    ad, bd = O.fp8_bits_to_f64(a, O.E4M3) * sa, O.fp8_bits_to_f64(b, O.E4M3) * sb
    c2 = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, b_layout, config={"NUM_CTAS": 2, "BLOCK_SIZE_N": 256})
    c1 = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, b_layout, config={"NUM_CTAS": 1, "BLOCK_SIZE_N": 256})
    _check(c2, ref, ad, bd, f"pair {shape} {b_layout}")
    _check(c1, ref, ad, bd, f"single {shape} {b_layout}")
    assert b2x_status_ok()


def b2x_status_ok():
    return _b2x().read_device_status() == 0


@pytest.mark.parametrize("M", [1, 7, 16, 17, 33, 64])
@pytest.mark.parametrize("split_k", [1, 3])
@pytest.mark.parametrize("b_layout", ["kmajor", "rowmajor"])
def test_small_m_paths(M, split_k, b_layout):
    """M <= 64: the operand-swapped kernel (K-major B) and the 64-row-A kernel (row-major B)."""
    N, K = 520, 2048
    a, sa = _quant((M, K), O.E4M3, 31 + M)
    b, sb = _quant((K, N), O.E4M3, 32)
    ref = O.gemm(a, b, scale_mode="tensor", scale_a=sa, scale_b=sb)
    ad, bd = O.fp8_bits_to_f64(a, O.E4M3) * sa, O.fp8_bits_to_f64(b, O.E4M3) * sb
    for rep in range(2):
        c = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, b_layout, config={"SPLIT_K": split_k})
        _check(c, ref, ad, bd, f"M={M} split={split_k} {b_layout} rep={rep}")


def test_splitk_decode_shape_full():
    """Decode benchmark configuration: M=64 N=8192 K=28672, SPLIT_K=8, per-tensor e4m3, bf16 out.
    Checked against the oracle on a sample of 512 output columns."""
    M, N, K = 64, 8192, 28672
    a, sa = _quant((M, K), O.E4M3, 9)
    b, sb = _quant((K, N), O.E4M3, 10)
    c = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, "kmajor", config={"SPLIT_K": 8})
    c1 = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, "kmajor", config={"SPLIT_K": 1})
    cols = np.random.default_rng(0).choice(N, 512, replace=False)
    ad = O.fp8_bits_to_f64(a, O.E4M3).astype(np.float32) * sa
    bd = O.fp8_bits_to_f64(b[:, cols], O.E4M3).astype(np.float32) * sb
    ref = ad.astype(np.float64) @ bd.astype(np.float64)
    _check(c[:, cols], ref, ad, bd, "decode split-K")
    _check(c, c1.astype(np.float64), ad, bd, "decode split vs non-split")


def test_gemm_512_config0():
    """The CPU-runnable benchmark configuration: 512^3, A,B ~N(0,1) per-tensor e4m3, bf16 out."""
    a, sa = _quant((512, 512), O.E4M3, 0)
    b, sb = _quant((512, 512), O.E4M3, 1)
    ref = O.gemm(a, b, scale_mode="tensor", scale_a=sa, scale_b=sb)
    for layout in ("kmajor", "rowmajor"):
        c = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, layout)
        _check(c, ref, O.fp8_bits_to_f64(a, O.E4M3) * sa, O.fp8_bits_to_f64(b, O.E4M3) * sb, layout)


def test_gemm_8192_sampled():
    """8192^3 (the perf shape): a sampled 256 x 256 block against the oracle."""
    b2x = _b2x()
    M = N = K = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    xa = torch.randn((M, K), device="cuda", generator=g)
    xb = torch.randn((N, K), device="cuda", generator=g)
    A, sa = b2x.quantize(xa, "tensor", torch.float8_e4m3fn)
    W, sb = b2x.quantize(xb, "tensor", torch.float8_e4m3fn)
    C = b2x.matmul(A, W.t(), {}, scale_a=sa, scale_b=sb).float()
    rows = torch.randperm(M, device="cuda", generator=g)[:256]
    cols = torch.randperm(N, device="cuda", generator=g)[:256]
    a_bits = A[rows].view(torch.uint8).cpu().numpy()
    b_bits = W[cols].view(torch.uint8).cpu().numpy().T
    ref = O.gemm(a_bits, b_bits, scale_mode="tensor", scale_a=sa.item(), scale_b=sb.item())
    got = C[rows][:, cols].cpu().numpy()
    _check(got, ref, O.fp8_bits_to_f64(a_bits, O.E4M3) * sa.item(), O.fp8_bits_to_f64(b_bits, O.E4M3) * sb.item(),
           "8192^3 sample")


def _block_inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    xa = rng.standard_normal((M, K), dtype=np.float32)
    xw = rng.standard_normal((N, K), dtype=np.float32)  # weight [N, K]
    qa, sa = O.quantize(xa, "block1x128", O.E4M3)       # sa [M, K/128]
    qw, sw = O.quantize(xw, "block128x128", O.E4M3)     # sw [N/128, K/128]
    return qa, sa, qw, sw


@pytest.mark.parametrize("shape", [(256, 384, 512), (200, 256, 1000), (128, 128, 128)])
def test_blockscaled_vs_oracle(shape):
    b2x = _b2x()
    M, N, K = shape
    qa, sa, qw, sw = _block_inputs(M, N, K, 11)
    sb_kn = sw.T  # [K/128, N/128]
    ref = O.gemm(qa, qw.T, scale_mode="block", scale_a=sa, scale_b=sb_kn)
    A = _dev_fp8(qa, O.E4M3)
    W = _dev_fp8(qw, O.E4M3)
    C = b2x.matmul(A, W.t(), {}, scale_a=torch.from_numpy(sa).cuda(),
                   scale_b=torch.from_numpy(sw).cuda().t()).float().cpu().numpy()
    ad = O.fp8_bits_to_f64(qa, O.E4M3) * np.repeat(sa, 128, axis=1)[:, :K]
    bd = (O.fp8_bits_to_f64(qw, O.E4M3) * np.repeat(np.repeat(sw, 128, 0), 128, 1)[:N, :K]).T
    _check(C, ref, ad, bd, f"block {shape}")


def test_blockscaled_config2_sampled():
    """The block-scaled benchmark configuration: 4096 x 7168 x 7168, A 1x128 scales, B 128x128 scales."""
    b2x = _b2x()
    M, N, K = 4096, 7168, 7168
    g = torch.Generator(device="cuda").manual_seed(2)
    A, sa = b2x.quantize(torch.randn((M, K), device="cuda", generator=g), "block1x128", torch.float8_e4m3fn)
    W, sw = b2x.quantize(torch.randn((N, K), device="cuda", generator=g), "block128x128", torch.float8_e4m3fn)
    C = b2x.matmul(A, W.t(), {}, scale_a=sa, scale_b=sw.t()).float()
    rows = torch.randperm(M, device="cuda", generator=g)[:128]
    qa = A[rows].view(torch.uint8).cpu().numpy()
    qw = W.view(torch.uint8).cpu().numpy()
    cols = np.arange(0, N, 7)[:512]
    # per-column B scales depend on the column's 128-wide tile: build the sampled scale grid
    swn = sw.cpu().numpy()
    sa_np = sa[rows].cpu().numpy()
    Aq = O.fp8_bits_to_f64(qa, O.E4M3)
    Bq = O.fp8_bits_to_f64(qw[cols], O.E4M3)  # [ncols, K]
    ref = np.zeros((len(rows), len(cols)))
    for kb in range(K // 128):
        ks = slice(kb * 128, kb * 128 + 128)
        ref += (Aq[:, ks] @ Bq[:, ks].T) * sa_np[:, kb][:, None] * swn[cols // 128, kb][None, :]
    got = C[rows][:, torch.from_numpy(cols).cuda()].cpu().numpy()
    ad = Aq * np.repeat(sa_np, 128, axis=1)
    bd = (Bq * np.repeat(swn[cols // 128], 128, axis=1)).T
    _check(got, ref, ad, bd, "config2 sample")


def test_reduce_k_reference_semantics():
    b2x = _b2x()
    M, N, S = 100, 72, 3
    ws = torch.randn((S * M, N), device="cuda", dtype=torch.bfloat16)
    c = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    b2x.reduce_k(ws, c, M, N, S)
    ref = ws.float().reshape(S, M, N).sum(0).to(torch.bfloat16)
    assert torch.equal(c, ref)


def test_errors_are_raised_not_faulted():
    b2x = _b2x()
    A = torch.zeros((128, 128), device="cuda", dtype=torch.float8_e4m3fn)
    with pytest.raises(AssertionError):
        b2x.matmul(A, torch.zeros((64, 128), device="cuda", dtype=torch.float8_e4m3fn))
    with pytest.raises(NotImplementedError):
        b2x.matmul(torch.zeros((8, 8), device="cuda", dtype=torch.float16),
                   torch.zeros((8, 8), device="cuda", dtype=torch.float16))
    rowmajor_b = torch.zeros((128, 128), device="cuda", dtype=torch.float8_e4m3fn)
    with pytest.raises(b2x.B2XError):  # block scales need a K-major B
        b2x.matmul(A, rowmajor_b, {}, scale_a=torch.ones((128, 1), device="cuda"),
                   scale_b=torch.ones((1, 1), device="cuda"))
    assert b2x.read_device_status() == 0


@pytest.mark.parametrize("M,N,K", [(64, 8192, 28672), (16, 1000, 3000), (33, 4096, 7168), (1, 256, 128)])
def test_stream_k_decode(M, N, K):
    """SPLIT_K = -1 (stream-K): K blocks of all tiles cut into one equal range
    per SM, so ranges cross tile boundaries and a tile is summed from a
    varying number of pieces.  Against the oracle (sampled columns for the
    decode benchmark shape) and against non-split, three calls in a row (the
    workspace and the tile counters must come back clean)."""
    a, sa = _quant((M, K), O.E4M3, 40 + M)
    b, sb = _quant((K, N), O.E4M3, 41)
    c1 = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, "kmajor", config={"SPLIT_K": 1})
    cols = np.random.default_rng(1).choice(N, min(N, 512), replace=False)
    ad = O.fp8_bits_to_f64(a, O.E4M3) * sa
    bd = O.fp8_bits_to_f64(b[:, cols], O.E4M3) * sb
    ref = ad @ bd
    for rep in range(3):
        c = _gemm(a, b, O.E4M3, O.E4M3, sa, sb, "kmajor", config={"SPLIT_K": -1})
        _check(c[:, cols], ref, ad, bd, f"stream-K {M}x{N}x{K} rep={rep}")
        _check(c, c1.astype(np.float64), ad, O.fp8_bits_to_f64(b, O.E4M3) * sb, "stream-K vs non-split")
    assert _b2x().read_device_status() == 0
