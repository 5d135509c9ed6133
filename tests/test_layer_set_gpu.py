"""The chained Llama-3-70B fp8 linear set at 8192 tokens on one GPU (the
benchmark's workload): qkv = x.Wq^T, h = fp8(silu(x.Wg^T) * (x.Wu^T)) with
the static h scale, out = h.Wd^T.  32 random token rows (and the last) are
checked in full against the float64 oracle:
  * qkv and out rows within the GEMM tolerance (fp8_oracle.gemm_error);
  * h codes equal the oracle's quantization of the oracle's h with the set's
    scale, except neighbouring codes where h lies within 1e-3 relative of the
    rounding boundary (the rule of tests/test_swiglu_gpu.py);
  * out is checked against the kernel's own h (its parity is the line above).
"""
import numpy as np
import pytest
import torch

import fp8_oracle as O

pytestmark = pytest.mark.gpu


def _deq(t, s):
    return O.fp8_bits_to_f64(t.view(torch.uint8).cpu().numpy(), O.E4M3) * float(s)


def test_chained_layer_set_sampled():
    import b2x
    from b2x.sharded import LlamaFP8LinearSet
    from test_swiglu_gpu import _check_codes
    dev = torch.device("cuda", 0)
    ls = LlamaFP8LinearSet(0, 1, dev)
    before = b2x.launch_count()
    q, h, d = ls.step()
    torch.cuda.synchronize()
    assert b2x.launch_count() - before == 3, "qkv, gate+up+SwiGLU and down: three libb2x kernels"
    g = torch.Generator(device="cuda").manual_seed(3)
    rows = torch.cat([torch.randperm(8192, device="cuda", generator=g)[:32], torch.tensor([8191], device="cuda")])
    xs = _deq(ls.x[rows], ls.sx.item())
    # qkv rows
    wq = _deq(ls.wq, ls.sq.item())
    ref_q = xs @ wq.T
    err, tol = O.gemm_error(q[rows].float().cpu().numpy(), ref_q, xs, wq.T)
    assert err <= tol, f"qkv: {err} > {tol}"
    del wq
    # h rows: silu(g) * u from the interleaved gate/up weight
    wgu = _deq(ls.wgu, ls.sgu.item())
    y = (xs @ wgu.T).reshape(xs.shape[0], -1, 2, 128)
    gg, uu = y[:, :, 0], y[:, :, 1]
    href = (gg / (1.0 + np.exp(-gg)) * uu).reshape(xs.shape[0], -1)
    del wgu, y
    sh = float(ls.sh.item())
    _check_codes(h[rows].view(torch.uint8).cpu().numpy(), href / sh)
    # down rows from the kernel's own h
    hs = _deq(h[rows], sh)
    wd = _deq(ls.wd, ls.sd.item())
    ref_d = hs @ wd.T
    err, tol = O.gemm_error(d[rows].float().cpu().numpy(), ref_d, hs, wd.T)
    assert err <= tol, f"down: {err} > {tol}"
    assert b2x.read_device_status() == 0
