"""Multi-rank partitioning of the fp8 linear set, checked on CPU with two gloo
ranks: column-parallel shards concatenate to the unsharded product, and the
row-parallel partials all-reduce to it.  The GEMM is a float64 CPU stand-in
(the sharding logic, not the kernel, is under test here)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mm(a, w, sa, sw, cfg):
    return (a.double() @ w.double().t()) * float(sa) * float(sw)


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from b2x import sharded
        g = torch.Generator().manual_seed(0)
        M, K, N, Kd = 16, 64, 96, 128
        x = torch.randn(M, K, generator=g)
        w = torch.randn(N, K, generator=g)
        a2 = torch.randn(M, Kd, generator=g)
        wd = torch.randn(N, Kd, generator=g)
        sx, sw = torch.tensor(0.5), torch.tensor(2.0)
        # column-parallel: gather the column shards and compare with the full product
        part = sharded.column_parallel(x, sx, sharded.shard_rows(w, rank, world), sw, mm=_mm)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        full = torch.cat(parts, dim=1)
        ok_col = torch.allclose(full, _mm(x, w, sx, sw, None), rtol=1e-12, atol=1e-10)
        # row-parallel: partials all-reduced over the K shards
        d = sharded.row_parallel(sharded.shard_cols(a2, rank, world), sx, sharded.shard_cols(wd, rank, world), sw,
                                 mm=_mm)
        ok_row = torch.allclose(d, _mm(a2, wd, sx, sw, None), rtol=1e-10, atol=1e-9)
        lo, hi = sharded.shard_range(N, rank, world)
        q.put((rank, bool(ok_col), bool(ok_row), (lo, hi)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, False, repr(e)))


def _swiglu(x, w, sx, sw, h_scale, h_amax=None):
    """float64 stand-in of gemm_swiglu on the interleaved gate/up weight."""
    y = (x.double() @ w.double().t()) * float(sx) * float(sw)
    y = y.reshape(y.shape[0], -1, 2, 128)
    g, u = y[:, :, 0], y[:, :, 1]
    h = (g * torch.sigmoid(g) * u).reshape(y.shape[0], -1)
    if h_amax is not None:
        h_amax.copy_(h.abs().max().float().reshape(1))
    return h / float(h_scale)


def _rand(shape, gen, device):
    return torch.randn(shape, generator=gen, dtype=torch.float64), torch.tensor(0.5)


def _chain_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from b2x import sharded

        class Small(sharded.LlamaFP8LinearSet):
            SHAPES = {"qkv": (16, 64, 32), "gate_up": (16, 512, 32), "down": (16, 48, 256)}

        ls = Small(rank, world, "cpu", tokens=16, mm=_mm, swiglu=_swiglu, make_input=_rand)
        qo, h, d = ls.step()

        def gather(t, dim):
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous())
            return torch.cat(parts, dim=dim)

        wq, wgu, wd = gather(ls.wq, 0), gather(ls.wgu, 0), gather(ls.wd, 1)
        ok_q = torch.allclose(gather(qo, 1), _mm(ls.x, wq, ls.sx, ls.sq, None), rtol=1e-12, atol=1e-10)
        h_full = _swiglu(ls.x, wgu, ls.sx, ls.sgu, 1.0)
        ok_h = torch.allclose(gather(h * ls.sh, 1), h_full, rtol=1e-12, atol=1e-10)
        ok_d = torch.allclose(d, _mm(h_full, wd, 1.0, ls.sd, None), rtol=1e-10, atol=1e-9)
        q.put((rank, bool(ok_q and ok_h and ok_d), (bool(ok_q), bool(ok_h), bool(ok_d))))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def test_two_rank_chained_layer_set_matches_unsharded():
    """LlamaFP8LinearSet on two gloo ranks with float64 stand-ins for the
    kernels: gathered QKV and h shards, and the all-reduced down output,
    equal the unsharded chain qkv = x.Wq^T, h = silu(x.Wg^T)*(x.Wu^T),
    out = h.Wd^T."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_chain_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in results:
        assert ok, (rank, info)


def test_two_rank_sharding_matches_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    results.sort()
    for rank, ok_col, ok_row, info in results:
        assert ok_col and ok_row, (rank, info)
    assert [r[3] for r in results] == [(0, 48), (48, 96)]


def test_shard_range_rejects_uneven_split():
    from b2x import sharded
    with pytest.raises(ValueError):
        sharded.shard_range(10, 0, 3)
    assert sharded.shard_range(57344, 7, 8) == (7 * 7168, 8 * 7168)
