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
