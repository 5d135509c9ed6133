"""GPU parity of the row-parallel fp8 GEMM with its all-reduce fused into the
kernel (b2x_fp8_gemm_allreduce), on 2 or more GPUs of one node.

Every rank r holds the K-slice (A_r, B_r) of a row-parallel layer and gets
C = sum_r A_r . B_r back.  The expected value is the float64 oracle sum of
the ranks' partial GEMMs.  Tolerance: each partial may carry its GEMM error
bound (fp8_oracle.gemm_tolerance) plus the rounding of that partial to bf16,
and the sum its own bf16 rounding:
    max(|C - ref| - 2^-8 (|ref| + sum_r |P_r|)) <= sum_r tol_r.
Both reduction modes run when the node offers them (NVSwitch multicast and
peer loads/stores), over several consecutive calls on the same buffers (the
arrival counters must come back to zero and the done word advance by the
unit count per call).  Ranks run as child processes, one per GPU, over NCCL.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_inputs(M, N, Kr, rank, call, fmt_a, fmt_b, scaled):
    import fp8_oracle as O
    rng = np.random.default_rng(1000 * call + rank)
    a = rng.standard_normal((M, Kr), dtype=np.float32)
    w = rng.standard_normal((N, Kr), dtype=np.float32)
    mode = "tensor" if scaled else "none"
    qa, sa = O.quantize(a, mode, fmt_a)
    qw, sw = O.quantize(0.5 * w if not scaled else w, mode, fmt_b)
    return qa, (np.float32(sa) if scaled else None), qw, (np.float32(sw) if scaled else None)


def _expected(M, N, Kr, world, call, fmt_a, fmt_b, scaled):
    import fp8_oracle as O
    ref = np.zeros((M, N))
    abs_parts = np.zeros((M, N))
    tol = 0.0
    for r in range(world):
        qa, sa, qw, sw = _rank_inputs(M, N, Kr, r, call, fmt_a, fmt_b, scaled)
        p = O.gemm(qa, qw.T, fmt_a, fmt_b, "tensor" if scaled else "none", sa, sw)
        ref += p
        abs_parts += np.abs(p)
        a_deq = O.fp8_bits_to_f64(qa, fmt_a) * (float(sa) if scaled else 1.0)
        b_deq = O.fp8_bits_to_f64(qw.T, fmt_b) * (float(sw) if scaled else 1.0)
        tol += O.gemm_tolerance(a_deq, b_deq)
    return ref, abs_parts, tol


def _worker(rank, world, port, q, cases):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as dist
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        import b2x
        import fp8_oracle as O
        from b2x import _lib as L
        from b2x.sharded import FusedRowParallel
        FP8 = {O.E4M3: torch.float8_e4m3fn, O.E5M2: torch.float8_e5m2}
        out = []
        for (M, N, Kr, mode, fmt_a, fmt_b, scaled, calls) in cases:
            fr = FusedRowParallel(M, N, dev, mode=mode)
            lib = L.lib()
            units = int(lib.b2x_allreduce_signal_words(M, N)) - 64
            for call in range(calls):
                qa, sa, qw, sw = _rank_inputs(M, N, Kr, rank, call, fmt_a, fmt_b, scaled)
                A = torch.from_numpy(qa).to(dev).view(FP8[fmt_a])
                W = torch.from_numpy(qw).to(dev).view(FP8[fmt_b])
                tsa = torch.tensor([sa], device=dev) if scaled else None
                tsw = torch.tensor([sw], device=dev) if scaled else None
                torch.cuda.synchronize(dev)
                dist.barrier()  # no rank's kernel waits on a peer still busy on the host
                before = b2x.launch_count()
                C = fr(A, tsa, W, tsw)
                torch.cuda.synchronize(dev)
                launched = b2x.launch_count() - before
                status = L.read_device_status()
                c = C.float().cpu().numpy()
                err = None
                if rank == 0 or call == calls - 1:
                    ref, abs_parts, tol = _expected(M, N, Kr, world, call, fmt_a, fmt_b, scaled)
                    excess = float((np.abs(c - ref) - O.OUTPUT_ROUNDING * (np.abs(ref) + abs_parts)).max())
                    err = (excess, float(tol))
                sig = fr.signal.cpu().numpy().astype(np.int64) & 0xFFFFFFFF
                out.append(dict(case=(M, N, Kr, fr.mode, fmt_a, fmt_b, scaled), call=call, err=err,
                                launched=launched, status=status,
                                arrive_zero=bool((sig[64:64 + units] == 0).all()),
                                done=int(sig[0]), done_expected=(call + 1) * units,
                                calls_counted=int(sig[2]), finite=bool(np.isfinite(c).all())))
            # the same call captured once in a CUDA graph and replayed: the
            # kernel counts the calls itself, so every replay is a new call
            qa, sa, qw, sw = _rank_inputs(M, N, Kr, rank, calls - 1, fmt_a, fmt_b, scaled)
            A = torch.from_numpy(qa).to(dev).view(FP8[fmt_a])
            W = torch.from_numpy(qw).to(dev).view(FP8[fmt_b])
            tsa = torch.tensor([sa], device=dev) if scaled else None
            tsw = torch.tensor([sw], device=dev) if scaled else None
            torch.cuda.synchronize(dev)
            dist.barrier()
            s_cap = torch.cuda.Stream(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s_cap):
                with torch.cuda.graph(graph, stream=s_cap):
                    fr(A, tsa, W, tsw)
            for rep in range(3):
                fr.out.fill_(float("nan"))
                torch.cuda.synchronize(dev)
                dist.barrier()
                graph.replay()
                torch.cuda.synchronize(dev)
                status = L.read_device_status()
                c = fr.out.float().cpu().numpy()
                ref, abs_parts, tol = _expected(M, N, Kr, world, calls - 1, fmt_a, fmt_b, scaled)
                excess = float((np.abs(c - ref) - O.OUTPUT_ROUNDING * (np.abs(ref) + abs_parts)).max())
                sig = fr.signal.cpu().numpy().astype(np.int64) & 0xFFFFFFFF
                out.append(dict(case=(M, N, Kr, fr.mode, fmt_a, fmt_b, scaled, "graph"), call=calls + rep,
                                err=(excess, float(tol)), launched=1, status=status,
                                arrive_zero=bool((sig[64:64 + units] == 0).all()),
                                done=int(sig[0]), done_expected=(calls + rep + 1) * units,
                                calls_counted=int(sig[2]), finite=bool(np.isfinite(c).all())))
            del graph, fr
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))


def _run(world, cases, timeout=600):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, cases)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, out, tb = q.get(timeout=timeout)
            results[r] = (out, tb)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r, (out, tb) in sorted(results.items()):
        assert tb is None, f"rank {r} failed:\n{tb}"
    return results


def _world():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    return min(n, 8)


def _check(results):
    for r, (out, _) in sorted(results.items()):
        for rec in out:
            what = f"rank {r} {rec['case']} call {rec['call']}"
            assert rec["status"] == 0, f"{what}: device status {rec['status']:#x}"
            assert rec["launched"] == 1, f"{what}: expected one fused kernel launch, saw {rec['launched']}"
            assert rec["finite"], what
            if rec["err"] is not None:
                excess, tol = rec["err"]
                assert excess <= tol, f"{what}: error {excess:.4g} > tol {tol:.4g}"
            assert rec["arrive_zero"], f"{what}: arrival counters not reset"
            assert rec["done"] == rec["done_expected"], f"{what}: done word {rec['done']} != {rec['done_expected']}"
            assert rec["calls_counted"] == rec["call"] + 1, f"{what}: call count {rec['calls_counted']}"


def test_fused_allreduce_modes_and_repeats():
    import fp8_oracle as O
    world = _world()
    cases = [
        # M, N, K per rank, mode, fmt A, fmt B, per-tensor scales, consecutive calls
        (512, 768, 384, "peer", O.E4M3, O.E4M3, True, 3),
        (256, 256, 128, "peer", O.E4M3, O.E4M3, False, 2),
        (512, 512, 256, "peer", O.E5M2, O.E4M3, True, 1),
        (512, 768, 384, "auto", O.E4M3, O.E4M3, True, 3),
        (768, 1024, 640, "auto", O.E4M3, O.E5M2, True, 2),
    ]
    _check(_run(world, cases))


def test_fused_allreduce_bench_shape_rows():
    """The benchmark's down projection (8192 x 8192, K = 28672 split over the
    ranks), on a 1024-row slice so the float64 oracle stays quick."""
    import fp8_oracle as O
    world = _world()
    cases = [(1024, 8192, 28672 // world, "auto", O.E4M3, O.E4M3, True, 2)]
    _check(_run(world, cases, timeout=900))
