"""Multi-GPU partitioning of fp8 linear layers (one process per GPU).

The reference has no multi-GPU code; the benchmark's layer set (Llama-3-70B
shapes at 8192 tokens) is partitioned the way tensor-parallel MLP/attention
projections are:

* column-parallel (QKV, gate+up): each rank holds rows [r*N/g, (r+1)*N/g) of
  the [N, K] weight and computes its slice of the output columns -- no
  collective (the gate+up output stays column-sharded, which is exactly the
  K-sharding the down projection consumes);
* row-parallel (down): each rank holds columns [r*K/g, (r+1)*K/g) of the
  [N, K] weight and the matching K-slice of the input, computes a partial
  [M, N] output and the partials are summed over the group.  On GPUs the sum
  is fused into the GEMM kernel (FusedRowParallel: every 128 x 256 output
  unit is reduced over NVSwitch multicast or NVLink peer memory as soon as
  the last rank has stored it); `row_parallel` with an NCCL all-reduce after
  the GEMM is the unfused form.

The GEMM is injectable (`mm`) so the partitioning logic can be checked on
CPU ranks (gloo) against an unsharded product.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int):
    """[lo, hi) of the rank's contiguous share of n items (n divisible by world)."""
    if n % world:
        raise ValueError(f"{n} does not split evenly over {world} ranks")
    step = n // world
    return rank * step, (rank + 1) * step


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Column-parallel shard of a [N, K] weight: its rows for this rank."""
    lo, hi = shard_range(w.shape[0], rank, world)
    return w[lo:hi].contiguous()


def shard_cols(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Row-parallel shard of a [*, K] tensor: its K-slice for this rank."""
    lo, hi = shard_range(x.shape[-1], rank, world)
    return x[..., lo:hi].contiguous()


def _default_mm(a, w, sa, sw, cfg):
    from .blackwell_gemm_ws import matmul
    return matmul(a, w.t(), cfg, scale_a=sa, scale_b=sw)


def column_parallel(x, sx, w_shard, sw, mm: Callable = _default_mm, cfg: Optional[dict] = None):
    """Local output columns: x [M, K] . w_shard[N/g, K]^T -> [M, N/g]."""
    return mm(x, w_shard, sx, sw, cfg if cfg is not None else {})


def row_parallel(a_shard, sa, w_shard, sw, group=None, mm: Callable = _default_mm, cfg: Optional[dict] = None,
                 async_op: bool = False):
    """Partial a_shard [M, K/g] . w_shard [N, K/g]^T summed over the group.
    With async_op=True returns (partial, work) and the caller waits."""
    part = mm(a_shard, w_shard, sa, sw, cfg if cfg is not None else {})
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        work = dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
        if async_op:
            return part, work
    return (part, None) if async_op else part


class FusedRowParallel:
    """Row-parallel fp8 GEMM with the all-reduce of its output inside the GEMM
    kernel (include/b2x.h, b2x_fp8_gemm_allreduce).

    Owns, per process group and output shape, a bf16 [M, N] output buffer and
    a small signal buffer in symmetric memory (every rank maps every rank's
    copy; with NVSwitch multicast support one multicast address covers all
    copies).  Each call returns the output buffer itself: the next call
    overwrites it.  All ranks must make the same calls in the same order.

    mode: "auto" (multicast when the group supports it, else peer loads and
    stores), "multicast" or "peer".

    Failure handling: the kernel's waits for peers are bounded (10 s).  A
    wait that gives up records a timeout in the device status word and can
    leave the arrival counters of the signal buffer partly counted, which a
    later call would misread.  `check()` (collective: every rank calls it)
    reads the status on every rank and, if any rank timed out, zeroes the
    signal buffers everywhere and raises B2XError.
    `reset()` does the clearing alone.  The calls are counted by the kernel
    in the signal buffer (epoch 0 in the C arguments), so a call has no
    per-call host state and can be captured in a CUDA graph.
    """

    def __init__(self, M: int, N: int, device, group=None, mode: str = "auto"):
        import torch.distributed._symmetric_memory as symm_mem
        from . import _lib as L
        self.M, self.N = M, N
        self.device = torch.device(device)
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > L.AR_MAX_RANKS:
            raise ValueError(f"fused all-reduce supports at most {L.AR_MAX_RANKS} ranks, got {self.world}")
        words = int(L.lib().b2x_allreduce_signal_words(M, N))
        self.out = symm_mem.empty((M, N), dtype=torch.bfloat16, device=self.device)
        self.signal = symm_mem.empty((words,), dtype=torch.int32, device=self.device)
        self.signal.zero_()
        name = self.group.group_name
        h_out = symm_mem.rendezvous(self.out, name)
        h_sig = symm_mem.rendezvous(self.signal, name)
        use_mc = mode == "multicast" or (mode == "auto" and bool(h_out.has_multicast_support)
                                         and bool(h_sig.has_multicast_support))
        if mode not in ("auto", "multicast", "peer"):
            raise ValueError(f"mode must be auto, multicast or peer, got {mode!r}")
        if use_mc and not (h_out.multicast_ptr and h_sig.multicast_ptr):
            raise RuntimeError("NVSwitch multicast is not available for this group")
        self.mode = "multicast" if use_mc else "peer"
        ar = L.AllReduceArgs()
        ar.rank, ar.world = self.rank, self.world
        off_c = self.out.data_ptr() - h_out.buffer_ptrs[self.rank]
        off_s = self.signal.data_ptr() - h_sig.buffer_ptrs[self.rank]
        for r in range(self.world):
            ar.c_peers[r] = h_out.buffer_ptrs[r] + off_c
            ar.signal_peers[r] = h_sig.buffer_ptrs[r] + off_s
        if use_mc:
            ar.c_multicast = h_out.multicast_ptr + off_c
            ar.signal_multicast = h_sig.multicast_ptr + off_s
        self._ar = ar
        self._handles = (h_out, h_sig)
        self._plans = {}  # GEMM argument structs per (operands, config): the host cost of a repeat call is one C call
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)  # every rank's signal buffer is zero before any kernel runs

    def __call__(self, a_shard: torch.Tensor, sa: Optional[torch.Tensor], w_shard: torch.Tensor,
                 sw: Optional[torch.Tensor], cfg: Optional[dict] = None) -> torch.Tensor:
        """sum over ranks of a_shard [M, K/g] . w_shard [N, K/g]^T (fp8, per-tensor
        scales or none) into the shared bf16 [M, N] buffer, which is returned."""
        import ctypes
        from . import _lib as L
        from . import ops
        from .blackwell_gemm_ws import _to_b2x_config
        if a_shard.shape[0] != self.M or w_shard.shape[0] != self.N:
            raise ValueError(f"shapes {tuple(a_shard.shape)} x {tuple(w_shard.shape)} do not match this "
                             f"[{self.M}, {self.N}] buffer")
        key = (a_shard.data_ptr(), tuple(a_shard.shape), a_shard.stride(), a_shard.dtype, w_shard.data_ptr(),
               tuple(w_shard.shape), w_shard.stride(), w_shard.dtype, None if sa is None else sa.data_ptr(),
               None if sw is None else sw.data_ptr(), tuple(sorted((cfg or {}).items())))
        g = self._plans.get(key)
        if g is None:
            mode = "none" if sa is None else "tensor"
            fields = tuple(_to_b2x_config(cfg or {}, a_shard.shape[1]))
            g = ops._gemm_args(a_shard, w_shard.t(), self.out, mode, sa, sw, fields)
            if len(self._plans) > 64:
                self._plans.clear()
            self._plans[key] = g
        self._ar.epoch = 0  # the kernel counts the calls in the signal buffer (graph-capturable)
        with torch.cuda.device(self.device):
            st = L.lib().b2x_fp8_gemm_allreduce(ctypes.byref(g), ctypes.byref(self._ar),
                                                ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        L.check(st)
        return self.out


    def reset(self) -> None:
        """Collective: zero the signal buffer (counters and call count) on every
        rank.  No fused call may be in flight on any rank."""
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        self.signal.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    def check(self) -> None:
        """Collective: raise B2XError (after reset()) if a fused call on any
        rank gave up waiting for its peers since the last check."""
        from . import _lib as L
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            st = L.read_device_status()
        flag = torch.tensor([st], dtype=torch.int64, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        if flag.item():
            self.reset()
            raise L.B2XError(L.ERR_TIMEOUT, f"fused all-reduce: a rank gave up waiting for its peers "
                                            f"(device status 0x{int(flag.item()):x}); signal buffers were reset")


def _default_swiglu(x, w_gu, sx, sw, h_scale, h_amax=None):
    from .ops import gemm_swiglu
    h, _ = gemm_swiglu(x, w_gu, sx, sw, mode="given", h_scale=h_scale, h_amax=h_amax)
    return h


class LlamaFP8LinearSet:
    """The Llama-3-70B-shaped fp8 linear set of one transformer block at a
    fixed token count, chained the way the block uses it and sharded over the
    process group:

      qkv = x . Wqkv^T                        (bf16 out; column-parallel, no collective)
      h   = fp8(silu(x . Wg^T) * (x . Wu^T))  (gate+up GEMM with the SwiGLU and the
                                               fp8 quantization of h in its epilogue;
                                               column-parallel, no collective)
      out = sum over ranks of h_r . Wd_r^T    (bf16 out; row-parallel: h's column shard
                                               is exactly down's K shard, + all-reduce)

    h is quantized with a static per-tensor scale (amax / 448 of one
    calibration pass at construction, the static activation scaling of fp8
    inference).  Wgu is the interleaved gate/up weight (interleave_gate_up):
    a contiguous row shard of it yields a contiguous column shard of h.

    comm = "fused" (default on GPUs): the down GEMM and the sum of its partials
    over the group are one kernel (FusedRowParallel).  comm = "nccl": the
    down GEMM followed by an NCCL all-reduce of its output.  The three GEMMs
    run one after another on all SMs.

    `mm` and `swiglu` are injectable so the partitioning can be checked on
    CPU ranks against an unsharded product.
    """

    SHAPES = {"qkv": (8192, 10240, 8192), "gate_up": (8192, 57344, 8192), "down": (8192, 8192, 28672)}

    def __init__(self, rank: int, world: int, device, tokens: int = 8192, seed: int = 1234,
                 mm: Callable = _default_mm, swiglu: Callable = _default_swiglu, make_input: Optional[Callable] = None,
                 comm: str = "fused", fused_mode: str = "auto"):
        self.rank, self.world, self.device, self.mm, self.swiglu = rank, world, device, mm, swiglu
        self.tokens = tokens
        M = tokens
        K = self.SHAPES["qkv"][2]
        nq = self.SHAPES["qkv"][1] // world
        ngu = self.SHAPES["gate_up"][1] // world
        kd = self.SHAPES["down"][2] // world
        nd = self.SHAPES["down"][1]
        if ngu != 2 * kd or kd % 128:
            raise ValueError("gate+up must produce down's K shard in 128-column blocks")
        make = make_input or _rand_fp8
        gx = torch.Generator(device=device).manual_seed(seed)  # the activations are the same on every rank
        self.x, self.sx = make((M, K), gx, device)
        g = torch.Generator(device=device).manual_seed(seed + 1 + rank)
        self.wq, self.sq = make((nq, K), g, device)
        self.wgu, self.sgu = make((ngu, K), g, device)
        self.wd, self.sd = make((nd, kd), g, device)
        self.flops_total = sum(2.0 * (M / 8192) * m * n * k for (m, n, k) in self.SHAPES.values())
        on_gpu = world > 1 and torch.device(device).type == "cuda"
        if comm not in ("fused", "nccl"):
            raise ValueError(f"comm must be 'fused' or 'nccl', got {comm!r}")
        self.comm = comm if on_gpu else "nccl"
        self.fused = FusedRowParallel(M, nd, device, mode=fused_mode) if self.comm == "fused" else None
        self.cfg = {}
        self.sh = self._calibrate_h_scale()

    def _calibrate_h_scale(self) -> torch.Tensor:
        one = torch.ones(1, dtype=torch.float32, device=self.device)
        amax = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.swiglu(self.x, self.wgu, self.sx, self.sgu, one, amax)
        sh = amax / 448.0
        return torch.where(sh > 0, sh, one)

    def capture(self):
        """Record step() once in a CUDA graph (collective: every rank calls it).
        replay() then runs the three kernels with no host work per launch;
        the fused all-reduce counts its calls on the device, so every replay
        is a new call.  Returns the (qkv_out, h, down_out) tensors that every
        replay overwrites."""
        dev = torch.device(self.device)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self.step()  # builds the argument plans and the allocator's blocks
        torch.cuda.synchronize(dev)
        if self.world > 1:
            dist.barrier()
        from ._lib import launch_count
        self.graph = torch.cuda.CUDAGraph()
        n0 = launch_count()
        with torch.cuda.graph(self.graph, stream=s):
            self.graph_outputs = self.step()
        self.graph_launches = launch_count() - n0  # libb2x kernels per replay
        torch.cuda.synchronize(dev)
        return self.graph_outputs

    def replay(self):
        """One step by replaying the graph of capture()."""
        self.graph.replay()
        return self.graph_outputs

    def step(self, events=None):
        """One pass over the set; returns (qkv_out, h, down_out)."""
        q = self.mm(self.x, self.wq, self.sx, self.sq, self.cfg)
        if events:
            events[0].record()
        h = self.swiglu(self.x, self.wgu, self.sx, self.sgu, self.sh)
        if events:
            events[1].record()
        if self.fused is not None:
            d = self.fused(h, self.sh, self.wd, self.sd)
        else:
            d = row_parallel(h, self.sh, self.wd, self.sd, mm=self.mm, cfg=self.cfg)
        return q, h, d


def _rand_fp8(shape, gen, device):
    from .ops import quantize
    x = torch.randn(shape, device=device, generator=gen)
    return quantize(x, "tensor", torch.float8_e4m3fn)
