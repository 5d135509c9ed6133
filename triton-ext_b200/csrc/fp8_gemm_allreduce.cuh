// Epilogue steps of the fused GEMM + all-reduce (b2x_fp8_gemm_allreduce).
//
// Each rank of a node computes a partial C_r = A_r . B_r (the row-parallel
// layer: A and B sharded along K) into its own copy of a buffer that every
// rank can reach (a peer mapping of each copy, and for mode 1 one NVSwitch
// multicast address for all copies).  The sum C = sum_r C_r is formed unit by
// unit (128 x 256 outputs, one CTA's half of a paired tile) while the GEMM is
// still running:
//
//   1. the epilogue warpgroup that stored a unit of C_r waits for its TMA
//      stores to complete, publishes them at system scope and adds 1 to the
//      unit's arrival counter, kept on the unit's owner rank (a hash of the
//      unit index spreads the units evenly over the ranks);
//   2. the owner's warpgroup that stored the same unit queues it; between
//      tiles it checks (without blocking) whether the oldest queued unit has
//      all arrivals and if so reduces it: mode 1 reads the unit once through
//      the multicast address (multimem.ld_reduce: the switch fetches every
//      rank's copy and adds them in fp32) and writes the bf16 sum back
//      through the same address (multimem.st: the switch stores it on every
//      rank); mode 2 reads every rank's copy over NVLink, adds in fp32 in
//      rank order and stores the sum to every rank;
//   3. it resets the arrival counter and adds 1 to the done word of every rank.
// A queue that fills up, and the queue left at the end of the tile loop, are
// served with bounded waits.  These waits cannot form a cycle: every rank
// launches the same grid, so a unit is stored by the same warpgroup index on
// every rank, in the same sequence; a warpgroup waits only for a unit it has
// already stored, i.e. for a peer's same warpgroup that is behind it in that
// sequence, and following such waits always leads to a warpgroup that is not
// waiting.  Each rank's kernel ends with one bounded wait
// until its done word shows every unit of this call reduced, so the output
// is complete on every rank when the kernel retires.
//
// The done word grows by `units` per call, so consecutive calls need no
// clearing as long as every rank makes the same calls in the same order.
// Fixed owners (rather than "the last rank to arrive reduces") keep the
// reduction work even: a rank that reduces falls behind and would otherwise
// arrive last again and again.
#pragma once
#include <cstdint>
#include "b2x_ptx.cuh"
#include "fp8_gemm_common.cuh"

namespace b2x {

constexpr uint64_t kArWaitNs = 10000000000ull;  // 10 s: covers launch skew between ranks

__device__ __forceinline__ void bf16x8_add(float (&acc)[8], uint4 x) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ int ar_owner(int unit, int world) {
  return (int)(((uint32_t)unit * 0x9E3779B1u) >> 20) % world;
}

// Thread 0 of the warpgroup that issued the TMA stores of `unit`: make them
// visible system-wide and count them on the owner rank.
__device__ __forceinline__ void ar_arrive(const ArParams& ar, int unit) {
  bulk_wait_group0();          // the unit's stores are complete in global memory
  fence_proxy_async_global();  // ... and ordered before generic-proxy accesses
  fence_acq_rel_sys();
  red_add_release_sys(ar.sig_peer[ar_owner(unit, ar.world)] + kArArrive0 + unit, 1u);
}

// All 128 threads of one warpgroup: C[unit] = sum over ranks, on every rank.
template <int AR>
__device__ __forceinline__ void ar_reduce_unit(const GemmParams& p, int unit, int wg_tid) {
  const ArParams& ar = p.ar;
  int pid_m, pid_n;
  compute_pid(unit >> 1, p.group_size_m * p.num_pid_n, p.num_pid_m, p.group_size_m, pid_m, pid_n);
  const int m0 = pid_m * 2 * kBM + (unit & 1) * kBM;
  const int n0 = pid_n * 256;
  const int64_t rb = p.ldc * 2;  // bytes per C row
  const int64_t base = (int64_t)m0 * rb + (int64_t)n0 * 2;
  // 128 rows x 512 bytes = 4096 16-byte vectors; 32 consecutive threads cover one row.
  if constexpr (AR == 1) {
#pragma unroll 1
    for (int it = 0; it < 32; it += 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int idx = (it + j) * 128 + wg_tid;
        v[j] = multimem_ld_reduce_bf16x8(ar.c_mc + base + (idx >> 5) * rb + (idx & 31) * 16);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int idx = (it + j) * 128 + wg_tid;
        multimem_st_16(ar.c_mc + base + (idx >> 5) * rb + (idx & 31) * 16, v[j]);
      }
    }
  } else {
#pragma unroll 1
    for (int it = 0; it < 32; it += 4) {
      float acc[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[j][i] = 0.f;
#pragma unroll 1
      for (int r = 0; r < ar.world; ++r) {
        const uint8_t* src = ar.c_peer[r] + base;
        uint4 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int idx = (it + j) * 128 + wg_tid;
          x[j] = __ldcv(reinterpret_cast<const uint4*>(src + (idx >> 5) * rb + (idx & 31) * 16));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) bf16x8_add(acc[j], x[j]);
      }
      uint4 out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        out[j] = make_uint4(pack_bf16x2(acc[j][0], acc[j][1]), pack_bf16x2(acc[j][2], acc[j][3]),
                            pack_bf16x2(acc[j][4], acc[j][5]), pack_bf16x2(acc[j][6], acc[j][7]));
#pragma unroll 1
      for (int r = 0; r < ar.world; ++r) {
        uint8_t* dst = ar.c_peer[r] + base;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int idx = (it + j) * 128 + wg_tid;
          __stcg(reinterpret_cast<uint4*>(dst + (idx >> 5) * rb + (idx & 31) * 16), out[j]);
        }
      }
    }
  }
  fence_acq_rel_sys();  // this thread's share of the sum is visible on every rank
}

// Per-warpgroup queue of owned units waiting for their arrivals (shared
// memory, touched by thread 0 only) and the word that broadcasts thread 0's
// decision to the warpgroup.
constexpr int kArQueue = 16;
struct ArQueue {
  int unit[kArQueue];
  int head, count;
  int cmd;  // >= 0: reduce this unit; -1: nothing to do; -2: gave up (timeout)
  int pad;
};

// One warpgroup after storing `unit` (unit < 0: end of the tile loop, drain
// the queue).  Reduces at most `max_reduce` ready units, waiting (bounded)
// only when the queue is full or when draining.
template <int AR>
__device__ __forceinline__ void ar_service(const GemmParams& p, int unit, int wg_tid, uint32_t bar_id,
                                           volatile ArQueue* q) {
  const ArParams& ar = p.ar;
  const bool drain = unit < 0;
  if (wg_tid == 0 && !drain) {
    ar_arrive(ar, unit);
    if (ar_owner(unit, ar.world) == ar.rank) {
      q->unit[(q->head + q->count) % kArQueue] = unit;
      q->count = q->count + 1;
    }
  }
  for (int served = 0;; ++served) {
    if (wg_tid == 0) {
      int cmd = -1;
      if (q->count > 0 && (drain || served < 2)) {
        const int u = q->unit[q->head];
        const uint32_t* ctr = ar.sig_peer[ar.rank] + kArArrive0 + u;
        bool ready = ld_acquire_sys(ctr) >= (uint32_t)ar.world;
        if (!ready && (drain || q->count == kArQueue)) {
          const long long t0 = clock64();
          ready = wait_counter_sys(ctr, (uint32_t)ar.world, kArWaitNs);
          trace_add(p.trace, 9, (unsigned long long)(clock64() - t0));
        }
        if (ready) {
          st_relaxed_sys(const_cast<uint32_t*>(ctr), 0u);  // all arrived: reset for the next call
          q->head = (q->head + 1) % kArQueue;
          q->count = q->count - 1;
          cmd = u;
        } else if (drain || q->count == kArQueue) {
          cmd = -2;  // a peer never arrived; the status word says so
          q->count = 0;
        }
      }
      q->cmd = cmd;
    }
    named_bar_sync(bar_id, 128);
    const int cmd = q->cmd;
    named_bar_sync(bar_id, 128);  // everyone has read cmd before thread 0 rewrites it
    if (cmd < 0) break;
    const long long t0 = clock64();
    ar_reduce_unit<AR>(p, cmd, wg_tid);
    named_bar_sync(bar_id, 128);
    if (wg_tid == 0) {
      trace_add(p.trace, 8, (unsigned long long)(clock64() - t0));
      trace_add(p.trace, drain ? 11 : 10, 1);
      if constexpr (AR == 1) {
        multimem_red_add_release_sys(ar.sig_mc, 1u);
      } else {
        for (int r = 0; r < ar.world; ++r) red_add_release_sys(ar.sig_peer[r], 1u);
      }
      atomicAdd(ar.sig_peer[ar.rank] + 1, 1u);  // units this rank reduced (diagnostic)
    }
  }
}

}  // namespace b2x
