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
//   2. if this rank owns the unit, the warpgroup also pushes it into a ring in
//      shared memory, read by a fifth warpgroup of the CTA that does nothing
//      but reduce: for each owned unit, in the order the epilogues stored
//      them, it waits (bounded) until the unit has all arrivals and reduces
//      it -- mode 1 reads the unit once through the multicast address
//      (multimem.ld_reduce: the switch fetches every rank's copy and adds
//      them in fp32) and writes the bf16 sum back through the same address
//      (multimem.st: the switch stores it on every rank); mode 2 reads every
//      rank's copy over NVLink, adds in fp32 in rank order and stores the sum
//      to every rank;
//   3. it resets the arrival counter and adds 1 to the done word of every rank.
// So the GEMM's epilogues never wait for a peer: the reductions run beside
// the tile loop and keep NVLink busy while the tensor cores work.  The waits
// cannot form a cycle: every rank launches the same grid, so a unit is
// stored by the same CTA and warpgroup on every rank, in the same sequence,
// and a reducer waits only for units its own CTA has already stored, i.e.
// for peers' same CTA that are behind in that sequence.  A full ring makes
// an epilogue wait for its reducer, which again waits only on such units.
// After its last unit the reducer waits (bounded) until its done word shows
// every unit of this call reduced, so the output is complete on every rank
// when the kernel retires.
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
    for (int it = 0; it < 32; it += 16) {
      uint4 v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int idx = (it + j) * 128 + wg_tid;
        v[j] = multimem_ld_reduce_bf16x8(ar.c_mc + base + (idx >> 5) * rb + (idx & 31) * 16);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
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
  // No per-thread fence: the caller orders every thread's stores before the
  // done signal with a warpgroup barrier and one system-scope fence.
}

// Ring of owned units in shared memory, from the two epilogue warpgroups
// (producers, thread 0 of each) to the reducer warpgroup (thread 0).  A slot
// holds unit + 1, 0 when free; producers take tickets with an atomic add and
// wait (bounded) for their slot to be free.
constexpr int kArRing = 32;
struct ArRing {
  int slot[kArRing];
  int tail;  // tickets taken by the producers
  int cmd;   // reducer thread 0 -> its warpgroup: unit to reduce, -1 stop
};

__device__ __forceinline__ bool ar_ring_push(volatile ArRing* r, int unit, volatile int* abort) {
  const int t = atomicAdd(const_cast<int*>(&r->tail), 1);
  volatile int* s = &r->slot[t % kArRing];
  const uint64_t start = globaltimer();
  while (*s != 0) {
    if (*abort) return false;
    if (globaltimer() - start > kArWaitNs) {
      atomicCAS(&g_status, 0, kStatusTimeoutAllReduce);
      *abort = 1;
      return false;
    }
    __nanosleep(64);
  }
  *s = unit + 1;
  return true;
}

__device__ __forceinline__ int ar_ring_pop(volatile ArRing* r, int ticket, volatile int* abort) {
  volatile int* s = &r->slot[ticket % kArRing];
  const uint64_t start = globaltimer();
  int v;
  while ((v = *s) == 0) {
    if (*abort) return -1;
    if (globaltimer() - start > kArWaitNs) {
      atomicCAS(&g_status, 0, kStatusTimeoutAllReduce);
      *abort = 1;
      return -1;
    }
    __nanosleep(32);
  }
  *s = 0;
  return v - 1;
}

// Number of units the CTA at cluster rank `crank` of cluster `cluster_id`
// stores during the tile loop that this GPU rank owns.
__device__ __forceinline__ int ar_owned_units(const GemmParams& p, int cluster_id, int num_clusters, int crank) {
  int n = 0;
  for (int tile = cluster_id; tile < p.num_units; tile += num_clusters)
    n += ar_owner(2 * tile + crank, p.ar.world) == p.ar.rank;
  return n;
}

// The reducer warpgroup (128 threads, named barrier `bar_id`).  Returns
// false if it gave up (a peer never arrived, or the GEMM aborted).
template <int AR>
__device__ __forceinline__ bool ar_reducer(const GemmParams& p, int n_owned, int wg_tid, uint32_t bar_id,
                                           volatile ArRing* ring, volatile int* abort) {
  const ArParams& ar = p.ar;
  bool ok = true;
  for (int i = 0; i < n_owned; ++i) {
    if (wg_tid == 0) {
      int cmd = ar_ring_pop(ring, i, abort);
      if (cmd >= 0) {
        const uint32_t* ctr = ar.sig_peer[ar.rank] + kArArrive0 + cmd;
        const long long t0 = clock64();
        if (ld_acquire_sys(ctr) < (uint32_t)ar.world && !wait_counter_sys(ctr, (uint32_t)ar.world, kArWaitNs)) {
          *abort = 1;
          cmd = -1;
        } else {
          st_relaxed_sys(const_cast<uint32_t*>(ctr), 0u);  // all arrived: reset for the next call
        }
        trace_add(p.trace, 9, (unsigned long long)(clock64() - t0));
      }
      ring->cmd = cmd;
    }
    named_bar_sync(bar_id, 128);
    const int cmd = ring->cmd;
    named_bar_sync(bar_id, 128);  // everyone has read cmd before thread 0 rewrites it
    if (cmd < 0) {
      ok = false;
      break;
    }
    const long long t0 = clock64();
    ar_reduce_unit<AR>(p, cmd, wg_tid);
    named_bar_sync(bar_id, 128);
    if (wg_tid == 0) {
      // The barrier above orders the warpgroup's stores of the sum before this
      // thread's fence; the fence (cumulative) makes them visible on every
      // rank before the done signal.
      fence_acq_rel_sys();
      trace_add(p.trace, 8, (unsigned long long)(clock64() - t0));
      trace_add(p.trace, 10, 1);
      if constexpr (AR == 1) {
        multimem_red_add_release_sys(ar.sig_mc, 1u);
      } else {
        for (int r = 0; r < ar.world; ++r) red_add_release_sys(ar.sig_peer[r], 1u);
      }
      atomicAdd(ar.sig_peer[ar.rank] + 1, 1u);  // units this rank reduced (diagnostic)
    }
  }
  return ok;
}

}  // namespace b2x
