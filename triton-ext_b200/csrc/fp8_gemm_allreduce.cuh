// Epilogue step of the fused GEMM + all-reduce (b2x_fp8_gemm_allreduce).
//
// Each rank of a node computes a partial C_r = A_r . B_r (the row-parallel
// layer: A and B sharded along K) into its own copy of a buffer that every
// rank can reach (a peer mapping of each copy, and for mode 1 one NVSwitch
// multicast address for all copies).  The sum C = sum_r C_r is formed tile by
// tile while the GEMM is still running:
//
//   1. the epilogue warpgroup that stored a 128 x 256 unit of C_r waits for
//      its TMA stores to complete, publishes them at system scope and adds 1
//      to the unit's arrival counter (held on rank unit % world);
//   2. the rank whose add completes the count (the last to finish that unit)
//      reduces it: mode 1 reads the unit once through the multicast address
//      (multimem.ld_reduce: the switch fetches every rank's copy and adds
//      them in fp32) and writes the bf16 sum back through the same address
//      (multimem.st: the switch stores it on every rank); mode 2 reads every
//      rank's copy over NVLink, adds in fp32 in rank order and stores the sum
//      to every rank;
//   3. it then adds 1 to the done word of every rank.
// Nothing waits for another GPU inside the tile loop: the last rank to arrive
// finds the data already there.  Each rank's kernel ends with one bounded
// wait until its done word shows every unit of this call reduced, so the
// output is complete on every rank when the kernel retires.
//
// The arrival counters reset themselves (the reducer stores 0), and the done
// word grows by `units` per call, so consecutive calls need no clearing as
// long as every rank makes the same calls in the same order.
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

// One epilogue warpgroup (128 threads, named barrier `bar_id`) after issuing
// the TMA stores of output rows [m0, m0 + 128) x columns [n0, n0 + 256).
// `flag` is one shared word private to this warpgroup.
template <int AR>
__device__ __forceinline__ void ar_unit_stored(const GemmParams& p, int unit, int m0, int n0, int wg_tid,
                                               uint32_t bar_id, volatile uint32_t* flag) {
  const ArParams& ar = p.ar;
  if (wg_tid == 0) {
    bulk_wait_group0();          // the unit's stores are complete in global memory
    fence_proxy_async_global();  // ... and ordered before generic-proxy accesses
    fence_acq_rel_sys();
    uint32_t* ctr = ar.sig_peer[unit % ar.world] + kArArrive0 + unit;
    const uint32_t before = atom_add_acq_rel_sys(ctr, 1u);
    const bool last = before == (uint32_t)(ar.world - 1);
    if (last) st_relaxed_sys(ctr, 0u);  // every rank has arrived: reset for the next call
    *flag = last ? 1u : 0u;
  }
  named_bar_sync(bar_id, 128);
  if (*flag == 0u) return;

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
  named_bar_sync(bar_id, 128);
  if (wg_tid == 0) {
    if constexpr (AR == 1) {
      multimem_red_add_release_sys(ar.sig_mc, 1u);
    } else {
      for (int r = 0; r < ar.world; ++r) red_add_release_sys(ar.sig_peer[r], 1u);
    }
  }
}

}  // namespace b2x
