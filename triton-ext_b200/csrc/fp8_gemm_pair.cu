// Paired-CTA (cta_group::2) persistent fp8 GEMM for sm_100a.
//
// The counterpart of the reference GEMM's 2-CTA mode (NUM_CTAS=2,
// ctas_per_cga=(2,1,1): extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py
// :1141-1150, 973-975, 1118-1120), where CTA pairs share the B tile.
//
// Two CTAs on the two SMs of a TPC form a cluster and own a 256 x 256 output
// tile: CTA r (r = 0, 1) holds rows [128 r, 128 r + 128) of the tile in its own
// TMEM and loads, per 128-deep K block, its own 128 rows of A and its own 128
// columns of B -- 32 KB per CTA per K block instead of the 48 KB a single CTA
// needs for a 128 x 256 tile.  No load uses multicast: each CTA fetches its own
// halves; the tensor cores exchange the B halves.
//
// Roles (384 threads per CTA, as in the single-CTA kernel):
//   warp 0  TMA producer (both CTAs).  Completion of both CTAs' loads is
//           counted on the even CTA's `full` barrier (cta_group::2 TMA).
//   warp 1  MMA issuer (even CTA only): tcgen05.mma.cta_group::2 M=256 N=256
//           K=32; tcgen05.commit multicasts to both CTAs' `empty` (stage free)
//           and `tfull` (accumulator ready) barriers.
//   warp 2  TMEM allocator (cta_group::2, both CTAs).
//   warps 4-11  two epilogue warpgroups per CTA, ping-ponging over two TMEM
//           accumulators.  Each CTA's warpgroup releases its buffer with one
//           arrive on the even CTA's `tempty` barrier (count 2: one per CTA).
// Every wait is bounded as in the single-CTA kernel; both CTAs meet at a final
// cluster barrier so no CTA leaves while its peer may still touch its smem.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"
#include "fp8_gemm_allreduce.cuh"
#include "fp8_gemm_swiglu.cuh"

namespace b2x {

constexpr int kPairBN = 256;        // output columns per pair tile
constexpr int kPairHalfN = 128;     // B columns loaded by each CTA
constexpr uint32_t kPairTmemCols = 512;

template <int STAGES>
struct PairSmem {
  static constexpr int kABytes = kBM * kBK;           // 16 KB
  static constexpr int kBBytes = kPairHalfN * kBK;    // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kCBytes = kBM * 128;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kCOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kCOff + 2 * kCBytes;
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kQOff = (kBarOff + kBarBytes + 15) / 16 * 16;  // fused all-reduce queues
  static constexpr int kAlloc = kQOff + (int)sizeof(ArRing) + 1024;
};

// AR: 0 plain GEMM; 1 / 2 the GEMM output is summed over the node's GPUs as
// its units are stored (fp8_gemm_allreduce.cuh; 1 NVSwitch multicast, 2 peer
// loads and stores).  EPI: 1 = the fused SwiGLU + fp8 quantize epilogue
// (fp8_gemm_swiglu.cuh; tmC then maps the fp8 output h).
template <int AR>
constexpr int pair_threads() {
  return AR != 0 ? kThreads + 128 : kThreads;  // + the reducer warpgroup of the fused all-reduce
}

template <int STAGES, int B_MN, int AR, int EPI = 0>
__global__ void __launch_bounds__(pair_threads<AR>(), 1)
    fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using L = PairSmem<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  // The dynamic smem base has the same offset in both CTAs, so the aligned
  // buffers below sit at identical offsets -- which the paired MMA requires.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile ArRing* ar_ring = reinterpret_cast<volatile ArRing*>(smem + L::kQOff);  // owned units for the reducer

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the even CTA's expect_tx arrive (covers both CTAs' bytes)
      mbar_init(&empty[s], 1);  // one multicast commit per use
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2);  // one arrive per CTA's epilogue warpgroup (used in the even CTA)
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    for (int i = 0; i < kArRing; ++i) ar_ring->slot[i] = 0;
    ar_ring->tail = 0;
    ar_ring->cmd = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kPairTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and TMEM allocation visible to the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const long long t_start = clock64();
  const int num_pid_in_group = p.group_size_m * p.num_pid_n;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = l2_policy(p.l2_a);
      const uint64_t pol_b = l2_policy(p.l2_b);
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0;
      uint32_t pend_phase[STAGES];
      bool ok = true;
      for (int tile = cluster_id; tile < p.num_units && ok; tile += num_clusters) {
        int pid_m, pid_n;
        compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
        const int row0 = pid_m * 2 * kBM + (int)rank * kBM;
        const int col0 = pid_n * kPairBN + (int)rank * kPairHalfN;
        for (int kb = 0; kb < p.k_tiles; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          uint8_t* sA = smem + L::kAOff + stage * L::kABytes;
          uint8_t* sB = smem + L::kBOff + stage * L::kBBytes;
          tma_load_2d_pair(sA, &tmA, full_leader, kb * kBK, row0, pol_a);
          if (B_MN)
            tma_load_2d_pair(sB, &tmB, full_leader, col0, kb * kBK, pol_b);
          else
            tma_load_2d_pair(sB, &tmB, full_leader, kb * kBK, col0, pol_b);
          issued_mask |= 1u << stage;
          pend_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // The even CTA's full barriers count both CTAs' loads: waiting on them
      // there guarantees no TMA write into either CTA's smem is in flight.
      if (leader)
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) {
            volatile int no_abort = 0;
            mbar_wait(&full[s], pend_phase[s], &no_abort, kStatusTimeoutProducer);
          }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      const bool withhold_first = g_inject == 1;  // test hook (b2x_debug_inject)
      for (int tile = cluster_id; tile < p.num_units && ok; tile += num_clusters, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kPairBN;
        for (int kb = 0; kb < p.k_tiles; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kBOff + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            const uint64_t adesc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_addr + k * 32 * 128, 128 * kBK, 1024)
                                        : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            mma_f8f6f4_pair(d_tmem, adesc, bdesc, p.idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (!(withhold_first && local == 0)) mma_commit_pair_mc(&tfull[buf], 0x3);
      }
      mma_commit_pair_mc(mma_done, 0x1);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, kStatusTimeoutMma);
    }
  } else if (AR != 0 && warp >= kEpiWarp0 + 8) {
    // ------------------------------------------------------------ all-reduce reducer (both CTAs)
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 8) * 32;
    const uint32_t bar_id = 3;
    // With the call count kept on the device, this call is number count + 1.
    // The count is read before any unit of this CTA is stored; the CTA that
    // advances it does so only after every unit of the call (this CTA's
    // included) has been reduced, so no CTA can read an advanced count.
    uint32_t call_no = 0, done_target = p.ar.done_target;
    if (p.ar.device_epoch && wg_tid == 0) {
      call_no = ld_relaxed_sys(p.ar.sig_peer[p.ar.rank] + kArEpochWord) + 1u;
      done_target = call_no * p.ar.units;  // modulo 2^32, like the done word
    }
    const int n_owned = ar_owned_units(p, cluster_id, num_clusters, (int)rank);
    const long long t_red = clock64();
    const bool ok = ar_reducer<AR>(p, n_owned, wg_tid, bar_id, ar_ring, abort_flag);
    if (wg_tid == 0) trace_add(p.trace, 13, (unsigned long long)(clock64() - t_red));
    // The output is complete here once every unit of this call has been
    // reduced by its owner rank.
    if (ok && wg_tid == 0 && !*abort_flag) {
      const long long t0 = clock64();
      const bool done = wait_counter_sys(p.ar.sig_peer[p.ar.rank], done_target, kArWaitNs);
      trace_add(p.trace, 12, (unsigned long long)(clock64() - t0));
      if (done && p.ar.device_epoch && blockIdx.x == 0)
        st_relaxed_sys(p.ar.sig_peer[p.ar.rank] + kArEpochWord, call_no);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 8) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int e = (warp - kEpiWarp0) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 4 * e) * 32;
    uint8_t* stage_c = smem + L::kCOff + e * L::kCBytes;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[e]), 0);
    float alpha = 1.0f;
    if (p.scale_mode != B2X_SCALE_NONE) alpha = __fmul_rn(__ldg(p.scale_a), __ldg(p.scale_b));
    int local = 0;
    for (int tile = cluster_id; tile < p.num_units; tile += num_clusters, ++local) {
      if ((local & 1) != e) continue;
      int pid_m, pid_n;
      compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
      const uint32_t use = (uint32_t)(local >> 1);
      bool ok = mbar_wait(&tfull[e], use & 1, abort_flag, kStatusTimeoutEpilogue);
      if (!wg_all(ok, bar_id)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + e * kPairBN + ((uint32_t)(q * 32) << 16);
      const int m0 = pid_m * 2 * kBM + (int)rank * kBM;
      const int n0 = pid_n * kPairBN;
      if constexpr (EPI == 1) {
        swiglu_quant_tile(p, &tmC, t_row, m0, pid_n, alpha, stage_c, bar_id, wg_tid, row, [&]() {
          tc_fence_before();
          named_bar_sync(bar_id, 128);
          if (wg_tid == 0) mbar_arrive_cluster_relaxed(tempty_leader);
        });
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < kPairBN; c0 += 64) {
          uint32_t v[64];
          tmem_ld_32x32b_x32(t_row + c0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          tmem_ld_32x32b_x32(t_row + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          tmem_ld_wait();
          if (c0 + 64 == kPairBN) {
            // Whole accumulator read: hand the buffer back to the MMA warp before
            // the last conversion and store.
            tc_fence_before();
            named_bar_sync(bar_id, 128);
            if (wg_tid == 0) mbar_arrive_cluster_relaxed(tempty_leader);
          }
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float lo = __fmul_rn(__uint_as_float(v[2 * i]), alpha);
            float hi = __fmul_rn(__uint_as_float(v[2 * i + 1]), alpha);
            if (p.c_half) {
              __half2 h = __floats2half2_rn(lo, hi);
              pk[i] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              pk[i] = pack_bf16x2(lo, hi);
            }
          }
          if (wg_tid == 0) bulk_wait_group_read0();
          named_bar_sync(bar_id, 128);
          const uint32_t srow = smem_u32(stage_c + row * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_v4(srow + ((j ^ (row & 7)) << 4), pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
          fence_proxy_async_smem();
          named_bar_sync(bar_id, 128);
          if (wg_tid == 0 && m0 < p.M) {  // the odd CTA's rows may lie wholly past M
            tma_store_2d(&tmC, stage_c, n0 + c0, m0);
            bulk_commit_group();
          }
        }
      }
      if constexpr (AR != 0) {
        // publish the unit's stores and count them on its owner; owned units
        // go to this CTA's reducer warpgroup
        if (wg_tid == 0) {
          const int unit = 2 * tile + (int)rank;
          ar_arrive(p.ar, unit);
          if (ar_owner(unit, p.ar.world) == p.ar.rank) ar_ring_push(ar_ring, unit, abort_flag);
        }
      }
    }
    if (wg_tid == 0) bulk_wait_group0();
  }

  if (threadIdx.x == 0) trace_add(p.trace, 5, (unsigned long long)(clock64() - t_start));
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still use its smem or barriers
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

template <int STAGES, int B_MN, int AR, int EPI = 0>
static cudaError_t launch_pair_t(const GemmLaunch& g, const GemmParams& p, cudaStream_t st) {
  using L = PairSmem<STAGES>;
  auto kern = fp8_gemm_pair_kernel<STAGES, B_MN, AR, EPI>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::kAlloc);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(pair_threads<AR>(), 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Persistent grid: as many CTA pairs as can be resident at once.
  static int max_clusters = 0;
  if (max_clusters == 0) {
    cfg.gridDim = dim3(2 * 74, 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = 74;
    (void)cudaGetLastError();
    max_clusters = n;
  }
  int clusters = p.num_units < max_clusters ? p.num_units : max_clusters;
  if (clusters > g.num_sms / 2) clusters = g.num_sms / 2;  // NUM_SMS cap
  if (clusters < 1) clusters = 1;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, g.tmA, g.tmB, g.tmC, p);
  note_launch(1);
  return e;
}

cudaError_t launch_fp8_gemm_pair(const GemmLaunch& g, cudaStream_t st) {
  constexpr int kStages = (kMaxDynSmem - 2 * kBM * 128 - 1024 - 256) / (kBM * kBK + kPairHalfN * kBK);
  constexpr int S = kStages > 8 ? 8 : kStages;
  GemmParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  p.num_pid_m = (int)((g.M + 2 * kBM - 1) / (2 * kBM));
  p.num_pid_n = (int)((g.N + kPairBN - 1) / kPairBN);
  p.num_mn_tiles = p.num_pid_m * p.num_pid_n;
  p.num_units = p.num_mn_tiles;
  p.split_k = 1;
  p.group_size_m = g.group_size_m;
  p.k_tiles = (int)((g.K + kBK - 1) / kBK);
  p.k_tiles_per_split = p.k_tiles;
  p.idesc = idesc_f8f6f4(g.a_fmt, g.b_fmt, 0, g.b_mn ? 1 : 0, 2 * kBM, kPairBN);
  p.c_half = g.c_half;
  p.scale_mode = g.scale_mode;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.c = g.c;
  p.ldc = g.ldc;
  p.l2_a = g.l2_a;
  p.l2_b = g.l2_b;
  p.ar = g.ar;
  p.trace = g.trace;
  p.sw_mode = g.sw_mode;
  p.sw_fmt = g.sw_fmt;
  p.sw_scale = g.sw_scale;
  p.sw_ld_scale = g.sw_ld_scale;
  p.sw_given = g.sw_given;
  p.sw_amax = g.sw_amax;
  if (g.swiglu) return launch_pair_t<S, 0, 0, 1>(g, p, st);  // K-major B only
  if (g.ar.mode == 1) return launch_pair_t<S, 0, 1>(g, p, st);  // fused all-reduce: K-major B only
  if (g.ar.mode == 2) return launch_pair_t<S, 0, 2>(g, p, st);
  return g.b_mn ? launch_pair_t<S, 1, 0>(g, p, st) : launch_pair_t<S, 0, 0>(g, p, st);
}

}  // namespace b2x
