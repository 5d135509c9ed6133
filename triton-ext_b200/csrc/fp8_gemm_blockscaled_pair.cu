// Block-scaled fp8 GEMM on CTA pairs (cta_group::2), 256 x 128 tiles.
//
//   C[m, n] = sum_kb sA[m, kb] * sB[kb, nb(n)] * (A[m, kb-block] . B[kb-block, n])
//
// Same per-K-block promotion as fp8_gemm_blockscaled.cu, on the operand
// traffic of a CTA pair: each CTA loads its 128 rows of A and its 64 columns
// of B per 128-deep K block, the even CTA issues tcgen05.mma.cta_group::2
// M=256 N=128 into one of four 128-column TMEM partial buffers, and each CTA
// promotes its 128 x 128 half of every partial into fp32 register
// accumulators.  Per SM and K block that moves 24 KB through TMA instead of
// the single-CTA kernel's 32 KB, with the same promotion work per SM.  (A
// 256 x 256 pair tile needs 128 fp32 accumulators per epilogue thread, or
// four warpgroups at under 100 registers whose TMEM loads cannot be hidden.)
//
// Threads (384 per CTA): warp 0 TMA producer, warp 1 MMA issuer (even CTA),
// warp 2 TMEM allocator, warps 4-11 two epilogue warpgroups of 64 columns
// each (64 fp32 accumulators per thread).  A K block's partial buffer is
// released with one arrive per epilogue warp of both CTAs (16 arrivals on the
// even CTA's barrier).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"

namespace b2x {

// Tile shapes: BN = 128 (two epilogue warpgroups, 384 threads) or BN = 256
// (four epilogue warpgroups of 64 columns, 576 threads, the TMEM allocator
// doubling as an epilogue warp).
template <int BN>
struct BpShape {
  static constexpr int kThreads = BN == 256 ? 576 : 384;
  static constexpr int kEpiWarp0 = BN == 256 ? 2 : 4;
  static constexpr int kEpiGroups = BN / 64;
  static constexpr int kHalfN = BN / 2;        // B columns loaded by each CTA
  static constexpr int kSlots = 512 / BN;      // TMEM partial buffers of BN columns
  static constexpr int kLoadCols = BN == 256 ? 16 : 32;  // tcgen05.ld width (register budget)
};

struct BpParams {
  int M, N, K;
  int num_pid_m, num_pid_n, num_tiles, group_size_m, k_tiles;
  uint32_t idesc;
  int c_half;
  const float* scale_a;
  const float* scale_b;
  int64_t sa_m, sa_k, sb_k, sb_n;
  int trace;
};

template <int STAGES, int BN>
struct BpSmem {
  static constexpr int kBpEpiGroups = BpShape<BN>::kEpiGroups;
  static constexpr int kBpSlots = BpShape<BN>::kSlots;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BpShape<BN>::kHalfN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kCBytes = kBM * 128;  // one 128-row x 64-column bf16 staging tile per warpgroup
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kCOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kCOff + kBpEpiGroups * kCBytes;
  static constexpr int kBarBytes = (2 * STAGES + 2 * kBpSlots + 1) * 8 + 16;
  static constexpr int kAlloc = kBarOff + kBarBytes + 1024;
};

template <int STAGES, int BN>
__global__ void __launch_bounds__(BpShape<BN>::kThreads, 1)
    fp8_gemm_blockscaled_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                     const __grid_constant__ CUtensorMap tmC, const BpParams p) {
  using L = BpSmem<STAGES, BN>;
  constexpr int kBpBN = BN;
  constexpr int kBpHalfN = BpShape<BN>::kHalfN;
  constexpr int kBpSlots = BpShape<BN>::kSlots;
  constexpr int kBpEpiGroups = BpShape<BN>::kEpiGroups;
  constexpr int kBpEpiWarp0 = BpShape<BN>::kEpiWarp0;
  constexpr int kLC = BpShape<BN>::kLoadCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;
  uint64_t* pempty = pfull + kBpSlots;
  uint64_t* mma_done = pempty + kBpSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const long long t_start = clock64();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kBpSlots; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 2 * 4 * kBpEpiGroups);  // every epilogue warp of both CTAs
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kBpSlots * kBpBN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_pid_in_group = p.group_size_m * p.num_pid_n;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0;
      uint32_t pend_phase[STAGES];
      bool ok = true;
      for (int tile = cluster_id; tile < p.num_tiles && ok; tile += num_clusters) {
        int pid_m, pid_n;
        compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
        const int row0 = pid_m * 2 * kBM + (int)rank * kBM;
        const int col0 = pid_n * kBpBN + (int)rank * kBpHalfN;
        for (int kb = 0; kb < p.k_tiles; ++kb) {
          if (!mbar_wait_traced(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer, p.trace, 0)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          tma_load_2d_pair(smem + L::kAOff + stage * L::kABytes, &tmA, full_leader, kb * kBK, row0, pol);
          tma_load_2d_pair(smem + L::kBOff + stage * L::kBBytes, &tmB, full_leader, kb * kBK, col0, pol);
          issued_mask |= 1u << stage;
          pend_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (leader)
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) {
            volatile int no_abort = 0;
            mbar_wait(&full[s], pend_phase[s], &no_abort, kStatusTimeoutProducer);
          }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < p.num_tiles && ok; tile += num_clusters) {
        for (int kb = 0; kb < p.k_tiles; ++kb, ++g) {
          const uint32_t slot = g % kBpSlots, use = g / kBpSlots;
          if (!mbar_wait_traced(&pempty[slot], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma, p.trace, 2) ||
              !mbar_wait_traced(&full[stage], phase, abort_flag, kStatusTimeoutMma, p.trace, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kBOff + stage * L::kBBytes);
          const uint32_t d_tmem = tmem_base + slot * kBpBN;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_f8f6f4_pair(d_tmem, smem_desc_sw128(a_addr + k * 32, 16, 1024),
                            smem_desc_sw128(b_addr + k * 32, 16, 1024), p.idesc, k > 0 ? 1u : 0u);
          mma_commit_pair_mc(&empty[stage], 0x3);
          mma_commit_pair_mc(&pfull[slot], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      mma_commit_pair_mc(mma_done, 0x1);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, kStatusTimeoutMma);
    }
  } else if (warp >= kBpEpiWarp0) {
    const int e = (warp - kBpEpiWarp0) >> 2;  // warpgroup: columns [64 e, 64 e + 64)
    const int q = warp & 3;                   // TMEM lane quarter of this warp
    const int row = q * 32 + lane;
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kBpEpiWarp0 + 4 * e) * 32;
    uint8_t* stage_c = smem + L::kCOff + e * L::kCBytes;
    uint32_t g = 0;
    for (int tile = cluster_id; tile < p.num_tiles; tile += num_clusters) {
      bool ok = true;
      int pid_m, pid_n;
      compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
      const int m0 = pid_m * 2 * kBM + (int)rank * kBM;
      const int n0 = pid_n * kBpBN;
      const int grow = m0 + row;
      const bool row_ok = grow < p.M;
      const float* sa_row = p.scale_a + (int64_t)(row_ok ? grow : 0) * p.sa_m;
      // 128x128 B scale tiles: this warpgroup's 64 columns lie in tile (n0 + 64 e) / 128
      const int nb = min((n0 >> 7) + (e >> 1), ((p.N + 127) >> 7) - 1);
      const float* sb_col = p.scale_b + (int64_t)nb * p.sb_n;
      float acc[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0.f;
      float sa_next = row_ok ? __ldg(sa_row) : 0.f;
      float sb_next = __ldg(sb_col);
      for (int kb = 0; kb < p.k_tiles; ++kb, ++g) {
        const float s = __fmul_rn(sa_next, sb_next);
        if (kb + 1 < p.k_tiles) {
          sa_next = row_ok ? __ldg(sa_row + (int64_t)(kb + 1) * p.sa_k) : 0.f;
          sb_next = __ldg(sb_col + (int64_t)(kb + 1) * p.sb_k);
        }
        const uint32_t slot = g % kBpSlots, use = g / kBpSlots;
        bool w = __all_sync(0xffffffffu, mbar_wait_traced(&pfull[slot], use & 1, abort_flag, kStatusTimeoutEpilogue,
                                                          p.trace && wg_tid == 0, 3 + e));
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t = tmem_base + slot * kBpBN + e * 64 + ((uint32_t)(q * 32) << 16);
        if constexpr (kLC == 16) {
          // Two-deep: the load of the next 16 columns is in flight while the
          // FMAs of the current 16 run (tcgen05.wait::ld waits for all of a
          // thread's loads, so each wait covers exactly one load here).
          uint32_t v0[16], v1[16];
          tmem_ld_32x32b_x16(t, v0);
          tmem_ld_wait();
          tmem_regs_after_wait(v0);
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            tmem_ld_32x32b_x16(t + c + 16, v1);
#pragma unroll
            for (int i = 0; i < 16; i += 2)
              fma2_scalar(acc[c + i], acc[c + i + 1], __uint_as_float(v0[i]), __uint_as_float(v0[i + 1]), s);
            tmem_ld_wait();
            tmem_regs_after_wait(v1);
            if (c + 32 < 64) tmem_ld_32x32b_x16(t + c + 32, v0);
            if (c + 32 == 64) {
              // the whole partial is in registers: hand the slot back to the
              // MMA warp before the last FMAs
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&pempty[slot]), 0));
            }
#pragma unroll
            for (int i = 0; i < 16; i += 2)
              fma2_scalar(acc[c + 16 + i], acc[c + 16 + i + 1], __uint_as_float(v1[i]), __uint_as_float(v1[i + 1]),
                          s);
            if (c + 32 < 64) {
              tmem_ld_wait();
              tmem_regs_after_wait(v0);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += kLC) {
            uint32_t v[kLC];
            tmem_ld_32x32b_x32(t + c, v);
            tmem_ld_wait();
            if (c + kLC == 64) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&pempty[slot]), 0));
            }
#pragma unroll
            for (int i = 0; i < kLC; i += 2)
              fma2_scalar(acc[c + i], acc[c + i + 1], __uint_as_float(v[i]), __uint_as_float(v[i + 1]), s);
          }
        }
      }
      if (!wg_all(ok, bar_id)) break;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (p.c_half) {
          __half2 h = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
          pk[i] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          pk[i] = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
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
      if (wg_tid == 0 && m0 < p.M && n0 + e * 64 < p.N) {
        tma_store_2d(&tmC, stage_c, n0 + e * 64, m0);
        bulk_commit_group();
      }
    }
    if (wg_tid == 0) bulk_wait_group0();
  }

  tc_fence_before();
  cluster_sync();
  if (threadIdx.x == 0) trace_add(p.trace, 5, (unsigned long long)(clock64() - t_start));
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kBpSlots * kBpBN);
  }
}

template <int BN>
static cudaError_t launch_bp_t(const GemmLaunch& g, cudaStream_t st) {
  constexpr int kBpEpiGroups = BpShape<BN>::kEpiGroups;
  constexpr int kBpHalfN = BpShape<BN>::kHalfN;
  constexpr int kBpBN = BN;
  constexpr int kStages = (kMaxDynSmem - kBpEpiGroups * kBM * 128 - 1024 - 256) / (kBM * kBK + kBpHalfN * kBK);
  constexpr int S = kStages > 8 ? 8 : kStages;
  BpParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  p.num_pid_m = (int)((g.M + 2 * kBM - 1) / (2 * kBM));
  p.num_pid_n = (int)((g.N + kBpBN - 1) / kBpBN);
  p.num_tiles = p.num_pid_m * p.num_pid_n;
  p.group_size_m = g.group_size_m;
  p.k_tiles = (int)((g.K + kBK - 1) / kBK);
  p.idesc = idesc_f8f6f4(g.a_fmt, g.b_fmt, 0, 0, 2 * kBM, kBpBN);
  p.c_half = g.c_half;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.sa_m = g.sa_stride_m;
  p.sa_k = g.sa_stride_k;
  p.sb_k = g.sb_stride_k;
  p.sb_n = g.sb_stride_n;
  p.trace = g.trace;
  auto kern = fp8_gemm_blockscaled_pair_kernel<S, BN>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), BpSmem<S, BN>::kAlloc);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(BpShape<BN>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = BpSmem<S, BN>::kAlloc;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int max_clusters = 0;
  if (max_clusters == 0) {
    cfg.gridDim = dim3(2 * 74, 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = 74;
    (void)cudaGetLastError();
    max_clusters = n;
  }
  int clusters = p.num_tiles < max_clusters ? p.num_tiles : max_clusters;
  if (clusters > g.num_sms / 2) clusters = g.num_sms / 2;
  if (clusters < 1) clusters = 1;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, g.tmA, g.tmB, g.tmC, p);
  note_launch(1);
  return e;
}

cudaError_t launch_fp8_gemm_blockscaled_pair(const GemmLaunch& g, cudaStream_t st) {
  return g.bn == 256 ? launch_bp_t<256>(g, st) : launch_bp_t<128>(g, st);
}

}  // namespace b2x
