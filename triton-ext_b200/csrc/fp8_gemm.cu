// Warp-specialized persistent fp8 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
// Native re-design of matmul_kernel_tma_ws_blackwell
// (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:1089-1349):
//   producer warp  (:1293-1349, _process_tile_producer_inner :943-1022)
//       TMA loads of the A and B K-blocks into a ring of STAGES smem buffers;
//   MMA warp       (:1233-1291, _process_tile_mma_inner :828-939)
//       one thread issues tcgen05.mma kind::f8f6f4 into a TMEM accumulator,
//       tcgen05.commit releases each smem stage and, per tile, signals the
//       accumulator full;
//   epilogue       (:1180-1231, _process_tile_epilogue_inner :673-824)
//       two warpgroups ping-pong over two TMEM accumulators (tile i is drained
//       by warpgroup i%2 while the MMA warp fills the other buffer), scale by
//       sA*sB, convert, and TMA-store through a 128B-swizzled staging tile --
//       or, for split-K, reduce fp32 partials with red.global.add.v4.f32.
// The tile order is the reference's grouped order (_compute_pid :433-439) over
// a persistent grid (tile_id += gridDim.x), and a split-K unit covers
// k_tiles_per_split = cdiv(k_tiles, SPLIT_K) K-blocks (:1258-1264).
//
// With p.clc the grid has one CTA per unit and the tiles are handed out by
// cluster launch control, as in the reference's
// matmul_kernel_tma_ws_blackwell_clc (extensions/utlx/tlx/tutorials/
// blackwell_gemm_clc.py:62-281; clc_producer / clc_consumer of
// tlx/language/tlx/dynamic_launch.py): a CTA starts with the unit of its own
// index; warp 3 asks the hardware to cancel a CTA that has not launched yet
// (clusterlaunchcontrol.try_cancel) and publishes the cancelled CTA's index,
// which is the next unit, through a ring of kClcStages 16-byte responses.
// The four roles read every response (the epilogue warpgroups included, to
// keep the tile sequence) and release it; a response with no CTA left ends
// every role's loop.
//
// Thread layout (384 threads): warp 0 producer, warp 1 MMA, warp 2 TMEM
// allocator, warp 3 spare, warps 4-7 epilogue warpgroup 0, warps 8-11
// epilogue warpgroup 1.  BLOCK_M = 128 (one tcgen05 M=128 group), BLOCK_K =
// 128 (one 128-byte swizzle row of fp8), BLOCK_N in {64, 128, 256}.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"

namespace b2x {

// SMALLM: the variant for M <= 64 (decode shapes, HBM-bound).  A is loaded
// as 64-row boxes (the MMA still runs M=128; rows 64-127 of its A operand are
// whatever the neighbouring smem holds and only feed accumulator rows that
// are never stored), and each stage holds kKPS consecutive 128-deep K blocks
// (4 / 2 / 1 for BN = 64 / 128 / 256, about 64 KB per stage), fetched as one
// 3-D box per operand so every row of B is read in 256-512 contiguous bytes.
template <int SMALLM, int BN>
struct MShape {
  static constexpr int kARows = SMALLM ? 64 : 128;
  static constexpr int kKPS = SMALLM ? (BN == 64 ? 4 : (BN == 128 ? 2 : 1)) : 1;
};

constexpr int kClcStages = 3;
constexpr int kClcConsumers = 5;  // producer, MMA, two epilogue warpgroups, the scheduler itself

// SPLITK kernels reduce with red.global and need no C staging tiles.
template <int BN, int STAGES, int SMALLM = 0, int SPLITK = 0>
struct SmemLayout {
  static constexpr int kASub = MShape<SMALLM, BN>::kARows * kBK;  // one K block of A
  static constexpr int kBSub = BN * kBK;                          // one K block of B
  static constexpr int kABytes = kASub * MShape<SMALLM, BN>::kKPS;
  static constexpr int kBBytes = kBSub * MShape<SMALLM, BN>::kKPS;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kCBytes = kBM * 128;        // one 128 x 128 B staging tile per epilogue warpgroup
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kCOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kCOff + (SPLITK ? 0 : 2 * kCBytes);
  // barriers: full[STAGES], empty[STAGES], tfull[2], tempty[2], mma_done, + tmem slot + flags
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  // cluster launch control: kClcStages 16-byte responses, full / empty barriers
  static constexpr int kClcOff = (kBarOff + kBarBytes + 15) / 16 * 16;
  static constexpr int kClcBytes = kClcStages * 16 + 2 * kClcStages * 8;
  static constexpr int kTotal = kClcOff + kClcBytes;
  static constexpr int kAlloc = kTotal + 1024;  // slack to align the base to 1024 B
};

template <int BN>
struct TmemCols {
  static constexpr uint32_t kPerBuf = BN;
  static constexpr uint32_t kAlloc = 2 * BN < 32 ? 32 : 2 * BN;
};

template <int BN, int STAGES, int B_MN, int SPLITK, int SMALLM>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using L = SmemLayout<BN, STAGES, SMALLM, SPLITK>;
  constexpr int KPS = MShape<SMALLM, BN>::kKPS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* clc_resp = smem + L::kClcOff;
  uint64_t* clc_full = reinterpret_cast<uint64_t*>(clc_resp + kClcStages * 16);
  uint64_t* clc_empty = clc_full + kClcStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long t_start = clock64();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(mma_done, 1);
    for (int s = 0; s < kClcStages; ++s) {
      mbar_init(&clc_full[s], 1);
      mbar_init(&clc_empty[s], kClcConsumers);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Next unit of this CTA with p.clc: the next cluster-launch-control
  // response (-1: none left); `ci` counts the responses read.  Every reader
  // waits itself; one thread per role releases the response.
  auto clc_read = [&](int& ci) -> int {
    const int s = ci % kClcStages;
    const uint32_t ph = (uint32_t)(ci / kClcStages) & 1u;
    ++ci;
    if (!mbar_wait(&clc_full[s], ph, abort_flag, kStatusTimeoutProducer)) return -1;
    return clc_first_ctaid_x(clc_resp + s * 16);
  };
  auto clc_release = [&](int ci_after) { mbar_arrive(&clc_empty[(ci_after - 1) % kClcStages]); };
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (!SPLITK) tma_prefetch_desc(&tmC);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TmemCols<BN>::kAlloc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_pid_in_group = p.group_size_m * p.num_pid_n;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;
      uint32_t pend_phase[STAGES > 0 ? STAGES : 1];
      bool ok = true;
      int ci = 0;
      for (int unit = blockIdx.x; unit >= 0 && unit < p.num_units && ok;) {
        const int mn = unit % p.num_mn_tiles;
        const int split = unit / p.num_mn_tiles;
        int pid_m, pid_n;
        compute_pid(mn, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
        const int k0 = split * p.k_tiles_per_split;
        const int k1 = min(k0 + p.k_tiles_per_split, p.k_tiles);
        for (int kb = k0; kb < k1; kb += KPS) {
          if (!mbar_wait_traced(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer, p.trace, 0)) {
            ok = false;
            break;
          }
          const int cnt = min(KPS, k1 - kb);
          uint8_t* sA = smem + L::kAOff + stage * L::kABytes;
          uint8_t* sB = smem + L::kBOff + stage * L::kBBytes;
          if (SMALLM && p.chunk3d) {
            // One 3-D box per operand: KPS consecutive 128-byte K chunks of
            // every row (a box always moves all KPS chunks; chunks past the
            // end of K read as zeros and past this split are simply unused).
            mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
            tma_load_3d(sA, &tmA, &full[stage], 0, pid_m * kBM, kb, pol_a);
            tma_load_3d(sB, &tmB, &full[stage], 0, pid_n * BN, kb, pol_b);
            issued_mask |= 1u << stage;
            pend_phase[stage] = phase;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], cnt * (L::kASub + L::kBSub));
          for (int j = 0; j < cnt; ++j) {
            const int kx = (kb + j) * kBK;
            tma_load_2d(sA + j * L::kASub, &tmA, &full[stage], kx, pid_m * kBM, pol_a);
            if (B_MN) {
              // B row-major [K, N]: slabs of 128 N-columns x 128 K-rows.
#pragma unroll
              for (int s2 = 0; s2 < (BN + 127) / 128; ++s2)
                tma_load_2d(sB + j * L::kBSub + s2 * 128 * kBK, &tmB, &full[stage], pid_n * BN + s2 * 128, kx,
                            pol_b);
            } else {
              tma_load_2d(sB + j * L::kBSub, &tmB, &full[stage], kx, pid_n * BN, pol_b);
            }
          }
          issued_mask |= 1u << stage;
          pend_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (p.clc) {
          unit = clc_read(ci);
          clc_release(ci);
        } else {
          unit += gridDim.x;
        }
      }
      // Never leave the CTA with TMA writes into its shared memory in flight.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], pend_phase[s], &no_abort, kStatusTimeoutProducer);
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      int ci = 0;
      for (int unit = blockIdx.x; unit >= 0 && unit < p.num_units && ok; ++local) {
        const int split = unit / p.num_mn_tiles;
        const int k0 = split * p.k_tiles_per_split;
        const int k1 = min(k0 + p.k_tiles_per_split, p.k_tiles);
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        trace_add(p.trace, 7, 1);
        if (!mbar_wait_traced(&tempty[buf], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma, p.trace, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * TmemCols<BN>::kPerBuf;
        for (int kb = k0; kb < k1; kb += KPS) {
          if (!mbar_wait_traced(&full[stage], phase, abort_flag, kStatusTimeoutMma, p.trace, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const long long t_issue = p.trace ? clock64() : 0;
          const int cnt = min(KPS, k1 - kb);
          for (int j = 0; j < cnt; ++j) {
            const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes + j * L::kASub);
            const uint32_t b_addr = smem_u32(smem + L::kBOff + stage * L::kBBytes + j * L::kBSub);
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k) {
              const uint64_t adesc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
              const uint64_t bdesc = B_MN ? smem_desc_sw128(b_addr + k * 32 * 128, 128 * kBK, 1024)
                                          : smem_desc_sw128(b_addr + k * 32, 16, 1024);
              mma_f8f6f4(d_tmem, adesc, bdesc, p.idesc, (kb > k0 || j > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty[stage]);
          if (p.trace) trace_add(1, 6, (unsigned long long)(clock64() - t_issue));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);
        if (p.clc) {
          unit = clc_read(ci);
          clc_release(ci);
        } else {
          unit += gridDim.x;
        }
      }
      // All MMAs of this thread must finish before TMEM is released.
      mma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, kStatusTimeoutMma);
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const int e = (warp - kEpiWarp0) >> 2;   // warpgroup 0 / 1
    const int q = warp & 3;                  // TMEM lane quarter of this warp
    const int row = q * 32 + lane;           // accumulator row held by this thread
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 4 * e) * 32;
    uint8_t* stage_c = smem + L::kCOff + e * L::kCBytes;
    float alpha = 1.0f;
    if (p.scale_mode != B2X_SCALE_NONE) alpha = __fmul_rn(__ldg(p.scale_a), __ldg(p.scale_b));
    int local = 0, ci = 0;
    for (int unit = blockIdx.x; unit >= 0 && unit < p.num_units; ++local) {
      if ((local & 1) != e) {
        if (p.clc) {
          unit = clc_read(ci);
          named_bar_sync(bar_id, 128);
          if (wg_tid == 0) clc_release(ci);
        } else {
          unit += gridDim.x;
        }
        continue;
      }
      const int mn = unit % p.num_mn_tiles;
      int pid_m, pid_n;
      compute_pid(mn, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
      const uint32_t use = (uint32_t)(local >> 1);
      bool ok = mbar_wait_traced(&tfull[e], use & 1, abort_flag, kStatusTimeoutEpilogue,
                                 p.trace && wg_tid == 0, 3 + e);
      if (!wg_all(ok, bar_id)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + e * TmemCols<BN>::kPerBuf + ((uint32_t)(q * 32) << 16);
      const int m0 = pid_m * kBM, n0 = pid_n * BN;
      const int grow = m0 + row;

      if (!SPLITK) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 64) {
          uint32_t v[64];
          tmem_ld_32x32b_x32(t_row + c0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          tmem_ld_32x32b_x32(t_row + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          tmem_ld_wait();
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
          // The staging tile may still be read by the previous TMA store.
          if (wg_tid == 0) bulk_wait_group_read0();
          named_bar_sync(bar_id, 128);
          const uint32_t srow = smem_u32(stage_c + row * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_v4(srow + ((j ^ (row & 7)) << 4), pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
          fence_proxy_async_smem();
          named_bar_sync(bar_id, 128);
          if (wg_tid == 0) {
            tma_store_2d(&tmC, stage_c, n0 + c0, m0);
            bulk_commit_group();
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[e]);
      } else {
        // Split-K: reduce this unit's fp32 partial into the workspace.  The
        // accumulator buffer goes back to the MMA warp as soon as its last
        // columns are in registers, before the reductions are issued.
        const bool row_ok = grow < p.M;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c0, v);
          tmem_ld_wait();
          if (c0 + 32 == BN) {
            tc_fence_before();
            mbar_arrive(&tempty[e]);
          }
          if (row_ok) {
            float* dst = p.ws + (int64_t)grow * p.N + n0 + c0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int col = n0 + c0 + 4 * j;
              if (col + 3 < p.N) {
                red_add_v4(dst + 4 * j, __uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                           __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
              } else {
                for (int t = 0; t < 4; ++t)
                  if (col + t < p.N) atomicAdd(dst + 4 * j + t, __uint_as_float(v[4 * j + t]));
              }
            }
          }
        }
        // Last unit to arrive on this tile converts the sum and re-zeroes the
        // workspace so the next call finds it clean.  The warpgroup barrier
        // orders every thread's reductions before thread 0's acq_rel counter
        // increment (release is cumulative); the finisher's reads are ordered
        // after it by the same increment (acquire) and the second barrier.
        named_bar_sync(bar_id, 128);
        __shared__ int s_last[2];
        if (wg_tid == 0) {
          int old = atomic_add_acq_rel_gpu(p.counters + mn, 1);
          s_last[e] = (old == p.split_k - 1);
        }
        named_bar_sync(bar_id, 128);
        if (s_last[e]) {
          // Finish the tile with the whole warpgroup: coalesced float4 reads of
          // the fp32 sum (all loads of a batch issued before any store),
          // scaled conversion to C and zeroing of the workspace behind it.
          const int rows_v = min(kBM, p.M - m0);
          const int cols_v = min(BN, p.N - n0);
          const int G = cols_v >> 2;  // float4 groups per row (N % 4 == 0 for split-K)
          const int total = rows_v * G;
          for (int base = wg_tid; base < total; base += 128 * 8) {
            float4 f[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int idx = base + u * 128;
              if (idx < total) {
                const int r = idx / G, cg = idx - r * G;
                f[u] = __ldcg(reinterpret_cast<const float4*>(p.ws + (int64_t)(m0 + r) * p.N + n0 + cg * 4));
              }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int idx = base + u * 128;
              if (idx < total) {
                const int r = idx / G, cg = idx - r * G;
                __stcg(reinterpret_cast<float4*>(p.ws + (int64_t)(m0 + r) * p.N + n0 + cg * 4),
                       make_float4(0.f, 0.f, 0.f, 0.f));
                const float a0 = __fmul_rn(f[u].x, alpha), a1 = __fmul_rn(f[u].y, alpha);
                const float a2 = __fmul_rn(f[u].z, alpha), a3 = __fmul_rn(f[u].w, alpha);
                uint2 o;
                if (p.c_half) {
                  __half2 h0 = __floats2half2_rn(a0, a1), h1 = __floats2half2_rn(a2, a3);
                  o = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
                } else {
                  o = make_uint2(pack_bf16x2(a0, a1), pack_bf16x2(a2, a3));
                }
                *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p.c) + (int64_t)(m0 + r) * p.ldc + n0 +
                                          cg * 4) = o;
              }
            }
          }
          if (wg_tid == 0) p.counters[mn] = 0;
        }
      }
      if (p.clc) {
        unit = clc_read(ci);
        named_bar_sync(bar_id, 128);
        if (wg_tid == 0) clc_release(ci);
      } else {
        unit += gridDim.x;
      }
    }
    if (!SPLITK && wg_tid == 0) bulk_wait_group0();
  } else if (warp == 3) {
    // ------------------------------------------------------------ CLC scheduler
    if (p.clc && lane == 0) {
      for (int i = 0;; ++i) {
        const int s = i % kClcStages;
        const uint32_t ph = (uint32_t)(i / kClcStages) & 1u;
        if (!mbar_wait(&clc_empty[s], ph ^ 1u, abort_flag, kStatusTimeoutProducer)) break;
        fence_proxy_async_smem();  // the consumers' reads of this response precede its rewrite
        mbar_arrive_expect_tx(&clc_full[s], 16);
        clc_try_cancel(clc_resp + s * 16, &clc_full[s]);
        if (!mbar_wait(&clc_full[s], ph, abort_flag, kStatusTimeoutProducer)) break;
        const int next = clc_first_ctaid_x(clc_resp + s * 16);
        mbar_arrive(&clc_empty[s]);
        if (next < 0) break;  // no CTA left: issuing again would be undefined
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_add(p.trace, 5, (unsigned long long)(clock64() - t_start));
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TmemCols<BN>::kAlloc);
  }
}

// ----------------------------------------------------------------------------
// Host launch.

template <int BN, int B_MN, int SPLITK, int SMALLM>
static cudaError_t launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                                 const GemmParams& p, int grid, cudaStream_t st) {
  // Deepest ring that fits next to the two epilogue staging tiles.
  constexpr int kStage = SmemLayout<BN, 1, SMALLM>::kStageBytes;
  constexpr int kS0 = (kMaxDynSmem - (SPLITK ? 0 : 2 * kBM * 128) - 1024 - 256) / kStage;
  constexpr int STAGES = kS0 > 8 ? 8 : kS0;
  using L = SmemLayout<BN, STAGES, SMALLM, SPLITK>;
  static_assert(L::kAlloc <= 232448, "shared memory layout exceeds the 227 KB per-CTA limit");
  auto kern = fp8_gemm_ws_kernel<BN, STAGES, B_MN, SPLITK, SMALLM>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::kAlloc);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, L::kAlloc, st>>>(ta, tb, tc, p);
  note_launch(1);
  return cudaGetLastError();
}

template <int B_MN, int SPLITK>
static cudaError_t dispatch_bn(int bn, int small_m, const CUtensorMap& ta, const CUtensorMap& tb,
                               const CUtensorMap& tc, const GemmParams& p, int grid, cudaStream_t st) {
  if (small_m) {
    switch (bn) {
      case 256: return launch_gemm_t<256, B_MN, SPLITK, 1>(ta, tb, tc, p, grid, st);
      case 128: return launch_gemm_t<128, B_MN, SPLITK, 1>(ta, tb, tc, p, grid, st);
      case 64: return launch_gemm_t<64, B_MN, SPLITK, 1>(ta, tb, tc, p, grid, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (bn) {
    case 256: return launch_gemm_t<256, B_MN, SPLITK, 0>(ta, tb, tc, p, grid, st);
    case 128: return launch_gemm_t<128, B_MN, SPLITK, 0>(ta, tb, tc, p, grid, st);
    case 64: return launch_gemm_t<64, B_MN, SPLITK, 0>(ta, tb, tc, p, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_fp8_gemm(const GemmLaunch& g, cudaStream_t st) {
  GemmParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  p.num_pid_m = (int)((g.M + kBM - 1) / kBM);
  p.num_pid_n = (int)((g.N + g.bn - 1) / g.bn);
  p.num_mn_tiles = p.num_pid_m * p.num_pid_n;
  p.split_k = g.split_k;
  p.num_units = p.num_mn_tiles * g.split_k;
  p.group_size_m = g.group_size_m;
  p.k_tiles = (int)((g.K + kBK - 1) / kBK);
  p.k_tiles_per_split = (p.k_tiles + g.split_k - 1) / g.split_k;
  p.idesc = idesc_f8f6f4(g.a_fmt, g.b_fmt, 0, g.b_mn ? 1 : 0, kBM, g.bn);
  p.c_half = g.c_half;
  p.scale_mode = g.scale_mode;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.ws = g.ws;
  p.counters = g.counters;
  p.c = g.c;
  p.ldc = g.ldc;
  p.chunk3d = g.chunk3d;
  p.trace = g.trace;
  p.clc = g.clc;
  int grid = g.clc ? p.num_units : (p.num_units < g.num_sms ? p.num_units : g.num_sms);
  if (g.split_k > 1) {
    return g.b_mn ? dispatch_bn<1, 1>(g.bn, g.small_m, g.tmA, g.tmB, g.tmC, p, grid, st)
                  : dispatch_bn<0, 1>(g.bn, g.small_m, g.tmA, g.tmB, g.tmC, p, grid, st);
  }
  return g.b_mn ? dispatch_bn<1, 0>(g.bn, g.small_m, g.tmA, g.tmB, g.tmC, p, grid, st)
                : dispatch_bn<0, 0>(g.bn, g.small_m, g.tmA, g.tmB, g.tmC, p, grid, st);
}

}  // namespace b2x
