// Block-scaled fp8 GEMM for sm_100a: A with one fp32 scale per (row, 128-deep
// K block), B with one fp32 scale per (128 K x 128 N) tile.
//
//   C[m, n] = sum_kb sA[m, kb] * sB[kb, nb(n)] * (A[m, kb-block] . B[kb-block, n])
//
// The scales change every 128-deep K block and A's scale changes per row, so
// the tensor-core accumulator cannot carry the sum across K blocks.  Instead
// ("per-K-block promotion", the method of DeepSeek's DeepGEMM fp8 kernels):
//   MMA warp      writes the product of each K block into one of four TMEM
//                 partial buffers (128 x 128 fp32 each, 512 columns in all),
//                 signalling `pfull[slot]` through tcgen05.commit;
//   epilogue      two warpgroups split the 128 columns (64 each), load every
//                 partial with tcgen05.ld, release the slot, and promote it
//                 into fp32 register accumulators with the per-row scale;
//                 at the end of the tile they convert and TMA-store.
// Producer, persistent schedule and barrier protocol are those of the
// per-tensor kernel (fp8_gemm.cu), which follows matmul_kernel_tma_ws_blackwell
// (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:1089-1349).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"

namespace b2x {

constexpr int kBsBN = 128;
constexpr int kBsSlots = 4;  // TMEM partial buffers (4 x 128 columns)

struct BsParams {
  int M, N, K;
  int num_pid_m, num_pid_n, num_tiles, group_size_m, k_tiles;
  uint32_t idesc;
  int c_half;
  const float* scale_a;
  const float* scale_b;
  int64_t sa_m, sa_k, sb_k, sb_n;
  int trace;
};

template <int STAGES>
struct BsSmem {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = kBsBN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kCBytes = kBM * 128;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kCOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kCOff + 2 * kCBytes;
  static constexpr int kBarBytes = (2 * STAGES + 2 * kBsSlots + 1) * 8 + 16;
  static constexpr int kAlloc = kBarOff + kBarBytes + 1024;
};

template <int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_blockscaled_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                const __grid_constant__ CUtensorMap tmC, const BsParams p) {
  using L = BsSmem<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;
  uint64_t* pempty = pfull + kBsSlots;
  uint64_t* mma_done = pempty + kBsSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long t_start = clock64();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kBsSlots; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 8);  // one arrive per epilogue warp
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
    tmem_alloc(tmem_slot, kBsSlots * kBsBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_pid_in_group = p.group_size_m * p.num_pid_n;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0;
      uint32_t pend_phase[STAGES];
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int pid_m, pid_n;
        compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
        for (int kb = 0; kb < p.k_tiles; ++kb) {
          if (!mbar_wait_traced(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer, p.trace, 0)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + L::kAOff + stage * L::kABytes;
          uint8_t* sB = smem + L::kBOff + stage * L::kBBytes;
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(sA, &tmA, &full[stage], kb * kBK, pid_m * kBM, pol);
          tma_load_2d(sB, &tmB, &full[stage], kb * kBK, pid_n * kBsBN, pol);
          issued_mask |= 1u << stage;
          pend_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], pend_phase[s], &no_abort, kStatusTimeoutProducer);
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;  // K blocks issued by this CTA so far (drives the slot ring)
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < p.k_tiles; ++kb, ++g) {
          const uint32_t slot = g % kBsSlots, use = g / kBsSlots;
          if (!mbar_wait_traced(&pempty[slot], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma, p.trace, 2) ||
              !mbar_wait_traced(&full[stage], phase, abort_flag, kStatusTimeoutMma, p.trace, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const long long t_issue = p.trace ? clock64() : 0;
          const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kBOff + stage * L::kBBytes);
          const uint32_t d_tmem = tmem_base + slot * kBsBN;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_f8f6f4(d_tmem, smem_desc_sw128(a_addr + k * 32, 16, 1024), smem_desc_sw128(b_addr + k * 32, 16, 1024),
                       p.idesc, k > 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          mma_commit(&pfull[slot]);
          if (p.trace) trace_add(1, 6, (unsigned long long)(clock64() - t_issue));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      mma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, kStatusTimeoutMma);
    }
  } else if (warp >= kEpiWarp0) {
    const int e = (warp - kEpiWarp0) >> 2;  // column half owned by this warpgroup
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 4 * e) * 32;
    uint8_t* stage_c = smem + L::kCOff + e * L::kCBytes;
    uint32_t g = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      bool ok = true;
      int pid_m, pid_n;
      compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
      const int m0 = pid_m * kBM, n0 = pid_n * kBsBN;
      const int grow = m0 + row;
      const bool row_ok = grow < p.M;
      const float* sa_row = p.scale_a + (int64_t)(row_ok ? grow : 0) * p.sa_m;
      const float* sb_col = p.scale_b + (int64_t)pid_n * p.sb_n;
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
        const uint32_t slot = g % kBsSlots, use = g / kBsSlots;
        // Warp-level agreement only: no warpgroup barrier on the per-K-block
        // path.  A warp that gave up skips its work; the warpgroup agrees at
        // the end of the tile.
        bool w = __all_sync(0xffffffffu, mbar_wait_traced(&pfull[slot], use & 1, abort_flag, kStatusTimeoutEpilogue,
                                                          p.trace && wg_tid == 0, 3 + e));
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t = tmem_base + slot * kBsBN + e * 64 + ((uint32_t)(q * 32) << 16);
        uint32_t v[32];
        tmem_ld_32x32b_x32(t, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          fma2_scalar(acc[i], acc[i + 1], __uint_as_float(v[i]), __uint_as_float(v[i + 1]), s);
        tmem_ld_32x32b_x32(t + 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          fma2_scalar(acc[32 + i], acc[32 + i + 1], __uint_as_float(v[i]), __uint_as_float(v[i + 1]), s);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[slot]);
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
      if (wg_tid == 0) {
        tma_store_2d(&tmC, stage_c, n0 + e * 64, m0);
        bulk_commit_group();
      }
    }
    if (wg_tid == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_add(p.trace, 5, (unsigned long long)(clock64() - t_start));
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kBsSlots * kBsBN);
  }
}

cudaError_t launch_fp8_gemm_blockscaled(const GemmLaunch& g, cudaStream_t st) {
  constexpr int kStages = (kMaxDynSmem - 2 * kBM * 128 - 1024 - 256) / (kBM * kBK + kBsBN * kBK);
  constexpr int S = kStages > 8 ? 8 : kStages;
  BsParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  p.num_pid_m = (int)((g.M + kBM - 1) / kBM);
  p.num_pid_n = (int)((g.N + kBsBN - 1) / kBsBN);
  p.num_tiles = p.num_pid_m * p.num_pid_n;
  p.group_size_m = g.group_size_m;
  p.k_tiles = (int)((g.K + kBK - 1) / kBK);
  p.idesc = idesc_f8f6f4(g.a_fmt, g.b_fmt, 0, 0, kBM, kBsBN);
  p.c_half = g.c_half;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.sa_m = g.sa_stride_m;
  p.sa_k = g.sa_stride_k;
  p.sb_k = g.sb_stride_k;
  p.sb_n = g.sb_stride_n;
  p.trace = g.trace;
  auto kern = fp8_gemm_blockscaled_kernel<S>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), BsSmem<S>::kAlloc);
  if (e != cudaSuccess) return e;
  int grid = p.num_tiles < g.num_sms ? p.num_tiles : g.num_sms;
  kern<<<grid, kThreads, BsSmem<S>::kAlloc, st>>>(g.tmA, g.tmB, g.tmC, p);
  note_launch(1);
  return cudaGetLastError();
}

}  // namespace b2x
