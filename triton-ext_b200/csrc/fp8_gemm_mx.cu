// MX (microscaling) fp8 GEMM for sm_100a on the tensor core's block-scale
// path: A and B carry one E8M0 scale (a power of two, biased exponent byte)
// per 32 consecutive K elements of each row,
//
//   C[m, n] = sum_j 2^(sA[m, j] - 127) * 2^(sB[n, j] - 127) * (A[m, 32j:32j+32] . B[32j:32j+32, n])
//
// which is the semantics of the reference's `async_dot_scaled` with E8M0
// scales (extensions/utlx/python/utlx_plugin/mma_ops.py:163-237; the formula
// of test_async_dot_scaled, test_tlx.py:2298-2444).  The scales are applied
// by the tensor core itself (tcgen05.mma ... kind::mxf8f6f4.block_scale), so
// the K loop accumulates in one TMEM accumulator as for per-tensor scaling.
//
// Scale factors on their way to the tensor core:
//   global  row-major bytes, sX[row, j] at scale + row * ld + j (as written by
//           the MX cast, b2x_fp8_cast with B2X_SCALE_MX_1x32);
//   prep    mx_scale_tiles_kernel rewrites them, per tile of rows (128 for A,
//           BN for B, padded to 128-row atoms) and per 128-deep K block, into
//           512-byte atoms of 128 rows x 4 scales, byte
//           (r % 32) * 16 + (r / 32) * 4 + j -- the layout of the reference's
//           _swizzle_scale_to_5d (extensions/utlx/test/test_tlx.py:2000-2025),
//           but aligned to this kernel's tiles;
//   smem    the producer fetches a stage's atoms with one bulk copy each,
//           counted on the stage's `full` barrier with the A and B tiles;
//   TMEM    tcgen05.cp .32x128b.warpx4 copies each atom into 4 TMEM columns
//           (lane r % 32 of every sub-partition, column r / 32); the MMA of K
//           sub-block k (32 deep) selects byte k of those words through the
//           scale-factor id of its instruction descriptor.
// One TMEM scale buffer serves every K block: the copy for block kb+1 is
// issued by the MMA thread after the MMAs of block kb, and tcgen05 copies
// and MMAs from one thread execute in issue order.
//
// Tiles are 128 x BN (BN = 128 or 192): two TMEM accumulators of BN columns
// plus 4 + BN/32 scale columns must fit the 512 TMEM columns.  Roles,
// persistent grouped tile order, bounded waits and the ping-pong epilogue
// follow the per-tensor kernel (fp8_gemm.cu).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"

namespace b2x {

struct MxParams {
  int M, N, K;
  int num_pid_m, num_pid_n, num_tiles, group_size_m, k_tiles;
  uint32_t idesc;  // block-scaled instruction descriptor without the scale-factor ids
  int c_half;
  const uint8_t* sf_a;  // tiled scale atoms of A: [num_pid_m][k_tiles][512]
  const uint8_t* sf_b;  // tiled scale atoms of B: [num_pid_n][k_tiles][atoms per tile * 512]
  int trace;
};

template <int BN, int STAGES>
struct MxSmem {
  static constexpr int kABytes = kBM * kBK;             // 16 KB
  static constexpr int kBBytes = BN * kBK;              // 16 / 24 KB
  static constexpr int kSfaBytes = 512;                 // 128 rows x 4 scales
  static constexpr int kSfbBytes = (BN + 127) / 128 * 512;
  static constexpr int kSfBytes = kSfaBytes + kSfbBytes;
  static constexpr int kCBytes = kBM * 128;             // one 64-column bf16 chunk
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kSfOff = kBOff + STAGES * kBBytes;
  static constexpr int kCOff = (kSfOff + STAGES * kSfBytes + 1023) / 1024 * 1024;
  static constexpr int kBarOff = kCOff + 2 * kCBytes;
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kAlloc = kBarOff + kBarBytes + 1024;
};

template <int BN>
struct MxTmem {
  static constexpr uint32_t kSfaCol = 2 * BN;      // after the two accumulators
  static constexpr uint32_t kSfbCol = 2 * BN + 4;
  static constexpr uint32_t kCols = 512;
  static_assert(kSfbCol + (BN + 127) / 128 * 4 <= kCols, "accumulators + scale factors exceed TMEM");
};

// Instruction descriptor for kind::mxf8f6f4 with E8M0 scales and an fp32
// accumulator (K-major A and B).  Bits: [4,6) B scale-factor id, [7,10) A
// format, [10,13) B format, [17,23) N >> 3, [23] scale format (1 = E8M0),
// [24,29) M >> 4, [29,31) A scale-factor id.
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(uint32_t a_fmt, uint32_t b_fmt, uint32_t M, uint32_t N) {
  return (a_fmt << 7) | (b_fmt << 10) | ((N >> 3) << 17) | (1u << 23) | ((M >> 4) << 24);
}
__device__ __forceinline__ uint32_t idesc_with_sf_ids(uint32_t idesc, uint32_t k) {
  return idesc | (k << 4) | (k << 29);
}

// No-swizzle K-major shared-memory descriptor for tcgen05.cp: 8-row core
// matrices of 16-byte rows, `sbo` bytes apart.
__device__ __forceinline__ uint64_t smem_desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100; layout 0 = no swizzle
  return d;
}

// Copy a 32-row x 16-byte smem block to TMEM columns [taddr, taddr + 4) of
// lanes 0-31 in all four sub-partitions (warpx4 broadcast).
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void mma_mxf8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// Row-major E8M0 scales [rows, K/32] -> tiled atoms.  One thread per output
// word (the 4 scales of one row for one 128-deep K block); rows past `rows`
// get zero bytes (their operand rows are zero-filled by TMA).  Grid-stride
// over both operands: words [0, words_a) build A's atoms, the rest B's.
struct MxPrepArgs {
  const uint8_t* src[2];
  int64_t ld[2];
  int rows[2];
  int tile_rows[2];   // 128 for A, BN for B
  int atoms[2];       // 128-row atoms per tile
  uint32_t* dst[2];
  int64_t words[2];
  int k_tiles;
};

__global__ void mx_scale_tiles_kernel(const MxPrepArgs a) {
  const int64_t total = a.words[0] + a.words[1];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int op = i < a.words[0] ? 0 : 1;
    const int64_t w = op ? i - a.words[0] : i;
    // w = ((tile * k_tiles + kb) * atoms + atom) * 128 + word
    const int word = (int)(w & 127);
    const int64_t rest = w >> 7;
    const int atom = (int)(rest % a.atoms[op]);
    const int64_t tk = rest / a.atoms[op];
    const int kb = (int)(tk % a.k_tiles);
    const int64_t tile = tk / a.k_tiles;
    const int r = (word >> 2) + 32 * (word & 3);  // inverse of word = (r % 32) * 4 + r / 32
    const int in_tile = atom * 128 + r;
    const int64_t row = tile * a.tile_rows[op] + in_tile;
    uint32_t v = 0;
    if (in_tile < a.tile_rows[op] && row < a.rows[op])
      v = __ldg(reinterpret_cast<const uint32_t*>(a.src[op] + row * a.ld[op] + (int64_t)kb * 4));
    a.dst[op][w] = v;
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const MxParams p) {
  using L = MxSmem<BN, STAGES>;
  using T = MxTmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long t_start = clock64();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the producer's expect_tx arrive (A, B and scale bytes)
      mbar_init(&empty[s], 1);  // one commit per use
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrive per warp of the epilogue warpgroup
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
    tmem_alloc(tmem_slot, T::kCols);
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
      const uint64_t pol = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0;
      uint32_t pend_phase[STAGES];
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int pid_m, pid_n;
        compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
        const int m0 = pid_m * kBM, n0 = pid_n * BN;
        for (int kb = 0; kb < p.k_tiles; ++kb) {
          if (!mbar_wait_traced(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer, p.trace, 0)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + L::kAOff + stage * L::kABytes;
          uint8_t* sB = smem + L::kBOff + stage * L::kBBytes;
          uint8_t* sSf = smem + L::kSfOff + stage * L::kSfBytes;
          mbar_arrive_expect_tx(&full[stage], L::kABytes + L::kBBytes + L::kSfBytes);
          tma_load_2d(sA, &tmA, &full[stage], kb * kBK, m0, pol);
          tma_load_2d(sB, &tmB, &full[stage], kb * kBK, n0, pol);
          bulk_load_1d(sSf, p.sf_a + ((int64_t)pid_m * p.k_tiles + kb) * L::kSfaBytes, L::kSfaBytes, &full[stage],
                       pol);
          bulk_load_1d(sSf + L::kSfaBytes, p.sf_b + ((int64_t)pid_n * p.k_tiles + kb) * L::kSfbBytes, L::kSfbBytes,
                       &full[stage], pol);
          issued_mask |= 1u << stage;
          pend_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // No TMA write may be in flight when the CTA exits.
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
      const uint32_t sfa_t = tmem_base + T::kSfaCol;
      const uint32_t sfb_t = tmem_base + T::kSfbCol;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        trace_add(p.trace, 7, 1);
        if (!mbar_wait_traced(&tempty[buf], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma, p.trace, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_tiles; ++kb) {
          if (!mbar_wait_traced(&full[stage], phase, abort_flag, kStatusTimeoutMma, p.trace, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kBOff + stage * L::kBBytes);
          const uint32_t sf_addr = smem_u32(smem + L::kSfOff + stage * L::kSfBytes);
          tmem_cp_32x128b_x4(sfa_t, smem_desc_plain(sf_addr, 512, 128));
#pragma unroll
          for (int blk = 0; blk < (BN + 127) / 128; ++blk)
            tmem_cp_32x128b_x4(sfb_t + 4 * blk, smem_desc_plain(sf_addr + L::kSfaBytes + blk * 512, 512, 128));
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            const uint64_t adesc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = smem_desc_sw128(b_addr + k * 32, 16, 1024);
            mma_mxf8f6f4(d_tmem, adesc, bdesc, idesc_with_sf_ids(p.idesc, (uint32_t)k), sfa_t | ((uint32_t)k << 30),
                         sfb_t | ((uint32_t)k << 30), (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);
      }
      mma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, kStatusTimeoutMma);
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const int e = (warp - kEpiWarp0) >> 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 4 * e) * 32;
    uint8_t* stage_c = smem + L::kCOff + e * L::kCBytes;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      if ((local & 1) != e) continue;
      int pid_m, pid_n;
      compute_pid(tile, num_pid_in_group, p.num_pid_m, p.group_size_m, pid_m, pid_n);
      const uint32_t use = (uint32_t)(local >> 1);
      bool ok = mbar_wait_traced(&tfull[e], use & 1, abort_flag, kStatusTimeoutEpilogue, p.trace && wg_tid == 0,
                                 3 + e);
      if (!wg_all(ok, bar_id)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + e * BN + ((uint32_t)(q * 32) << 16);
      const int m0 = pid_m * kBM, n0 = pid_n * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        uint32_t v[64];
        tmem_ld_32x32b_x32(t_row + c0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld_32x32b_x32(t_row + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_ld_wait();
        if (c0 + 64 == BN) {
          // Whole accumulator read: hand it back to the MMA warp (one arrive per warp).
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[e]);
        }
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float lo = __uint_as_float(v[2 * i]), hi = __uint_as_float(v[2 * i + 1]);
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
        if (wg_tid == 0 && n0 + c0 < p.N) {
          tma_store_2d(&tmC, stage_c, n0 + c0, m0);
          bulk_commit_group();
        }
      }
    }
    if (wg_tid == 0) bulk_wait_group0();
  }

  if (threadIdx.x == 0) trace_add(p.trace, 5, (unsigned long long)(clock64() - t_start));
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, T::kCols);
  }
}

template <int BN>
static cudaError_t launch_mx_t(const GemmLaunch& g, cudaStream_t st) {
  constexpr int kStageBytes = kBM * kBK + BN * kBK + 512 + (BN + 127) / 128 * 512;
  constexpr int kFixed = 2 * kBM * 128 + 1024 + 1024 + 256;
  constexpr int kS = (kMaxDynSmem - kFixed) / kStageBytes;
  constexpr int S = kS > 8 ? 8 : kS;
  using L = MxSmem<BN, S>;
  static_assert(L::kAlloc <= kMaxDynSmem, "MX GEMM smem plan exceeds the opt-in limit");
  auto kern = fp8_gemm_mx_kernel<BN, S>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::kAlloc);
  if (e != cudaSuccess) return e;
  MxParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  p.num_pid_m = (int)((g.M + kBM - 1) / kBM);
  p.num_pid_n = (int)((g.N + BN - 1) / BN);
  p.num_tiles = p.num_pid_m * p.num_pid_n;
  p.group_size_m = g.group_size_m;
  p.k_tiles = (int)((g.K + kBK - 1) / kBK);
  p.idesc = idesc_mxf8f6f4(g.a_fmt, g.b_fmt, kBM, BN);
  p.c_half = g.c_half;
  // Tiled scale atoms in the workspace: A's, then B's (256-byte aligned).
  uint8_t* ws = reinterpret_cast<uint8_t*>(g.ws);
  const int64_t sfa_bytes = (int64_t)p.num_pid_m * p.k_tiles * L::kSfaBytes;
  p.sf_a = ws;
  p.sf_b = ws + (sfa_bytes + 255) / 256 * 256;
  MxPrepArgs pa{};
  pa.src[0] = reinterpret_cast<const uint8_t*>(g.scale_a);
  pa.src[1] = reinterpret_cast<const uint8_t*>(g.scale_b);
  pa.ld[0] = g.sa_stride_m;
  pa.ld[1] = g.sb_stride_n;
  pa.rows[0] = (int)g.M;
  pa.rows[1] = (int)g.N;
  pa.tile_rows[0] = kBM;
  pa.tile_rows[1] = BN;
  pa.atoms[0] = 1;
  pa.atoms[1] = (BN + 127) / 128;
  pa.dst[0] = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(p.sf_a));
  pa.dst[1] = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(p.sf_b));
  pa.words[0] = sfa_bytes / 4;
  pa.words[1] = (int64_t)p.num_pid_n * p.k_tiles * L::kSfbBytes / 4;
  pa.k_tiles = p.k_tiles;
  {
    const int64_t total = pa.words[0] + pa.words[1];
    int blocks = (int)((total + 255) / 256);
    if (blocks > 4 * g.num_sms) blocks = 4 * g.num_sms;
    mx_scale_tiles_kernel<<<blocks, 256, 0, st>>>(pa);
    note_launch(1);
  }
  p.trace = g.trace;
  int grid = p.num_tiles < g.num_sms ? p.num_tiles : g.num_sms;
  if (grid < 1) grid = 1;
  fp8_gemm_mx_kernel<BN, S><<<grid, kThreads, L::kAlloc, st>>>(g.tmA, g.tmB, g.tmC, p);
  note_launch(1);
  return cudaGetLastError();
}

// Workspace bytes of the MX GEMM: the tiled scale atoms of A and of B.
size_t mx_workspace_bytes(int64_t M, int64_t N, int64_t K, int bn) {
  const int64_t kt = (K + kBK - 1) / kBK;
  const int64_t a = (M + kBM - 1) / kBM * kt * 512;
  const int64_t b = (N + bn - 1) / bn * kt * ((bn + 127) / 128) * 512;
  return (size_t)((a + 255) / 256 * 256 + (b + 255) / 256 * 256);
}

cudaError_t launch_fp8_gemm_mx(const GemmLaunch& g, cudaStream_t st) {
  return g.bn == 192 ? launch_mx_t<192>(g, st) : launch_mx_t<128>(g, st);
}

}  // namespace b2x
