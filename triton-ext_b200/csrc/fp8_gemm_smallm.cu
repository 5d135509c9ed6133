// Small-M (decode) fp8 GEMM for sm_100a: operands swapped so the weights
// feed the 128-row side of the tensor core.
//
// For M <= 64 tokens the GEMM C[M, N] = A[M, K] . B[K, N] is HBM-bound on B
// (e.g. 64 x 8192 x 28672: 235 MB of weights for 30 GFLOP).  Computing the
// transposed tile  D[n, m] = sum_k B[k, n] A[m, k]  puts 128 weight rows on the
// MMA's M side and the tokens on its N side (N_MMA = M rounded up to 16, at
// most 64), so every byte the tensor core reads from shared memory is useful
// and each K-major weight row is streamed in 256-byte pieces (two 128-deep K
// blocks per stage).  Unit = (128 weight rows, K split); split-K partials are
// reduced with coalesced red.global.add.f32 (a warp covers 32 consecutive n of
// one token row) and the last unit of a tile converts and re-zeroes it, as in
// the main kernel.  Tile order and K ranges follow the reference's split-K
// scheme (blackwell_gemm_ws.py:1258-1264).
//
// Stream-K (p.stream_k, SPLIT_K = -1): the K blocks of all tiles, taken as one
// flat sequence (tile-major), are cut into gridDim.x equal ranges, one per
// CTA, so every SM streams the same number of weight bytes whatever the tile
// count (a fixed split leaves the last wave partly empty: 64 tiles x 8 splits
// is 3.46 waves on 148 SMs).  A CTA's range crosses one or more tiles; each
// piece is a segment, reduced like a split-K unit, and a tile is finished by
// the last of the CTAs whose ranges touch it.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"

namespace b2x {

constexpr int kSmKPS = 2;      // 128-deep K blocks per stage
constexpr int kSmRows = 128;   // weight rows per unit (MMA M)

template <int NT>
struct SmLayout {
  static constexpr int kWSub = kSmRows * kBK;   // 16 KB
  static constexpr int kASub = NT * kBK;        // NT x 128 B
  static constexpr int kWBytes = kWSub * kSmKPS;
  static constexpr int kABytes = kASub * kSmKPS;
  static constexpr int kStageBytes = kWBytes + kABytes;
  static constexpr int kStages0 = (kMaxDynSmem - 1024 - 256) / kStageBytes;
  static constexpr int kStages = kStages0 > 8 ? 8 : kStages0;
  static constexpr int kWOff = 0;
  static constexpr int kAOff = kStages * kWBytes;
  static constexpr int kBarOff = kAOff + kStages * kABytes;
  static constexpr int kBarBytes = (2 * kStages + 5) * 8 + 16;
  static constexpr int kAlloc = kBarOff + kBarBytes + 1024;
};

// Segment i of this CTA: tile nt, K blocks [k0, k1), and the number of
// segments (over all CTAs) that cover the tile.  False past the last one.
struct SmSeg {
  int nt, k0, k1, parts;
};
__device__ __forceinline__ bool smallm_segment(const GemmParams& p, int i, SmSeg& sg) {
  if (!p.stream_k) {
    const int unit = blockIdx.x + i * gridDim.x;
    if (unit >= p.num_units) return false;
    sg.nt = unit % p.num_mn_tiles;
    const int split = unit / p.num_mn_tiles;
    sg.k0 = split * p.k_tiles_per_split;
    sg.k1 = min(sg.k0 + p.k_tiles_per_split, p.k_tiles);
    sg.parts = p.split_k;
    return true;
  }
  const int64_t KT = p.k_tiles;
  const int64_t total = (int64_t)p.num_mn_tiles * KT;
  const int64_t W = (total + gridDim.x - 1) / gridDim.x;
  const int64_t lo = (int64_t)blockIdx.x * W, hi = min(total, lo + W);
  if (lo >= hi) return false;
  const int64_t t = lo / KT + i;
  if (t * KT >= hi) return false;
  sg.nt = (int)t;
  sg.k0 = (int)(max(lo, t * KT) - t * KT);
  sg.k1 = (int)(min(hi, (t + 1) * KT) - t * KT);
  sg.parts = (int)(((t + 1) * KT - 1) / W - (t * KT) / W + 1);
  return true;
}

// tmW: weights [N, K] K-major, box {128, 128}; tmA: activations [M, K], box {128, NT}.
template <int NT, int SPLITK>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_smallm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                           const GemmParams p) {
  using L = SmLayout<NT>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t kBufCols = NT < 32 ? 32 : NT;  // each accumulator buffer owns >= 32 columns
  constexpr uint32_t kTmemCols = 2 * kBufCols;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long t_start = clock64();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrive per epilogue warp
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmA);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();  // weights are streamed once
      const uint64_t pol_a = policy_evict_last();   // activations are re-read by every unit
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0;
      uint32_t pend_phase[S];
      bool ok = true;
      SmSeg sg;
      for (int si = 0; ok && smallm_segment(p, si, sg); ++si) {
        const int nt = sg.nt, k0 = sg.k0, k1 = sg.k1;
        for (int kb = k0; kb < k1; kb += kSmKPS) {
          if (!mbar_wait_traced(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer, p.trace, 0)) {
            ok = false;
            break;
          }
          const int cnt = min(kSmKPS, k1 - kb);
          uint8_t* sW = smem + L::kWOff + stage * L::kWBytes;
          uint8_t* sA = smem + L::kAOff + stage * L::kABytes;
          mbar_arrive_expect_tx(&full[stage], cnt * (L::kWSub + L::kASub));
          for (int j = 0; j < cnt; ++j) {
            tma_load_2d(sW + j * L::kWSub, &tmW, &full[stage], (kb + j) * kBK, nt * kSmRows, pol_w);
            tma_load_2d(sA + j * L::kASub, &tmA, &full[stage], (kb + j) * kBK, 0, pol_a);
          }
          issued_mask |= 1u << stage;
          pend_phase[stage] = phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < S; ++s)
        if (issued_mask & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], pend_phase[s], &no_abort, kStatusTimeoutProducer);
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      SmSeg sg;
      for (int si = 0; ok && smallm_segment(p, si, sg); ++si, ++local) {
        const int k0 = sg.k0, k1 = sg.k1;
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        trace_add(p.trace, 7, 1);
        if (!mbar_wait_traced(&tempty[buf], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma, p.trace, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBufCols;
        for (int kb = k0; kb < k1; kb += kSmKPS) {
          if (!mbar_wait_traced(&full[stage], phase, abort_flag, kStatusTimeoutMma, p.trace, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int cnt = min(kSmKPS, k1 - kb);
          for (int j = 0; j < cnt; ++j) {
            const uint32_t w_addr = smem_u32(smem + L::kWOff + stage * L::kWBytes + j * L::kWSub);
            const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes + j * L::kASub);
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k)
              mma_f8f6f4(d_tmem, smem_desc_sw128(w_addr + k * 32, 16, 1024), smem_desc_sw128(a_addr + k * 32, 16, 1024),
                         p.idesc, (kb > k0 || j > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == S) {
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
    const int e = (warp - kEpiWarp0) >> 2;
    const int q = warp & 3;
    const int nl = q * 32 + lane;  // weight row (output column) held by this thread
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 4 * e) * 32;
    float alpha = 1.0f;
    if (p.scale_mode != B2X_SCALE_NONE) alpha = __fmul_rn(__ldg(p.scale_a), __ldg(p.scale_b));
    __shared__ int s_last[2];
    int local = 0;
    SmSeg sg;
    for (int si = 0; smallm_segment(p, si, sg); ++si, ++local) {
      if ((local & 1) != e) continue;
      const int nt = sg.nt;
      const uint32_t use = (uint32_t)(local >> 1);
      bool ok = mbar_wait_traced(&tfull[e], use & 1, abort_flag, kStatusTimeoutEpilogue, p.trace && wg_tid == 0,
                                 3 + e);
      if (!wg_all(ok, bar_id)) break;
      tc_fence_after();
      const int n = nt * kSmRows + nl;
      const bool n_ok = n < p.N;
      const uint32_t t_row = tmem_base + e * kBufCols + ((uint32_t)(q * 32) << 16);
      uint32_t v[NT < 32 ? 32 : NT];
#pragma unroll
      for (int c0 = 0; c0 < NT; c0 += 32) {
        if (NT >= 32) {
          tmem_ld_32x32b_x32(t_row + c0, *reinterpret_cast<uint32_t(*)[32]>(&v[c0]));
        } else {
          uint32_t tmp[32];
          tmem_ld_32x32b_x32(t_row, tmp);  // NT = 16: the buffer's 32 columns, 16 used
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = tmp[i];
        }
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[e]);
      if (!SPLITK) {
        if (n_ok) {
          uint16_t* c = reinterpret_cast<uint16_t*>(p.c) + n;
#pragma unroll
          for (int m = 0; m < NT; ++m) {
            if (m < p.M) {
              const float o = __fmul_rn(__uint_as_float(v[m]), alpha);
              c[(int64_t)m * p.ldc] = p.c_half ? __half_as_ushort(__float2half_rn(o))
                                              : __bfloat16_as_ushort(__float2bfloat16_rn(o));
            }
          }
        }
      } else {
        if (n_ok) {
          float* w = p.ws + n;
#pragma unroll
          for (int m = 0; m < NT; ++m)
            if (m < p.M) red_add_f32(w + (int64_t)m * p.N, __uint_as_float(v[m]));
        }
        named_bar_sync(bar_id, 128);
        if (wg_tid == 0) {
          int old = atomic_add_acq_rel_gpu(p.counters + nt, 1);
          s_last[e] = (old == sg.parts - 1);
        }
        named_bar_sync(bar_id, 128);
        if (s_last[e]) {
          // Each thread finishes its output column n: coalesced across the
          // warp (32 consecutive n per token row), loads issued first.
          if (n_ok) {
            float f[NT];
#pragma unroll
            for (int m = 0; m < NT; ++m)
              if (m < p.M) f[m] = __ldcg(p.ws + (int64_t)m * p.N + n);
            uint16_t* c = reinterpret_cast<uint16_t*>(p.c) + n;
#pragma unroll
            for (int m = 0; m < NT; ++m) {
              if (m < p.M) {
                __stcg(p.ws + (int64_t)m * p.N + n, 0.f);
                const float o = __fmul_rn(f[m], alpha);
                c[(int64_t)m * p.ldc] = p.c_half ? __half_as_ushort(__float2half_rn(o))
                                                : __bfloat16_as_ushort(__float2bfloat16_rn(o));
              }
            }
          }
          if (wg_tid == 0) p.counters[nt] = 0;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_add(p.trace, 5, (unsigned long long)(clock64() - t_start));
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int NT, int SPLITK>
static cudaError_t launch_smallm_t(const CUtensorMap& tw, const CUtensorMap& ta, const GemmParams& p, int grid,
                                   cudaStream_t st) {
  using L = SmLayout<NT>;
  auto kern = fp8_gemm_smallm_kernel<NT, SPLITK>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::kAlloc);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, L::kAlloc, st>>>(tw, ta, p);
  note_launch(1);
  return cudaGetLastError();
}

int smallm_tokens_tile(int64_t M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

cudaError_t launch_fp8_gemm_smallm(const GemmLaunch& g, cudaStream_t st) {
  const int NT = smallm_tokens_tile(g.M);
  GemmParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  p.num_pid_m = 1;
  p.num_pid_n = (int)((g.N + kSmRows - 1) / kSmRows);
  p.num_mn_tiles = p.num_pid_n;
  p.split_k = g.split_k;
  p.num_units = p.num_mn_tiles * g.split_k;
  p.group_size_m = 1;
  p.k_tiles = (int)((g.K + kBK - 1) / kBK);
  p.k_tiles_per_split = (p.k_tiles + g.split_k - 1) / g.split_k;
  // D[n, m] = W[n, :] . A[m, :]: the weights are the MMA's A operand.
  p.idesc = idesc_f8f6f4(g.b_fmt, g.a_fmt, 0, 0, kSmRows, NT);
  p.c_half = g.c_half;
  p.scale_mode = g.scale_mode;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.ws = g.ws;
  p.counters = g.counters;
  p.c = g.c;
  p.ldc = g.ldc;
  p.trace = g.trace;
  p.stream_k = g.split_k < 0;
  if (p.stream_k) {  // one flat K-block sequence over all tiles, cut into grid equal ranges
    p.split_k = 2;   // any value > 1: selects the reducing epilogue
    p.num_units = p.num_mn_tiles;
    p.k_tiles_per_split = p.k_tiles;
  }
  const int64_t items = (int64_t)p.num_mn_tiles * p.k_tiles;
  const int grid = p.stream_k ? (int)(items < g.num_sms ? items : g.num_sms)
                              : (p.num_units < g.num_sms ? p.num_units : g.num_sms);
  // g.tmB holds the weights (box {128, 128}), g.tmA the activations (box {128, NT}).
  if (g.split_k > 1 || p.stream_k) {
    switch (NT) {
      case 16: return launch_smallm_t<16, 1>(g.tmB, g.tmA, p, grid, st);
      case 32: return launch_smallm_t<32, 1>(g.tmB, g.tmA, p, grid, st);
      default: return launch_smallm_t<64, 1>(g.tmB, g.tmA, p, grid, st);
    }
  }
  switch (NT) {
    case 16: return launch_smallm_t<16, 0>(g.tmB, g.tmA, p, grid, st);
    case 32: return launch_smallm_t<32, 0>(g.tmB, g.tmA, p, grid, st);
    default: return launch_smallm_t<64, 0>(g.tmB, g.tmA, p, grid, st);
  }
}

}  // namespace b2x
