// Grouped fp8 GEMM for sm_100a: one persistent launch computes a list of
// independent GEMMs C_g = sA_g * sB_g * (A_g . B_g^T) of different shapes
// (the expert layers of a mixture-of-experts block).
//
// Counterpart of the reference's grouped GEMM tutorial,
// grouped_matmul_tlx_kernel (extensions/utlx/tlx/tutorials/
// blackwell-grouped-gemm_test.py:366-668) with its host wrapper
// group_gemm_tlx_fn (:727-784): device arrays of A/B/C pointers, sizes and
// leading dimensions, tiles of all groups enumerated over a fixed number of
// persistent CTAs.  Here the host writes one descriptor per group -- the
// three TMA tensor maps plus shape, tile count and scales -- into the
// caller's workspace, and every role of every CTA walks the same global tile
// sequence: tile t belongs to the group whose [tile0, tile0 + tiles) holds
// it, and inside a group tiles follow the grouped order of the plain GEMM
// (compute_pid).  Producer / MMA / ping-pong epilogue and the bounded waits
// are those of the per-tensor kernel (fp8_gemm.cu); tiles are 128 x BN
// (BN = 128 or 256) on one CTA.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdlib>
#include <vector>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"
#include "fp8_gemm_common.cuh"

namespace b2x {

struct __align__(64) GroupDesc {
  CUtensorMap a, b, c;  // A [M, K], B [N, K] (K-major), C [M, N]
  int M, N, K, k_tiles;
  int num_pid_m, num_pid_n, tile0, group_size_m;
  const float* scale_a;  // per-tensor scales (NULL: 1)
  const float* scale_b;
  int c_half, a_fmt, b_fmt, pad_;
};

struct GroupedParams {
  const GroupDesc* groups;
  int num_groups;
  int total_tiles;
  int trace;
};

template <int BN, int STAGES>
struct GrSmem {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kCBytes = kBM * 128;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kCOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kCOff + 2 * kCBytes;
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kAlloc = kBarOff + kBarBytes + 1024;
};

// Advance `g` to the group holding global tile `t` (tiles are visited in
// increasing order, so the scan only moves forward).
__device__ __forceinline__ int advance_group(const GroupedParams& p, int g, int t) {
  while (g + 1 < p.num_groups && t >= p.groups[g + 1].tile0) ++g;
  return g;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) fp8_gemm_grouped_kernel(const GroupedParams p) {
  using L = GrSmem<BN, STAGES>;
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
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrive per warp of the epilogue warpgroup
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      int stage = 0, g = 0, prefetched = -1;
      uint32_t phase = 0, issued_mask = 0;
      uint32_t pend_phase[STAGES];
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        g = advance_group(p, g, tile);
        const GroupDesc* G = p.groups + g;
        if (g != prefetched) {
          tma_prefetch_desc(&G->a);
          tma_prefetch_desc(&G->b);
          prefetched = g;
        }
        int pid_m, pid_n;
        compute_pid(tile - G->tile0, G->group_size_m * G->num_pid_n, G->num_pid_m, G->group_size_m, pid_m, pid_n);
        const int k_tiles = G->k_tiles;
        for (int kb = 0; kb < k_tiles; ++kb) {
          if (!mbar_wait_traced(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutProducer, p.trace, 0)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + L::kAOff + stage * L::kABytes;
          uint8_t* sB = smem + L::kBOff + stage * L::kBBytes;
          mbar_arrive_expect_tx(&full[stage], L::kABytes + L::kBBytes);
          tma_load_2d(sA, &G->a, &full[stage], kb * kBK, pid_m * kBM, pol);
          tma_load_2d(sB, &G->b, &full[stage], kb * kBK, pid_n * BN, pol);
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
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, local = 0, g = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++local) {
        g = advance_group(p, g, tile);
        const int k_tiles = p.groups[g].k_tiles;
        const uint32_t idesc = idesc_f8f6f4(p.groups[g].a_fmt, p.groups[g].b_fmt, 0, 0, kBM, BN);
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        trace_add(p.trace, 7, 1);
        if (!mbar_wait_traced(&tempty[buf], (use & 1) ^ 1, abort_flag, kStatusTimeoutMma, p.trace, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < k_tiles; ++kb) {
          if (!mbar_wait_traced(&full[stage], phase, abort_flag, kStatusTimeoutMma, p.trace, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::kAOff + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kBOff + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_f8f6f4(d_tmem, smem_desc_sw128(a_addr + k * 32, 16, 1024), smem_desc_sw128(b_addr + k * 32, 16, 1024),
                       idesc, (kb > 0 || k > 0) ? 1u : 0u);
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
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t bar_id = 1 + e;
    const int wg_tid = threadIdx.x - (kEpiWarp0 + 4 * e) * 32;
    uint8_t* stage_c = smem + L::kCOff + e * L::kCBytes;
    int local = 0, g = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++local) {
      g = advance_group(p, g, tile);
      if ((local & 1) != e) continue;
      const GroupDesc* G = p.groups + g;
      int pid_m, pid_n;
      compute_pid(tile - G->tile0, G->group_size_m * G->num_pid_n, G->num_pid_m, G->group_size_m, pid_m, pid_n);
      const float alpha = (G->scale_a && G->scale_b) ? __fmul_rn(__ldg(G->scale_a), __ldg(G->scale_b)) : 1.0f;
      const int c_half = G->c_half, N = G->N;
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
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[e]);
        }
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float lo = __fmul_rn(__uint_as_float(v[2 * i]), alpha);
          const float hi = __fmul_rn(__uint_as_float(v[2 * i + 1]), alpha);
          if (c_half) {
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
        if (wg_tid == 0 && n0 + c0 < N) {
          tma_store_2d(&G->c, stage_c, n0 + c0, m0);
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
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

template <int BN>
static cudaError_t launch_grouped_t(const GroupDesc* d_groups, int num_groups, int total_tiles, int num_sms,
                                    int trace, cudaStream_t st) {
  constexpr int kS = (kMaxDynSmem - 2 * kBM * 128 - 1024 - 256) / (kBM * kBK + BN * kBK);
  constexpr int S = kS > 8 ? 8 : kS;
  using L = GrSmem<BN, S>;
  static_assert(L::kAlloc <= kMaxDynSmem, "grouped GEMM smem plan exceeds the opt-in limit");
  auto kern = fp8_gemm_grouped_kernel<BN, S>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::kAlloc);
  if (e != cudaSuccess) return e;
  GroupedParams p;
  p.groups = d_groups;
  p.num_groups = num_groups;
  p.total_tiles = total_tiles;
  p.trace = trace;
  int grid = total_tiles < num_sms ? total_tiles : num_sms;
  if (grid < 1) grid = 1;
  kern<<<grid, kThreads, L::kAlloc, st>>>(p);
  note_launch(1);
  return cudaGetLastError();
}

}  // namespace b2x

// ---------------------------------------------------------------- C ABI

extern "C" B2X_API size_t b2x_grouped_gemm_workspace_size(int num_groups) {
  return num_groups <= 0 ? 0 : (size_t)num_groups * sizeof(b2x::GroupDesc);
}

extern "C" B2X_API b2x_status b2x_fp8_grouped_gemm(const b2x_gemm_group* groups, int num_groups, b2x_dtype a_type,
                                                   b2x_dtype b_type, b2x_dtype c_type, int block_n, void* workspace,
                                                   size_t workspace_bytes, void* stream) {
  using namespace b2x;
  t_err[0] = 0;
  if (num_groups < 0 || (num_groups > 0 && !groups))
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_grouped_gemm: bad group list");
  if (num_groups == 0) return B2X_OK;
  if (!is_fp8(a_type) || !is_fp8(b_type))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_grouped_gemm: A and B must be e4m3 or e5m2");
  if (c_type != B2X_BF16 && c_type != B2X_F16)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_grouped_gemm: C must be bf16 or fp16");
  if (block_n != 0 && block_n != 128 && block_n != 256)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_grouped_gemm: block_n must be 0 (pick), 128 or 256");
  if (!workspace || workspace_bytes < b2x_grouped_gemm_workspace_size(num_groups) || ((uintptr_t)workspace % 64))
    return fail(B2X_ERR_WORKSPACE, "b2x_fp8_grouped_gemm: needs a 64-byte aligned workspace of %zu bytes",
                b2x_grouped_gemm_workspace_size(num_groups));
  int bn = block_n;
  if (bn == 0) {
    // 256-wide tiles unless no group is wider than 128 columns.
    int64_t max_n = 0;
    for (int i = 0; i < num_groups; ++i) max_n = groups[i].N > max_n ? groups[i].N : max_n;
    bn = max_n > 128 ? 256 : 128;
  }
  thread_local std::vector<GroupDesc> descs;
  descs.assign((size_t)num_groups, GroupDesc{});
  int64_t tiles = 0;
  for (int i = 0; i < num_groups; ++i) {
    const b2x_gemm_group& G = groups[i];
    GroupDesc& d = descs[(size_t)i];
    if (G.M < 0 || G.N < 0 || G.K < 0)
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_grouped_gemm: group %d has a negative shape", i);
    if (G.M >= (1LL << 31) || G.N >= (1LL << 31) || G.K >= (1LL << 31))
      return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_grouped_gemm: group %d: dimensions must be < 2^31", i);
    d.M = (int)G.M;
    d.N = (int)G.N;
    d.K = (int)G.K;
    d.tile0 = (int)tiles;
    d.c_half = c_type == B2X_F16 ? 1 : 0;
    d.a_fmt = a_type == B2X_E4M3 ? 0 : 1;
    d.b_fmt = b_type == B2X_E4M3 ? 0 : 1;
    d.scale_a = G.scale_a;
    d.scale_b = G.scale_b;
    if (G.M == 0 || G.N == 0) continue;  // no tiles
    if (G.K == 0) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_grouped_gemm: group %d has K == 0", i);
    if (!G.a || !G.b || !G.c) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_grouped_gemm: group %d has a NULL pointer", i);
    if ((G.scale_a == nullptr) != (G.scale_b == nullptr))
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_grouped_gemm: group %d: give both scales or neither", i);
    if (G.lda < G.K || G.ldb < G.K || G.ldc < G.N || (G.lda % 16) || (G.ldb % 16) || (G.ldc % 8) ||
        ((uintptr_t)G.a % 16) || ((uintptr_t)G.b % 16) || ((uintptr_t)G.c % 16))
      return fail(B2X_ERR_INVALID_ARG,
                  "b2x_fp8_grouped_gemm: group %d: A, B (K-major [N, K]) and C need 16-byte aligned bases, "
                  "lda/ldb >= K and %% 16 == 0, ldc >= N and %% 8 == 0",
                  i);
    d.k_tiles = (int)((G.K + kBK - 1) / kBK);
    d.num_pid_m = (int)((G.M + kBM - 1) / kBM);
    d.num_pid_n = (int)((G.N + bn - 1) / bn);
    d.group_size_m = d.num_pid_m < 8 ? d.num_pid_m : 8;  // _select_group_size_m's default band
    tiles += (int64_t)d.num_pid_m * d.num_pid_n;
    if (tiles >= (1LL << 31)) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_grouped_gemm: too many tiles");
  }
  if (tiles == 0) return B2X_OK;
  // Every group is valid: build the tensor maps.
  for (int i = 0; i < num_groups; ++i) {
    const b2x_gemm_group& G = groups[i];
    GroupDesc& d = descs[(size_t)i];
    if (G.M == 0 || G.N == 0) continue;
    b2x_status s = encode_2d(&d.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, G.a, (uint64_t)G.K, (uint64_t)G.M,
                             (uint64_t)G.lda, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B, "grouped A");
    if (s != B2X_OK) return s;
    s = encode_2d(&d.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, G.b, (uint64_t)G.K, (uint64_t)G.N, (uint64_t)G.ldb, 128,
                  (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B, "grouped B");
    if (s != B2X_OK) return s;
    s = encode_2d(&d.c, c_type == B2X_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, G.c,
                  (uint64_t)G.N, (uint64_t)G.M, (uint64_t)G.ldc * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B,
                  "grouped C");
    if (s != B2X_OK) return s;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  // Pageable source: the copy has consumed `descs` when this call returns.
  e = cudaMemcpyAsync(workspace, descs.data(), descs.size() * sizeof(GroupDesc), cudaMemcpyHostToDevice,
                      (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "b2x_fp8_grouped_gemm: copying the group descriptors");
  static const int trace_env = [] {
    const char* v = getenv("B2X_TRACE");
    return v && v[0] == '1' ? 1 : 0;
  }();
  const GroupDesc* d_groups = reinterpret_cast<const GroupDesc*>(workspace);
  e = bn == 256 ? launch_grouped_t<256>(d_groups, num_groups, (int)tiles, device_num_sms(dev), trace_env,
                                        (cudaStream_t)stream)
                : launch_grouped_t<128>(d_groups, num_groups, (int)tiles, device_num_sms(dev), trace_env,
                                        (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "b2x_fp8_grouped_gemm launch");
  return B2X_OK;
}
