// Pieces shared by the per-tensor and the block-scaled fp8 GEMM kernels.
#pragma once
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"

namespace b2x {

constexpr int kBM = 128;
constexpr int kBK = 128;
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4;

struct GemmParams {
  int M, N, K;
  int num_pid_m, num_pid_n, num_mn_tiles, num_units;
  int group_size_m;
  int k_tiles, k_tiles_per_split, split_k;
  uint32_t idesc;
  int c_half;  // 1: fp16 output, 0: bf16 output
  // scales
  int scale_mode;
  const float* scale_a;
  const float* scale_b;
  // split-K
  float* ws;        // fp32 [M, N] accumulation buffer (zero between calls)
  int* counters;    // [num_mn_tiles] arrival counters (zero between calls)
  void* c;          // raw C pointer (split-K finisher writes directly)
  int64_t ldc;
  int chunk3d;      // small-M kernel: A and B maps are 3-D (x, row, K chunk)
  int trace;        // record per-CTA wait cycles in g_trace
  int stream_k;     // small-M kernel: K blocks of all tiles spread evenly over the grid (SPLIT_K = -1)
  int clc;          // single-CTA kernel: tiles handed out by cluster launch control (grid = one CTA per unit)
  int l2_a, l2_b;   // L2 policy per operand: 0 evict_last, 1 evict_normal, 2 evict_first
  ArParams ar;      // fused all-reduce of C over the node's GPUs (paired kernel)
  // fused SwiGLU + fp8 quantize epilogue (paired kernel, fp8_gemm_swiglu.cuh)
  int sw_mode;            // 0: 1x128 block scales written to sw_scale; 1: given scale, amax into sw_amax;
                          // 2: MX E8M0 bytes per 32 columns written to sw_scale (uint8, row stride in bytes)
  int sw_fmt;             // 0: e4m3, 1: e5m2
  float* sw_scale;        // [M, N/256] fp32 (mode 0) or [M, N/64] uint8 (mode 2)
  int64_t sw_ld_scale;
  const float* sw_given;  // mode 1
  float* sw_amax;         // mode 1, optional: max |h| (atomicMax on the bits; start from 0)
};

__device__ __forceinline__ uint64_t l2_policy(int which) {
  return which == 2 ? policy_evict_first() : (which == 1 ? policy_evict_normal() : policy_evict_last());
}

// Grouped tile order, the same mapping as _compute_pid (blackwell_gemm_ws.py:433-439).
__device__ __forceinline__ void compute_pid(int tile, int num_pid_in_group, int num_pid_m, int group_size_m,
                                            int& pid_m, int& pid_n) {
  int group_id = tile / num_pid_in_group;
  int first_pid_m = group_id * group_size_m;
  int gsm = min(num_pid_m - first_pid_m, group_size_m);
  pid_m = first_pid_m + (tile % gsm);
  pid_n = (tile % num_pid_in_group) / gsm;
}

__device__ __forceinline__ bool wg_all(bool ok, uint32_t bar_id) {
  // AND-reduction over the 128 threads of one epilogue warpgroup.
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(bar_id)
      : "memory");
  return r != 0;
}

}  // namespace b2x
