// Internal declarations shared by the b2x host code and kernel launchers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "b2x.h"

namespace b2x {

// Opt-in shared memory per CTA on sm_100 is 232448 bytes; keep 1 KB for the
// kernels' static shared variables.
constexpr int kMaxDynSmem = 232448 - 1024;

// Counts kernel launches (reported through b2x_launch_count()).
void note_launch(int n);

// Sets cudaFuncAttributeMaxDynamicSharedMemorySize once per (device, kernel).
cudaError_t ensure_smem_attr(const void* func, int bytes);

cudaError_t launch_cast(const b2x_cast_args& a, int num_sms, cudaStream_t st);
int cast_num_partials(int64_t nsegs, int num_sms);
cudaError_t launch_amax(const void* x, b2x_dtype xt, int64_t rows, int64_t cols, int64_t ld_x, float* out,
                        uint32_t* partials, int num_sms, cudaStream_t st);

// Fused all-reduce of the GEMM output over the GPUs of one node
// (b2x_fp8_gemm_allreduce).  Signal buffer layout, in 32-bit words on every
// rank: word 0 counts finished reductions (done), word 1 the units this rank
// reduced (diagnostic), word 2 (kArEpochWord) the calls completed on this rank
// when the call count is kept on the device, words [kArArrive0, kArArrive0 +
// units) count, per
// 128 x 256 output unit, the ranks whose partial has landed (kept on the
// unit's owner rank, ar_owner in fp8_gemm_allreduce.cuh).
constexpr int kArMaxRanks = 8;
constexpr int kArArrive0 = 64;
constexpr int kArEpochWord = 2;
struct ArParams {
  int mode;                        // 0 off, 1 NVSwitch multicast, 2 peer loads/stores
  int rank, world;
  uint8_t* c_mc;                   // multicast address of C (mode 1)
  uint8_t* c_peer[kArMaxRanks];    // C on every rank (mode 2)
  uint32_t* sig_peer[kArMaxRanks]; // signal buffer on every rank
  uint32_t* sig_mc;                // multicast address of the signal buffer (mode 1)
  uint32_t done_target;            // value of the done word once this call is complete (host-counted calls)
  uint32_t units;                  // 128 x 256 output units of the call
  int device_epoch;                // 1: the call count lives in word kArEpochWord and the kernel advances it
};

struct GemmLaunch {
  CUtensorMap tmA, tmB, tmC;
  int64_t M, N, K;
  int bn, stages, group_size_m, split_k;
  int a_fmt, b_fmt;  // 0 = e4m3, 1 = e5m2
  int b_mn;          // B stored row-major [K, N]
  int c_half;        // fp16 output instead of bf16
  int scale_mode;
  const float* scale_a;
  const float* scale_b;
  int64_t sa_stride_m, sa_stride_k, sb_stride_k, sb_stride_n;
  float* ws;
  int* counters;
  void* c;
  int64_t ldc;
  int num_sms;
  int pair;          // paired-CTA (cta_group::2) 256x256 tiles
  int small_m;       // M <= 64: 64-row A boxes, 4 K blocks per stage
  int chunk3d;       // small_m with 3-D (x, row, K chunk) A/B tensor maps
  int swap_ab;       // small_m with K-major B: weights on the MMA's M side
  int trace;         // B2X_TRACE=1: per-CTA wait cycles into g_trace
  int clc;           // cluster-launch-control tile scheduling (single-CTA kernel)
  int l2_a, l2_b;    // L2 eviction policy per operand (0 last, 1 normal, 2 first)
  ArParams ar;       // fused all-reduce (pair kernel only)
  int swiglu;        // fused SwiGLU + fp8 quantize epilogue (pair kernel only)
  int sw_mode, sw_fmt;
  float* sw_scale;
  int64_t sw_ld_scale;
  const float* sw_given;
  float* sw_amax;
};

cudaError_t launch_fp8_gemm(const GemmLaunch& g, cudaStream_t st);
cudaError_t launch_fp8_gemm_smallm(const GemmLaunch& g, cudaStream_t st);
int smallm_tokens_tile(int64_t M);
cudaError_t launch_fp8_gemm_pair(const GemmLaunch& g, cudaStream_t st);
cudaError_t launch_fp8_gemm_blockscaled_pair(const GemmLaunch& g, cudaStream_t st);
cudaError_t launch_fp8_gemm_blockscaled(const GemmLaunch& g, cudaStream_t st);
cudaError_t launch_fp8_gemm_mx(const GemmLaunch& g, cudaStream_t st);
size_t mx_workspace_bytes(int64_t M, int64_t N, int64_t K, int bn);
cudaError_t launch_stoch_round(const float* x, const uint32_t* r, void* y, b2x_dtype yt, int64_t rows, int64_t cols,
                               int64_t ld_x, int64_t ld_r, int64_t ld_y, int num_sms, cudaStream_t st, int rs);
cudaError_t launch_splitk_reduce(const void* ws, b2x_dtype wt, void* c, b2x_dtype ct, int64_t M, int64_t N,
                                 int64_t ldc, int split_k, cudaStream_t st);

}  // namespace b2x
