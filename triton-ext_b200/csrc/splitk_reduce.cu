// Reference-compatible split-K reduction, the counterpart of _reduce_k_kernel
// (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:1033-1056):
//   c[m, n] = cast(sum_s ws[s*M + m, n])   (fp32 sum, planes of M x N, row stride N)
// The fused GEMM path does not need it (its partials are reduced in fp32 by
// red.global.add inside the GEMM); it is exported for callers that produce
// the reference's plane layout themselves.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "b2x_internal.h"

namespace b2x {

__device__ __forceinline__ float load_any(const void* p, int64_t i, int t) {
  if (t == B2X_F32) return reinterpret_cast<const float*>(p)[i];
  if (t == B2X_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_any(void* p, int64_t i, int t, float v) {
  if (t == B2X_F32)
    reinterpret_cast<float*>(p)[i] = v;
  else if (t == B2X_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

__global__ void __launch_bounds__(256) splitk_reduce_kernel(const void* ws, int wt, void* c, int ct, int64_t M,
                                                            int64_t N, int64_t ldc, int split_k) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float acc = 0.f;
    for (int s = 0; s < split_k; ++s) acc += load_any(ws, (int64_t)s * total + i, wt);
    store_any(c, m * ldc + n, ct, acc);
  }
}

cudaError_t launch_splitk_reduce(const void* ws, b2x_dtype wt, void* c, b2x_dtype ct, int64_t M, int64_t N,
                                 int64_t ldc, int split_k, cudaStream_t st) {
  int64_t total = M * N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  splitk_reduce_kernel<<<(int)blocks, 256, 0, st>>>(ws, wt, c, ct, M, N, ldc, split_k);
  note_launch(1);
  return cudaGetLastError();
}

}  // namespace b2x
