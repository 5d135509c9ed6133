// fp32/bf16 -> fp8 (e4m3fn / e5m2) quantization kernels for sm_100a.
//
// Semantics follow the reference quantize recipe, _compute_scale_and_quantize
// (extensions/utlx/tlx/language/tlx/mxfp8_utils.py:37-84):
//   amax  = NaN-ignoring max |x| over the scale group         (:49-50)
//   scale = amax / FMAX                                        (:53)
//   [MX 1x32 only] scale rounded up to a power of two (RCEIL)  (:59-65)
//   inv   = scale == 0 ? 0 : 1 / scale                         (:69)
//   q     = rne_satfinite_fp8(clamp(x * inv, -FMAX, FMAX))     (:72-84)
// with IEEE-rounded divisions and a single (non-fused) multiply.
//
// Work decomposition: a "segment" is 128 consecutive columns of one row; one
// warp owns a segment at a time and each lane holds 4 consecutive elements
// (16 B of fp32 / 8 B of bf16 per load, 4 B of fp8 per store, so a warp moves
// fully coalesced 512 B / 256 B in and 128 B out).  Segments are unrolled
// SEGS_PER_ITER deep per warp to keep enough bytes in flight for HBM3e.
#include <cuda_bf16.h>
#include <cstdint>
#include "b2x_ptx.cuh"
#include "b2x_internal.h"

namespace b2x {

template <int FP8>
struct Fp8Traits;
template <>
struct Fp8Traits<0> {  // e4m3fn
  static constexpr float kMax = 448.0f;
};
template <>
struct Fp8Traits<1> {  // e5m2
  static constexpr float kMax = 57344.0f;
};

template <int FP8>
__device__ __forceinline__ uint16_t cvt2(float lo, float hi) {
  if constexpr (FP8 == 0)
    return cvt_e4m3x2(lo, hi);
  else
    return cvt_e5m2x2(lo, hi);
}

// clamp(y, -m, m) as a B200 computes the reference's symmetric
// tl.clamp(propagate_nan=NONE): the magnitude is limited with a NaN-ignoring
// min and the sign bit of y is kept, so a NaN becomes +m or -m by its sign
// bit.  Pinned by the golden vectors in tests/golden (recorded on a B200 from
// a plain-Triton restatement of the recipe).
__device__ __forceinline__ float clamp_sym(float y, float m) { return copysignf(fminf(fabsf(y), m), y); }

// Quantize 4 values.  SCALED: multiply by inv first; the GPU's fp32 multiply
// returns the canonical (positive) NaN for any NaN result, so after scaling
// every NaN -- including Inf * 0 -- saturates to +FMAX.  Unscaled (mode NONE,
// where the recipe has no multiply) a NaN keeps its sign.
template <int FP8, bool SCALED = true>
__device__ __forceinline__ uint32_t quant4(float4 v, float inv) {
  constexpr float M = Fp8Traits<FP8>::kMax;
  if (SCALED) {
    v.x = __fmul_rn(v.x, inv);
    v.y = __fmul_rn(v.y, inv);
    v.z = __fmul_rn(v.z, inv);
    v.w = __fmul_rn(v.w, inv);
  }
  float a = clamp_sym(v.x, M), b = clamp_sym(v.y, M), c = clamp_sym(v.z, M), d = clamp_sym(v.w, M);
  return (uint32_t)cvt2<FP8>(a, b) | ((uint32_t)cvt2<FP8>(c, d) << 16);
}

__device__ __forceinline__ float nan_ignoring_absmax(float m, float v) { return fmaxf(m, fabsf(v)); }
__device__ __forceinline__ float absmax4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Load 4 consecutive elements starting at column `col` of a row; elements at
// or beyond `cols` read as 0.  `vec_ok` says the row base is aligned so a
// full 4-wide vector load is legal.
template <typename T>
__device__ __forceinline__ float4 load4(const T* row, int64_t col, int64_t cols, bool vec_ok);

template <>
__device__ __forceinline__ float4 load4<float>(const float* row, int64_t col, int64_t cols, bool vec_ok) {
  if (vec_ok && col + 3 < cols) return __ldcs(reinterpret_cast<const float4*>(row + col));
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col + 0 < cols) r.x = row[col + 0];
  if (col + 1 < cols) r.y = row[col + 1];
  if (col + 2 < cols) r.z = row[col + 2];
  if (col + 3 < cols) r.w = row[col + 3];
  return r;
}

template <>
__device__ __forceinline__ float4 load4<uint16_t>(const uint16_t* row, int64_t col, int64_t cols, bool vec_ok) {
  if (vec_ok && col + 3 < cols) {
    uint2 u = __ldcs(reinterpret_cast<const uint2*>(row + col));
    return make_float4(bf16_bits_to_f32(u.x & 0xFFFF), bf16_bits_to_f32(u.x >> 16), bf16_bits_to_f32(u.y & 0xFFFF),
                       bf16_bits_to_f32(u.y >> 16));
  }
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col + 0 < cols) r.x = bf16_bits_to_f32(row[col + 0]);
  if (col + 1 < cols) r.y = bf16_bits_to_f32(row[col + 1]);
  if (col + 2 < cols) r.z = bf16_bits_to_f32(row[col + 2]);
  if (col + 3 < cols) r.w = bf16_bits_to_f32(row[col + 3]);
  return r;
}

__device__ __forceinline__ void store4(uint8_t* row, int64_t col, int64_t cols, bool vec_ok, uint32_t q) {
  if (vec_ok && col + 3 < cols) {
    __stcs(reinterpret_cast<uint32_t*>(row + col), q);
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (col + i < cols) row[col + i] = (uint8_t)(q >> (8 * i));
}

struct CastGeom {
  const void* x;
  int64_t rows, cols, ld_x;
  uint8_t* q;
  int64_t ld_q;
  int64_t segs_per_row;  // ceil(cols / 128)
  int64_t nsegs;         // rows * segs_per_row
  bool x_vec, q_vec;     // vector loads / stores legal
};

template <int SEGS>
struct SegBatch {
  int64_t row[SEGS];
  int64_t col[SEGS];
  bool valid[SEGS];
};

// ----------------------------------------------------------------------------
// Per-tensor amax, pass 1: each CTA writes the NaN-ignoring max |x| of its
// share into partials[blockIdx.x] (as fp32 bits; values are >= 0 so the bit
// patterns order like the floats).
template <typename T, int SEGS>
__global__ void __launch_bounds__(256) amax_partial_kernel(CastGeom g, uint32_t* partials) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(g.x);
  float m = 0.f;
  for (int64_t s0 = warp * SEGS; s0 < g.nsegs; s0 += nwarps * SEGS) {
    float4 v[SEGS];
#pragma unroll
    for (int u = 0; u < SEGS; ++u) {
      int64_t s = s0 + u;
      if (s < g.nsegs) {
        int64_t r = g.segs_per_row == 1 ? s : s / g.segs_per_row;
        int64_t c = (s - r * g.segs_per_row) * 128 + lane * 4;
        v[u] = load4<T>(x + r * g.ld_x, c, g.cols, g.x_vec);
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < SEGS; ++u) m = fmaxf(m, absmax4(v[u]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[32];
  if (lane == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) partials[blockIdx.x] = __float_as_uint(t);
  }
}

// Final reduction of the partials by one CTA (every CTA of the quantize pass
// repeats it; the partials are a few KB and sit in L2).
__device__ __forceinline__ float reduce_partials(const uint32_t* partials, int n) {
  float m = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, __uint_as_float(__ldcg(partials + i)));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red2[32];
  __shared__ float result;
  if ((threadIdx.x & 31) == 0) red2[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red2[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) result = t;
  }
  __syncthreads();
  return result;
}

__global__ void amax_final_kernel(const uint32_t* partials, int n, float* out) {
  float m = reduce_partials(partials, n);
  if (threadIdx.x == 0) *out = m;
}

// ----------------------------------------------------------------------------
// Uniform-scale quantize: modes NONE (inv = 1), TENSOR_GIVEN (inv from
// scale[0]) and TENSOR (inv from the amax partials; CTA 0 writes scale[0]).
template <typename T, int FP8, int SEGS>
__global__ void __launch_bounds__(256) quant_uniform_kernel(CastGeom g, int mode, float* scale,
                                                            const uint32_t* partials, int npartials) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  __shared__ float s_inv;
  if (mode == B2X_SCALE_TENSOR) {
    float amax = reduce_partials(partials, npartials);
    if (threadIdx.x == 0) {
      float sc = __fdiv_rn(amax, FM);
      s_inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
      if (blockIdx.x == 0) *scale = sc;
    }
  } else if (threadIdx.x == 0) {
    if (mode == B2X_SCALE_TENSOR_GIVEN) {
      float sc = *scale;
      s_inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
    } else {
      s_inv = 1.0f;
    }
  }
  __syncthreads();
  const float inv = s_inv;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(g.x);
  for (int64_t s0 = warp * SEGS; s0 < g.nsegs; s0 += nwarps * SEGS) {
    float4 v[SEGS];
    int64_t rr[SEGS], cc[SEGS];
#pragma unroll
    for (int u = 0; u < SEGS; ++u) {
      int64_t s = s0 + u;
      rr[u] = -1;
      if (s < g.nsegs) {
        int64_t r = g.segs_per_row == 1 ? s : s / g.segs_per_row;
        rr[u] = r;
        cc[u] = (s - r * g.segs_per_row) * 128 + lane * 4;
        v[u] = load4<T>(x + r * g.ld_x, cc[u], g.cols, g.x_vec);
      }
    }
    if (mode == B2X_SCALE_NONE) {
#pragma unroll
      for (int u = 0; u < SEGS; ++u)
        if (rr[u] >= 0) store4(g.q + rr[u] * g.ld_q, cc[u], g.cols, g.q_vec, quant4<FP8, false>(v[u], inv));
    } else {
#pragma unroll
      for (int u = 0; u < SEGS; ++u)
        if (rr[u] >= 0) store4(g.q + rr[u] * g.ld_q, cc[u], g.cols, g.q_vec, quant4<FP8>(v[u], inv));
    }
  }
}

// ----------------------------------------------------------------------------
// Row-block scales: GROUP = 128 (fp32 scale per 1x128) or 32 (E8M0 per 1x32).
// A warp covers one 128-column segment: 128/GROUP groups of GROUP/4 lanes.
template <typename T, int FP8, int GROUP, int SEGS>
__global__ void __launch_bounds__(256) quant_rowblock_kernel(CastGeom g, void* scale, int64_t ld_scale) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  constexpr int LPG = GROUP / 4;  // lanes per group
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(g.x);
  for (int64_t s0 = warp * SEGS; s0 < g.nsegs; s0 += nwarps * SEGS) {
    float4 v[SEGS];
    int64_t rr[SEGS], cc[SEGS];
#pragma unroll
    for (int u = 0; u < SEGS; ++u) {
      int64_t s = s0 + u;
      rr[u] = -1;
      cc[u] = 0;
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (s < g.nsegs) {
        int64_t r = g.segs_per_row == 1 ? s : s / g.segs_per_row;
        rr[u] = r;
        cc[u] = (s - r * g.segs_per_row) * 128 + lane * 4;
        v[u] = load4<T>(x + r * g.ld_x, cc[u], g.cols, g.x_vec);
      }
    }
#pragma unroll
    for (int u = 0; u < SEGS; ++u) {
      // Lanes of a segment past the end of the tensor take part in the
      // shuffles (they hold zeros) but store nothing.
      float m = absmax4(v[u]);
#pragma unroll
      for (int o = LPG / 2; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float inv;
      if constexpr (GROUP == 32) {
        float descale = __fdiv_rn(m, FM);
        uint32_t e = (__float_as_uint(descale) + 0x007FFFFFu) & 0x7F800000u;
        float rounded = __uint_as_float(e);
        inv = rounded == 0.f ? 0.f : __fdiv_rn(1.0f, rounded);
        if (rr[u] >= 0 && (lane % LPG) == 0 && cc[u] < g.cols)
          reinterpret_cast<uint8_t*>(scale)[rr[u] * ld_scale + cc[u] / GROUP] = (uint8_t)(e >> 23);
      } else {
        float sc = __fdiv_rn(m, FM);
        inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
        if (rr[u] >= 0 && lane == 0 && cc[u] < g.cols)
          reinterpret_cast<float*>(scale)[rr[u] * ld_scale + cc[u] / GROUP] = sc;
      }
      if (rr[u] >= 0) store4(g.q + rr[u] * g.ld_q, cc[u], g.cols, g.q_vec, quant4<FP8>(v[u], inv));
    }
  }
}

// ----------------------------------------------------------------------------
// 128x128 tile scales: one CTA of 256 threads (8 warps x 16 rows) per tile,
// the tile held in registers between the amax and the quantize step.
template <typename T, int FP8>
__global__ void __launch_bounds__(256) quant_tile128_kernel(CastGeom g, float* scale, int64_t ld_scale,
                                                            int64_t tiles_c, int64_t ntiles) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const T* x = reinterpret_cast<const T*>(g.x);
  __shared__ float red[8];
  __shared__ float s_inv;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t tr = t / tiles_c, tc = t - tr * tiles_c;
    const int64_t c = tc * 128 + lane * 4;
    float4 v[16];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      int64_t r = tr * 128 + w * 16 + i;
      v[i] = r < g.rows ? load4<T>(x + r * g.ld_x, c, g.cols, g.x_vec) : make_float4(0.f, 0.f, 0.f, 0.f);
      m = fmaxf(m, absmax4(v[i]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[w] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      float a = red[0];
#pragma unroll
      for (int i = 1; i < 8; ++i) a = fmaxf(a, red[i]);
      float sc = __fdiv_rn(a, FM);
      s_inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
      scale[tr * ld_scale + tc] = sc;
    }
    __syncthreads();
    const float inv = s_inv;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      int64_t r = tr * 128 + w * 16 + i;
      if (r < g.rows) store4(g.q + r * g.ld_q, c, g.cols, g.q_vec, quant4<FP8>(v[i], inv));
    }
    __syncthreads();  // red / s_inv are reused by the next tile
  }
}

// ----------------------------------------------------------------------------
// Host-side launchers (called from b2x_api.cu after argument validation).

static int cast_grid(int64_t nsegs, int segs_per_warp, int num_sms) {
  int64_t warps_needed = (nsegs + segs_per_warp - 1) / segs_per_warp;
  int64_t blocks = (warps_needed + 7) / 8;
  int64_t cap = (int64_t)num_sms * 8;  // 8 CTAs of 256 threads per SM fill all 64 warp slots
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

int cast_num_partials(int64_t nsegs, int num_sms) { return cast_grid(nsegs, 4, num_sms); }

template <typename T, int FP8>
static cudaError_t launch_cast_t(const CastGeom& g, int mode, void* scale, int64_t ld_scale, uint32_t* partials,
                                 int num_sms, cudaStream_t st) {
  constexpr int SEGS = sizeof(T) == 4 ? 4 : 8;
  switch (mode) {
    case B2X_SCALE_NONE:
    case B2X_SCALE_TENSOR_GIVEN: {
      int grid = cast_grid(g.nsegs, SEGS, num_sms);
      quant_uniform_kernel<T, FP8, SEGS><<<grid, 256, 0, st>>>(g, mode, (float*)scale, nullptr, 0);
      note_launch(1);
      break;
    }
    case B2X_SCALE_TENSOR: {
      int np = cast_num_partials(g.nsegs, num_sms);
      amax_partial_kernel<T, 4><<<np, 256, 0, st>>>(g, partials);
      int grid = cast_grid(g.nsegs, SEGS, num_sms);
      quant_uniform_kernel<T, FP8, SEGS><<<grid, 256, 0, st>>>(g, mode, (float*)scale, partials, np);
      note_launch(2);
      break;
    }
    case B2X_SCALE_BLOCK_1x128: {
      int grid = cast_grid(g.nsegs, SEGS, num_sms);
      quant_rowblock_kernel<T, FP8, 128, SEGS><<<grid, 256, 0, st>>>(g, scale, ld_scale);
      note_launch(1);
      break;
    }
    case B2X_SCALE_MX_1x32: {
      int grid = cast_grid(g.nsegs, SEGS, num_sms);
      quant_rowblock_kernel<T, FP8, 32, SEGS><<<grid, 256, 0, st>>>(g, scale, ld_scale);
      note_launch(1);
      break;
    }
    case B2X_SCALE_BLOCK_128x128: {
      int64_t tiles_r = (g.rows + 127) / 128, tiles_c = (g.cols + 127) / 128;
      int64_t nt = tiles_r * tiles_c;
      int64_t grid = nt < (int64_t)num_sms * 8 ? nt : (int64_t)num_sms * 8;
      quant_tile128_kernel<T, FP8><<<(int)grid, 256, 0, st>>>(g, (float*)scale, ld_scale, tiles_c, nt);
      note_launch(1);
      break;
    }
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_cast(const b2x_cast_args& a, int num_sms, cudaStream_t st) {
  CastGeom g;
  g.x = a.x;
  g.rows = a.rows;
  g.cols = a.cols;
  g.ld_x = a.ld_x;
  g.q = reinterpret_cast<uint8_t*>(a.q);
  g.ld_q = a.ld_q;
  // A contiguous tensor is one long row: fewer divisions, same elements.
  if (a.ld_x == a.cols && a.ld_q == a.cols &&
      (a.mode == B2X_SCALE_NONE || a.mode == B2X_SCALE_TENSOR || a.mode == B2X_SCALE_TENSOR_GIVEN)) {
    g.cols = a.rows * a.cols;
    g.rows = 1;
  }
  g.segs_per_row = (g.cols + 127) / 128;
  g.nsegs = g.rows * g.segs_per_row;
  const int es = a.x_type == B2X_F32 ? 4 : 2;
  const int vb = es * 4;  // bytes per lane load
  g.x_vec = ((uintptr_t)a.x % vb == 0) && ((g.rows == 1) || ((g.ld_x * es) % vb == 0));
  g.q_vec = ((uintptr_t)a.q % 4 == 0) && ((g.rows == 1) || (g.ld_q % 4 == 0));
  uint32_t* partials = reinterpret_cast<uint32_t*>(a.workspace);
  const int fp8 = a.q_type == B2X_E4M3 ? 0 : 1;
  if (a.x_type == B2X_F32)
    return fp8 == 0 ? launch_cast_t<float, 0>(g, a.mode, a.scale, a.ld_scale, partials, num_sms, st)
                    : launch_cast_t<float, 1>(g, a.mode, a.scale, a.ld_scale, partials, num_sms, st);
  return fp8 == 0 ? launch_cast_t<uint16_t, 0>(g, a.mode, a.scale, a.ld_scale, partials, num_sms, st)
                  : launch_cast_t<uint16_t, 1>(g, a.mode, a.scale, a.ld_scale, partials, num_sms, st);
}

cudaError_t launch_amax(const void* x, b2x_dtype xt, int64_t rows, int64_t cols, int64_t ld_x, float* out,
                        uint32_t* partials, int num_sms, cudaStream_t st) {
  CastGeom g{};
  g.x = x;
  g.rows = rows;
  g.cols = cols;
  g.ld_x = ld_x;
  if (ld_x == cols) {
    g.cols = rows * cols;
    g.rows = 1;
  }
  g.segs_per_row = (g.cols + 127) / 128;
  g.nsegs = g.rows * g.segs_per_row;
  const int es = xt == B2X_F32 ? 4 : 2;
  g.x_vec = ((uintptr_t)x % (es * 4) == 0) && ((g.rows == 1) || ((g.ld_x * es) % (es * 4) == 0));
  int np = cast_num_partials(g.nsegs, num_sms);
  if (xt == B2X_F32)
    amax_partial_kernel<float, 4><<<np, 256, 0, st>>>(g, partials);
  else
    amax_partial_kernel<uint16_t, 4><<<np, 256, 0, st>>>(g, partials);
  amax_final_kernel<<<1, 256, 0, st>>>(partials, np, out);
  note_launch(2);
  return cudaGetLastError();
}

}  // namespace b2x
