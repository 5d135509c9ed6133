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
// Work decomposition: a "segment" is 256 consecutive columns of one row; one
// warp owns a segment at a time and each lane holds 8 consecutive elements
// (32 B of fp32 or 16 B of bf16 per lane, 8 B of fp8 out), so every access
// is a full 16-byte vector and a warp moves fully coalesced 1 KB / 512 B in
// and 256 B out.  Segments are unrolled per warp and the grid is sized from
// the occupancy calculator so all CTAs are resident at once (one wave) with
// enough bytes in flight for HBM3e.
#include <cuda_bf16.h>
#include <algorithm>
#include <cstring>
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
// One instruction: min.xorsign.abs gives min(|y|, |m|) with the sign bit of
// y XOR m (m > 0, so y's), and like min it returns the non-NaN operand.
__device__ __forceinline__ float clamp_sym(float y, float m) {
  float r;
  asm("min.xorsign.abs.f32 %0, %1, %2;" : "=f"(r) : "f"(y), "f"(m));
  return r;
}
// max(|a|, |b|) up to sign (the sign bit is a XOR b; callers take |result|
// once at the end); NaN operands are ignored like fmaxf.
__device__ __forceinline__ float absmax_xs(float a, float b) {
  float r;
  asm("max.xorsign.abs.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Quantize values.  SCALED: multiply by inv first; the GPU's fp32 multiply
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

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

constexpr int kSeg = 256;  // columns per warp step
constexpr int kLaneElems = 8;

// Eight consecutive input elements as loaded: kept packed (2 x 16 B of fp32
// or 16 B of bf16) until they are converted, so deep unrolling costs few
// registers and many loads can be in flight per thread.
template <typename T>
struct Raw8;
template <>
struct Raw8<float> {
  float4 a, b;
};
template <>
struct Raw8<uint16_t> {
  uint4 a;
};

// Load 8 consecutive elements from column `col` of a row; elements at or
// beyond `cols` read as 0.  `vec_ok`: the row base is 16-byte aligned.
__device__ __forceinline__ void load_raw(const float* row, int64_t col, int64_t cols, bool vec_ok, Raw8<float>& r) {
  if (vec_ok && col + 7 < cols) {
    r.a = __ldcs(reinterpret_cast<const float4*>(row + col));
    r.b = __ldcs(reinterpret_cast<const float4*>(row + col + 4));
    return;
  }
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = (col + i < cols) ? row[col + i] : 0.f;
  r.a = make_float4(v[0], v[1], v[2], v[3]);
  r.b = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void load_raw(const uint16_t* row, int64_t col, int64_t cols, bool vec_ok,
                                         Raw8<uint16_t>& r) {
  if (vec_ok && col + 7 < cols) {
    r.a = __ldcs(reinterpret_cast<const uint4*>(row + col));
    return;
  }
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (col + i < cols) w[i >> 1] |= (uint32_t)row[col + i] << (16 * (i & 1));
  r.a = make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
__device__ __forceinline__ void zero_raw(Raw8<T>& r) {
  memset(&r, 0, sizeof(r));
}

__device__ __forceinline__ void unpack(const Raw8<float>& r, float (&v)[8]) {
  v[0] = r.a.x, v[1] = r.a.y, v[2] = r.a.z, v[3] = r.a.w, v[4] = r.b.x, v[5] = r.b.y, v[6] = r.b.z, v[7] = r.b.w;
}
__device__ __forceinline__ void unpack(const Raw8<uint16_t>& r, float (&v)[8]) {
  v[0] = bf16lo(r.a.x), v[1] = bf16hi(r.a.x), v[2] = bf16lo(r.a.y), v[3] = bf16hi(r.a.y);
  v[4] = bf16lo(r.a.z), v[5] = bf16hi(r.a.z), v[6] = bf16lo(r.a.w), v[7] = bf16hi(r.a.w);
}

template <typename T>
__device__ __forceinline__ void load8(const T* row, int64_t col, int64_t cols, bool vec_ok, float (&v)[8]) {
  Raw8<T> r;
  load_raw(row, col, cols, vec_ok, r);
  unpack(r, v);
}

__device__ __forceinline__ void store8(uint8_t* row, int64_t col, int64_t cols, bool vec_ok, uint2 q) {
  if (vec_ok && col + 7 < cols) {
    __stcs(reinterpret_cast<uint2*>(row + col), q);
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (col + i < cols) row[col + i] = (uint8_t)((i < 4 ? q.x : q.y) >> (8 * (i & 3)));
}

template <int FP8, bool SCALED = true>
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float inv) {
  uint2 r;
  r.x = quant4<FP8, SCALED>(make_float4(v[0], v[1], v[2], v[3]), inv);
  r.y = quant4<FP8, SCALED>(make_float4(v[4], v[5], v[6], v[7]), inv);
  return r;
}

__device__ __forceinline__ float absmax8(const float (&v)[8]) {
  // pairwise tree of NaN-ignoring |max|; the sign bits are dropped at the end
  float a = absmax_xs(v[0], v[1]), b = absmax_xs(v[2], v[3]);
  float c = absmax_xs(v[4], v[5]), d = absmax_xs(v[6], v[7]);
  // fmaxf(0, .) turns the all-NaN case into 0, as a NaN-ignoring max from 0 would
  return fmaxf(0.f, fabsf(absmax_xs(absmax_xs(a, b), absmax_xs(c, d))));
}

struct CastGeom {
  const void* x;
  int64_t rows, cols, ld_x;
  uint8_t* q;
  int64_t ld_q;
  int64_t segs_per_row;  // ceil(cols / 256)
  int64_t nsegs;         // rows * segs_per_row
  bool x_vec, q_vec;     // 16-byte loads / 8-byte stores legal
};

// Row and first column of this lane in segment s.
__device__ __forceinline__ void seg_pos(const CastGeom& g, int64_t s, int lane, int64_t& r, int64_t& c) {
  r = g.segs_per_row == 1 ? s : s / g.segs_per_row;
  c = (s - r * g.segs_per_row) * kSeg + lane * kLaneElems;
}

// ----------------------------------------------------------------------------
// Per-tensor amax, pass 1: each CTA writes the NaN-ignoring max |x| of its
// share into partials[blockIdx.x] (as fp32 bits).
template <typename T, int U>
__global__ void __launch_bounds__(256) amax_partial_kernel(CastGeom g, uint32_t* partials) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(g.x);
  float m = 0.f;
  for (int64_t s0 = warp * U; s0 < g.nsegs; s0 += nwarps * U) {
    Raw8<T> raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int64_t r, c;
      seg_pos(g, s0 + u, lane, r, c);
      if (s0 + u < g.nsegs)
        load_raw(x + r * g.ld_x, c, g.cols, g.x_vec, raw[u]);
      else
        zero_raw(raw[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float v[8];
      unpack(raw[u], v);
      m = fmaxf(m, absmax8(v));
    }
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
// Uniform-scale quantize: modes NONE (no multiply), TENSOR_GIVEN (inv from
// scale[0]) and TENSOR (inv from the amax partials; CTA 0 writes scale[0]).
template <typename T, int FP8, int U>
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
  const bool scaled = mode != B2X_SCALE_NONE;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(g.x);
  for (int64_t s0 = warp * U; s0 < g.nsegs; s0 += nwarps * U) {
    Raw8<T> raw[U];
    int64_t rr[U], cc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      seg_pos(g, s0 + u, lane, rr[u], cc[u]);
      if (s0 + u < g.nsegs) load_raw(x + rr[u] * g.ld_x, cc[u], g.cols, g.x_vec, raw[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (s0 + u >= g.nsegs) continue;
      float v[8];
      unpack(raw[u], v);
      uint2 q = scaled ? quant8<FP8>(v, inv) : quant8<FP8, false>(v, inv);
      store8(g.q + rr[u] * g.ld_q, cc[u], g.cols, g.q_vec, q);
    }
  }
}

// ----------------------------------------------------------------------------
// Row-block scales: GROUP = 128 (fp32 scale per 1x128) or 32 (E8M0 per 1x32).
// A warp covers one 256-column segment: 256/GROUP groups of GROUP/8 lanes.
template <typename T, int FP8, int GROUP, int U>
__global__ void __launch_bounds__(256) quant_rowblock_kernel(CastGeom g, void* scale, int64_t ld_scale) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  constexpr int LPG = GROUP / kLaneElems;  // lanes per group
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(g.x);
  for (int64_t s0 = warp * U; s0 < g.nsegs; s0 += nwarps * U) {
    Raw8<T> raw[U];
    int64_t rr[U], cc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      seg_pos(g, s0 + u, lane, rr[u], cc[u]);
      if (s0 + u < g.nsegs)
        load_raw(x + rr[u] * g.ld_x, cc[u], g.cols, g.x_vec, raw[u]);
      else
        zero_raw(raw[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      // Lanes past the end of the row (or of the tensor) take part in the
      // shuffles holding zeros but store nothing.
      const bool live = s0 + u < g.nsegs;
      float v[8];
      unpack(raw[u], v);
      float m = absmax8(v);
#pragma unroll
      for (int o = LPG / 2; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float inv;
      const bool leader = live && (lane % LPG) == 0 && cc[u] < g.cols;
      if constexpr (GROUP == 32) {
        float descale = __fdiv_rn(m, FM);
        uint32_t e = (__float_as_uint(descale) + 0x007FFFFFu) & 0x7F800000u;
        float rounded = __uint_as_float(e);
        inv = rounded == 0.f ? 0.f : __fdiv_rn(1.0f, rounded);
        if (leader) reinterpret_cast<uint8_t*>(scale)[rr[u] * ld_scale + cc[u] / GROUP] = (uint8_t)(e >> 23);
      } else {
        float sc = __fdiv_rn(m, FM);
        inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
        if (leader) reinterpret_cast<float*>(scale)[rr[u] * ld_scale + cc[u] / GROUP] = sc;
      }
      if (live) store8(g.q + rr[u] * g.ld_q, cc[u], g.cols, g.q_vec, quant8<FP8>(v, inv));
    }
  }
}

// ----------------------------------------------------------------------------
// 128x128 tile scales: one CTA of 256 threads per tile.  A warp covers two
// rows per step (lanes 0-15 one row, 16-31 the next), 16 rows in 8 steps, and
// keeps them in registers between the amax and the quantize step.
template <typename T, int FP8>
__global__ void __launch_bounds__(256) quant_tile128_kernel(CastGeom g, float* scale, int64_t ld_scale,
                                                            int64_t tiles_c, int64_t ntiles) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int half = lane >> 4;
  const T* x = reinterpret_cast<const T*>(g.x);
  __shared__ float red[8];
  __shared__ float s_inv;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t tr = t / tiles_c, tc = t - tr * tiles_c;
    const int64_t c = tc * 128 + (lane & 15) * kLaneElems;
    float v[8][8];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t r = tr * 128 + w * 16 + 2 * i + half;
      if (r < g.rows && c < tc * 128 + 128)
        load8<T>(x + r * g.ld_x, c, g.cols, g.x_vec, v[i]);
      else
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      m = fmaxf(m, absmax8(v[i]));
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
    for (int i = 0; i < 8; ++i) {
      const int64_t r = tr * 128 + w * 16 + 2 * i + half;
      if (r < g.rows) store8(g.q + r * g.ld_q, c, g.cols, g.q_vec, quant8<FP8>(v[i], inv));
    }
    __syncthreads();  // red / s_inv are reused by the next tile
  }
}

// ----------------------------------------------------------------------------
// Staged streaming kernels for contiguous tensors (the common case): a
// producer warp streams 16 KB chunks of x into a ring of shared-memory stages
// with 1-D bulk copies (cp.async.bulk, completion counted on an mbarrier), so
// many KB per SM are in flight without holding registers, and 8 consumer
// warps convert each chunk from shared memory and write q with coalesced
// stores.  Chunk c of the tensor goes to CTA c % grid, in order.
//
// STAGED_MODE: 0 = cast only (NONE), 1 = one scale for the tensor (TENSOR /
// TENSOR_GIVEN), 2 = 1x128 row-block scales (rows a multiple of 128 long, so
// every 128 consecutive elements of the flat tensor are one group), 3 = amax
// pass of TENSOR (per-CTA NaN-ignoring max |x| into partials).
constexpr int kStChunk = 16384;  // bytes of x per stage
constexpr int kStStages = 4;
constexpr int kStConsumers = 256;
constexpr int kStThreads = kStConsumers + 32;
constexpr int kStSmem = kStStages * kStChunk + 2 * kStStages * 8 + 16 + 128;

struct StagedArgs {
  const uint8_t* x;     // 16-byte aligned
  uint8_t* q;           // 16-byte aligned (unused in mode 3)
  int64_t n;            // elements; n * sizeof(T) % 16 == 0
  int64_t nchunks;
  int64_t groups_per_row;  // mode 2: cols / 128
  void* scale;          // mode 2: fp32 [rows, ld_scale]; mode 1: scale[0]
  int64_t ld_scale;
  int tensor_mode;      // mode 1: B2X_SCALE_TENSOR (inv from partials) or B2X_SCALE_TENSOR_GIVEN
  uint32_t* partials;   // mode 1 (TENSOR) input, mode 3 output
  int npartials;
};

template <typename T>
__device__ __forceinline__ void staged_unpack(uint4 raw, float* e) {
  if constexpr (sizeof(T) == 4) {
    e[0] = __uint_as_float(raw.x), e[1] = __uint_as_float(raw.y);
    e[2] = __uint_as_float(raw.z), e[3] = __uint_as_float(raw.w);
  } else {
    e[0] = bf16lo(raw.x), e[1] = bf16hi(raw.x), e[2] = bf16lo(raw.y), e[3] = bf16hi(raw.y);
    e[4] = bf16lo(raw.z), e[5] = bf16hi(raw.z), e[6] = bf16lo(raw.w), e[7] = bf16hi(raw.w);
  }
}

template <int FP8, int MODE, int VE>
__device__ __forceinline__ void staged_store(uint8_t* qp, const float* e, float inv) {
  if constexpr (VE == 4) {
    const uint32_t w = MODE == 0 ? quant4<FP8, false>(make_float4(e[0], e[1], e[2], e[3]), 1.f)
                                 : quant4<FP8>(make_float4(e[0], e[1], e[2], e[3]), inv);
    __stcs(reinterpret_cast<unsigned int*>(qp), w);
  } else {
    const float(&e8)[8] = *reinterpret_cast<const float(*)[8]>(e);
    const uint2 w = MODE == 0 ? quant8<FP8, false>(e8, 1.f) : quant8<FP8>(e8, inv);
    __stcs(reinterpret_cast<uint2*>(qp), w);
  }
}

template <typename T, int FP8, int MODE, bool FULL>
__device__ __forceinline__ void staged_quant(const StagedArgs& a, const float (&e)[kStChunk / 16 / kStConsumers][16 / sizeof(T)],
                                             int64_t off, int nvec, float inv, int lane);

// One consumer warp's share of a staged chunk: vectors j * 256 + tid for
// j < VPT (a warp reads 32 consecutive 16-byte vectors per j).  FULL: the
// chunk holds kStChunk bytes (no bounds checks).
template <typename T, int FP8, int MODE, bool FULL>
__device__ __forceinline__ void staged_chunk(const StagedArgs& a, const uint8_t* buf, int64_t off, int nvec, float inv,
                                             float& m, int lane) {
  constexpr int VE = 16 / sizeof(T);
  constexpr int VPT = kStChunk / 16 / kStConsumers;
  float e[VPT][VE];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = j * kStConsumers + threadIdx.x;
    if (FULL || v < nvec) {
      staged_unpack<T>(*reinterpret_cast<const uint4*>(buf + v * 16), e[j]);
    } else {
#pragma unroll
      for (int i = 0; i < VE; ++i) e[j][i] = 0.f;
    }
  }
  if constexpr (MODE == 3) {
#pragma unroll
    for (int j = 0; j < VPT; ++j)
#pragma unroll
      for (int i = 0; i < VE; i += 2) m = fmaxf(m, fmaxf(0.f, fabsf(absmax_xs(e[j][i], e[j][i + 1]))));
  } else {
    staged_quant<T, FP8, MODE, FULL>(a, e, off, nvec, inv, lane);
  }
}

template <typename T, int FP8, int MODE, bool FULL>
__device__ __forceinline__ void staged_quant(const StagedArgs& a, const float (&e)[kStChunk / 16 / kStConsumers][16 / sizeof(T)],
                                             int64_t off, int nvec, float inv, int lane) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  constexpr int VE = 16 / sizeof(T);
  constexpr int VPT = kStChunk / 16 / kStConsumers;
  float vinv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) vinv[j] = inv;
  if constexpr (MODE == 2) {
    // A 128-element group is LPG consecutive vectors, so a warp covers GPJ
    // groups per j.  The group maxima are reduced within each group's lanes,
    // gathered one group per lane (group j * GPJ + h on lane j * GPJ + h), the
    // two IEEE divisions run once for all of the warp's groups, and the
    // inverses go back to the groups' lanes.
    constexpr int LPG = 128 / VE;
    constexpr int GPJ = 32 / LPG;
    float mine = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      float gm = 0.f;
#pragma unroll
      for (int i = 0; i < VE; i += 2) gm = fmaxf(gm, fabsf(absmax_xs(e[j][i], e[j][i + 1])));
#pragma unroll
      for (int o = LPG / 2; o; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
      const float got = __shfl_sync(0xffffffffu, gm, (lane % GPJ) * LPG);
      if (lane / GPJ == j) mine = got;
    }
    const float sc = __fdiv_rn(mine, FM);
    const float minv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
    const int warp_in_cta = threadIdx.x >> 5;
    if (lane < VPT * GPJ) {
      // group of (j, h) = lane: its first vector is j * 256 + warp * 32 + h * LPG
      const int jj = lane / GPJ, h = lane % GPJ;
      const int v0 = jj * kStConsumers + warp_in_cta * 32 + h * LPG;
      if (FULL || v0 < nvec) {
        const int64_t grp = (off / (int64_t)sizeof(T) + (int64_t)v0 * VE) >> 7;
        int64_t idx = grp;  // contiguous scales: the group index is the scale index
        if (a.ld_scale != a.groups_per_row) {
          const int64_t row = grp / a.groups_per_row;
          idx = row * a.ld_scale + (grp - row * a.groups_per_row);
        }
        reinterpret_cast<float*>(a.scale)[idx] = sc;
      }
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) vinv[j] = __shfl_sync(0xffffffffu, minv, j * GPJ + lane / LPG);
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = j * kStConsumers + threadIdx.x;
    if (FULL || v < nvec) staged_store<FP8, MODE, VE>(a.q + off / (int64_t)sizeof(T) + (int64_t)v * VE, e[j], vinv[j]);
  }
}

template <typename T, int FP8, int MODE>
__global__ void __launch_bounds__(kStThreads, 1) cast_staged_kernel(const StagedArgs a) {
  constexpr float FM = Fp8Traits<FP8>::kMax;
  constexpr int VPC = kStChunk / 16;                 // vectors per chunk
  extern __shared__ uint8_t st_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(st_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStStages * kStChunk);
  uint64_t* empty = full + kStStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStStages);
  __shared__ float s_inv;
  __shared__ float s_red[kStThreads / 32];

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStConsumers / 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if constexpr (MODE == 1) {
    if (a.tensor_mode == B2X_SCALE_TENSOR) {
      const float amax = reduce_partials(a.partials, a.npartials);
      if (threadIdx.x == 0) {
        const float sc = __fdiv_rn(amax, FM);
        s_inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
        if (blockIdx.x == 0) *reinterpret_cast<float*>(a.scale) = sc;
      }
    } else if (threadIdx.x == 0) {
      const float sc = *reinterpret_cast<const float*>(a.scale);
      s_inv = sc == 0.f ? 0.f : __fdiv_rn(1.0f, sc);
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bytes_total = a.n * (int64_t)sizeof(T);

  if (warp == kStConsumers / 32) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t c = blockIdx.x; c < a.nchunks; c += gridDim.x) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, kStatusTimeoutCast)) break;
        const int64_t off = c * kStChunk;
        const uint32_t bytes = (uint32_t)min((int64_t)kStChunk, bytes_total - off);
        mbar_arrive_expect_tx(&full[stage], bytes);
        bulk_load_1d(smem + stage * kStChunk, a.x + off, bytes, &full[stage], pol);
        if (++stage == kStStages) stage = 0, phase ^= 1;
      }
    }
    return;  // nothing below waits for the producer warp
  }

  // -------------------------------------------------------------- consumers
  float inv = 1.0f;
  if constexpr (MODE == 1) inv = s_inv;
  float m = 0.f;  // mode 3
  int stage = 0;
  uint32_t phase = 0;
  for (int64_t c = blockIdx.x; c < a.nchunks; c += gridDim.x) {
    if (!mbar_wait(&full[stage], phase, abort_flag, kStatusTimeoutCast)) break;
    const int64_t off = c * kStChunk;
    const int nvec = (int)(min((int64_t)kStChunk, bytes_total - off) / 16);
    const uint8_t* buf = smem + stage * kStChunk;
    if (nvec == VPC)
      staged_chunk<T, FP8, MODE, true>(a, buf, off, nvec, inv, m, lane);
    else
      staged_chunk<T, FP8, MODE, false>(a, buf, off, nvec, inv, m, lane);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == kStStages) stage = 0, phase ^= 1;
  }
  if constexpr (MODE == 3) {
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_red[warp] = m;
    named_bar_sync(1, kStConsumers);
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int i = 0; i < kStConsumers / 32; ++i) t = fmaxf(t, s_red[i]);
      a.partials[blockIdx.x] = __float_as_uint(t);
    }
  }
}

// Staged path eligibility: contiguous flat tensor, 16-byte aligned x and q,
// whole 16-byte vectors; 1x128 also needs rows that are a multiple of 128.
static bool staged_ok(const b2x_cast_args& a) {
  const int es = a.x_type == B2X_F32 ? 4 : 2;
  if (a.ld_x != a.cols || a.ld_q != a.cols) return false;
  if (((uintptr_t)a.x % 16) || ((uintptr_t)a.q % 16)) return false;
  const int64_t n = a.rows * a.cols;
  if ((n * es) % 16 || n == 0) return false;
  if (a.mode == B2X_SCALE_BLOCK_1x128) return a.cols % 128 == 0;
  return a.mode == B2X_SCALE_NONE || a.mode == B2X_SCALE_TENSOR || a.mode == B2X_SCALE_TENSOR_GIVEN;
}

template <typename T, int FP8, int MODE>
static cudaError_t launch_staged_t(const StagedArgs& sa, int num_sms, cudaStream_t st, int* grid_out = nullptr) {
  auto k = cast_staged_kernel<T, FP8, MODE>;
  static int per_sm = 0;  // one cache per instantiation
  if (per_sm == 0) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(k), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kStSmem);
    if (e != cudaSuccess) return e;
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k, kStThreads, kStSmem) != cudaSuccess || v <= 0) v = 1;
    per_sm = v;
  }
  int64_t grid = (int64_t)num_sms * per_sm;
  if (grid > sa.nchunks) grid = sa.nchunks;
  if (grid < 1) grid = 1;
  if (grid_out) *grid_out = (int)grid;
  k<<<(int)grid, kStThreads, kStSmem, st>>>(sa);
  note_launch(1);
  return cudaGetLastError();
}

template <typename T, int FP8>
static cudaError_t launch_cast_staged(const b2x_cast_args& a, uint32_t* partials, int num_sms, cudaStream_t st) {
  StagedArgs sa{};
  sa.x = reinterpret_cast<const uint8_t*>(a.x);
  sa.q = reinterpret_cast<uint8_t*>(a.q);
  sa.n = a.rows * a.cols;
  sa.nchunks = (sa.n * (int64_t)sizeof(T) + kStChunk - 1) / kStChunk;
  sa.groups_per_row = a.cols / 128;
  sa.scale = a.scale;
  sa.ld_scale = a.ld_scale;
  sa.tensor_mode = a.mode;
  sa.partials = partials;
  switch (a.mode) {
    case B2X_SCALE_NONE: return launch_staged_t<T, FP8, 0>(sa, num_sms, st);
    case B2X_SCALE_TENSOR_GIVEN: return launch_staged_t<T, FP8, 1>(sa, num_sms, st);
    case B2X_SCALE_TENSOR: {
      int np = 0;
      cudaError_t e = launch_staged_t<T, FP8, 3>(sa, num_sms, st, &np);
      if (e != cudaSuccess) return e;
      sa.npartials = np;
      return launch_staged_t<T, FP8, 1>(sa, num_sms, st);
    }
    case B2X_SCALE_BLOCK_1x128: return launch_staged_t<T, FP8, 2>(sa, num_sms, st);
    default: return cudaErrorInvalidValue;
  }
}

// ----------------------------------------------------------------------------
// Host-side launchers (called from b2x_api.cu after argument validation).

// CTAs of 256 threads that fit on one SM at once (per kernel, cached).
template <typename K>
static int resident_ctas(K kern) {
  static int n = 0;  // one cache per kernel instantiation
  if (n == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, 256, 0) != cudaSuccess || v <= 0) v = 4;
    n = v;
  }
  return n;
}

static int grid_for(int64_t nsegs, int segs_per_warp, int per_sm, int num_sms) {
  int64_t warps_needed = (nsegs + segs_per_warp - 1) / segs_per_warp;
  int64_t blocks = (warps_needed + 7) / 8;
  int64_t cap = (int64_t)num_sms * per_sm;  // one full wave
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// Upper bound on the per-tensor amax partials (one per CTA of the amax pass,
// whichever kernel runs it: at most 8 resident CTAs per SM in either).
int cast_num_partials(int64_t nsegs, int num_sms) {
  (void)nsegs;
  return 8 * num_sms;
}

template <typename T, int FP8>
static cudaError_t launch_cast_t(const CastGeom& g, int mode, void* scale, int64_t ld_scale, uint32_t* partials,
                                 int num_sms, cudaStream_t st) {
  // 8-element segments per lane per step: 4 for fp32 (128 B in flight per
  // lane), 8 for bf16 (the same 128 B), so both keep as many bytes in flight.
  constexpr int U = sizeof(T) == 4 ? 4 : 8;
  switch (mode) {
    case B2X_SCALE_NONE:
    case B2X_SCALE_TENSOR_GIVEN:
    case B2X_SCALE_TENSOR: {
      int np = 0;
      if (mode == B2X_SCALE_TENSOR) {
        auto ak = amax_partial_kernel<T, U>;
        np = grid_for(g.nsegs, U, std::min(8, resident_ctas(ak)), num_sms);
        ak<<<np, 256, 0, st>>>(g, partials);
        note_launch(1);
      }
      auto k = quant_uniform_kernel<T, FP8, U>;
      int grid = grid_for(g.nsegs, U, resident_ctas(k), num_sms);
      k<<<grid, 256, 0, st>>>(g, mode, (float*)scale, partials, np);
      note_launch(1);
      break;
    }
    case B2X_SCALE_BLOCK_1x128: {
      // Row-block kernels do a shuffle reduction and two divisions per group:
      // a shallower unroll keeps more warps resident to hide that latency.
      constexpr int UR = 4;  // 8 for bf16 measured slower (2.1 vs 3.2 TB/s at 64M)
      auto k = quant_rowblock_kernel<T, FP8, 128, UR>;
      k<<<grid_for(g.nsegs, UR, resident_ctas(k), num_sms), 256, 0, st>>>(g, scale, ld_scale);
      note_launch(1);
      break;
    }
    case B2X_SCALE_MX_1x32: {
      constexpr int UR = 4;
      auto k = quant_rowblock_kernel<T, FP8, 32, UR>;
      k<<<grid_for(g.nsegs, UR, resident_ctas(k), num_sms), 256, 0, st>>>(g, scale, ld_scale);
      note_launch(1);
      break;
    }
    case B2X_SCALE_BLOCK_128x128: {
      auto k = quant_tile128_kernel<T, FP8>;
      int64_t tiles_r = (g.rows + 127) / 128, tiles_c = (g.cols + 127) / 128;
      int64_t nt = tiles_r * tiles_c;
      int64_t cap = (int64_t)num_sms * resident_ctas(k);
      k<<<(int)(nt < cap ? nt : cap), 256, 0, st>>>(g, (float*)scale, ld_scale, tiles_c, nt);
      note_launch(1);
      break;
    }
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

static CastGeom make_geom(const void* x, b2x_dtype xt, int64_t rows, int64_t cols, int64_t ld_x, void* q,
                          int64_t ld_q, bool flatten) {
  CastGeom g{};
  g.x = x;
  g.rows = rows;
  g.cols = cols;
  g.ld_x = ld_x;
  g.q = reinterpret_cast<uint8_t*>(q);
  g.ld_q = ld_q;
  // A contiguous tensor is one long row: fewer divisions, same elements.
  if (flatten && ld_x == cols && (q == nullptr || ld_q == cols)) {
    g.cols = rows * cols;
    g.rows = 1;
  }
  g.segs_per_row = (g.cols + kSeg - 1) / kSeg;
  g.nsegs = g.rows * g.segs_per_row;
  const int es = xt == B2X_F32 ? 4 : 2;
  g.x_vec = ((uintptr_t)x % 16 == 0) && ((g.rows == 1) || ((g.ld_x * es) % 16 == 0));
  g.q_vec = ((uintptr_t)q % 8 == 0) && ((g.rows == 1) || (g.ld_q % 8 == 0));
  return g;
}

cudaError_t launch_cast(const b2x_cast_args& a, int num_sms, cudaStream_t st) {
  if (staged_ok(a)) {
    uint32_t* partials = reinterpret_cast<uint32_t*>(a.workspace);
    const int fp8 = a.q_type == B2X_E4M3 ? 0 : 1;
    if (a.x_type == B2X_F32)
      return fp8 == 0 ? launch_cast_staged<float, 0>(a, partials, num_sms, st)
                      : launch_cast_staged<float, 1>(a, partials, num_sms, st);
    return fp8 == 0 ? launch_cast_staged<uint16_t, 0>(a, partials, num_sms, st)
                    : launch_cast_staged<uint16_t, 1>(a, partials, num_sms, st);
  }
  const bool uniform = a.mode == B2X_SCALE_NONE || a.mode == B2X_SCALE_TENSOR || a.mode == B2X_SCALE_TENSOR_GIVEN;
  CastGeom g = make_geom(a.x, a.x_type, a.rows, a.cols, a.ld_x, a.q, a.ld_q, uniform);
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
  CastGeom g = make_geom(x, xt, rows, cols, ld_x, nullptr, 0, true);
  int np;
  if (xt == B2X_F32) {
    auto k = amax_partial_kernel<float, 4>;
    np = grid_for(g.nsegs, 4, std::min(8, resident_ctas(k)), num_sms);
    k<<<np, 256, 0, st>>>(g, partials);
  } else {
    auto k = amax_partial_kernel<uint16_t, 4>;
    np = grid_for(g.nsegs, 4, std::min(8, resident_ctas(k)), num_sms);
    k<<<np, 256, 0, st>>>(g, partials);
  }
  amax_final_kernel<<<1, 256, 0, st>>>(partials, np, out);
  note_launch(2);
  return cudaGetLastError();
}

}  // namespace b2x
