// Fused SwiGLU + fp8 re-quantize epilogue for the paired gate+up GEMM.
//
// The gate+up projection of a Llama MLP computes [gate | up] = X . W_gu^T and
// the down projection consumes h = silu(gate) * up, quantized to fp8.  With
// W_gu's rows interleaved in blocks of 128 (gate rows 128j..128j+127, then
// up rows 128j..128j+127, for j = 0, 1, ...), every 256-wide paired tile
// holds matching gate and up columns, so one CTA's 128 x 256 accumulator
// yields 128 x 128 values of h, and the epilogue writes h as fp8 directly:
//
//   g, u  = alpha * acc[:, 0:128], alpha * acc[:, 128:256]   (alpha = sA * sB)
//   h     = g / (1 + exp(-g)) * u      (fp32, fast exp and division)
//   block 1x128 scales:  s = amax_row(|h|) / FMAX, inv = s == 0 ? 0 : 1 / s
//   MX 1x32 scales:      per 32 columns, d = amax / FMAX rounded up to a power
//                        of two (RCEIL), E8M0 byte = exponent of d, inv = 1 / d
//                        (the reference's _to_mxfp8_block, mxfp8_utils.py:89-128)
//   given scale s:       inv = 1 / s, and amax |h| is max-reduced into *amax
//   q     = fp8_rne_satfinite(copysign(min(|h * inv|, FMAX), h * inv))
//
// (the cast recipe of the per-tensor / 1x128 quantize, applied in registers).
// The tile is read from TMEM twice -- once for the row amax, once to quantize
// -- so no 128-value row of h is held in registers.  No reference component
// does this; it composes the GEMM epilogue (blackwell_gemm_ws.py:673-824)
// with the quantize recipe (mxfp8_utils.py:37-84).
#pragma once
#include <cstdint>
#include "b2x_ptx.cuh"
#include "fp8_gemm_common.cuh"

namespace b2x {

__device__ __forceinline__ float swiglu_clamp(float y, float m) {
  float r;
  asm("min.xorsign.abs.f32 %0, %1, %2;" : "=f"(r) : "f"(y), "f"(m));
  return r;
}

__device__ __forceinline__ float swiglu_h(uint32_t g_bits, uint32_t u_bits, float alpha) {
  const float g = __fmul_rn(__uint_as_float(g_bits), alpha);
  const float u = __fmul_rn(__uint_as_float(u_bits), alpha);
  return __fmul_rn(__fdividef(g, 1.0f + __expf(-g)), u);
}

// One epilogue warpgroup on one 128 x 256 accumulator (t_row: this thread's
// TMEM row at column 0).  `release` hands the accumulator back to the MMA
// warp once it has been read for the last time.
template <typename Release>
__device__ __forceinline__ void swiglu_quant_tile(const GemmParams& p, const CUtensorMap* tmQ, uint32_t t_row, int m0,
                                                  int pid_n, float alpha, uint8_t* stage, uint32_t bar_id, int wg_tid,
                                                  int row, Release release) {
  const float fmax = p.sw_fmt ? 57344.0f : 448.0f;
  // pass 1: row amax of h (and, for MX, the amax of each 32-column group)
  float amax = 0.0f;
  float gmax[4];
#pragma unroll 1
  for (int c = 0; c < 128; c += 32) {
    uint32_t g[32], u[32];
    tmem_ld_32x32b_x32(t_row + c, g);
    tmem_ld_32x32b_x32(t_row + 128 + c, u);
    tmem_ld_wait();
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(swiglu_h(g[i], u[i], alpha)));
    gmax[c >> 5] = m;
    amax = fmaxf(amax, m);
  }
  float inv = 0.0f;
  float ginv[4] = {0.f, 0.f, 0.f, 0.f};
  if (p.sw_mode == 2) {
    uint32_t bytes = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float descale = __fdiv_rn(gmax[j], fmax);
      const uint32_t e = (__float_as_uint(descale) + 0x007FFFFFu) & 0x7F800000u;
      const float rounded = __uint_as_float(e);
      ginv[j] = rounded == 0.0f ? 0.0f : __fdiv_rn(1.0f, rounded);
      bytes |= (e >> 23) << (8 * j);
    }
    if (m0 + row < p.M)
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(p.sw_scale) + (int64_t)(m0 + row) * p.sw_ld_scale +
                                   pid_n * 4) = bytes;
  } else if (p.sw_mode == 0) {
    const float s = __fdiv_rn(amax, fmax);
    inv = s == 0.0f ? 0.0f : __fdiv_rn(1.0f, s);
    if (m0 + row < p.M) p.sw_scale[(int64_t)(m0 + row) * p.sw_ld_scale + pid_n] = s;
  } else {
    const float s = __ldg(p.sw_given);
    inv = s == 0.0f ? 0.0f : __fdiv_rn(1.0f, s);
    const unsigned m = __reduce_max_sync(0xffffffffu, m0 + row < p.M ? __float_as_uint(amax) : 0u);
    if ((threadIdx.x & 31) == 0 && p.sw_amax) atomicMax(reinterpret_cast<unsigned*>(p.sw_amax), m);
  }
  // the previous tile's store must have left the staging buffer
  if (wg_tid == 0) bulk_wait_group_read0();
  named_bar_sync(bar_id, 128);
  const uint32_t srow = smem_u32(stage + row * 128);
  // pass 2: quantize 32 columns at a time into the 128-byte staging row
#pragma unroll 1
  for (int c = 0; c < 128; c += 32) {
    uint32_t g[32], u[32];
    tmem_ld_32x32b_x32(t_row + c, g);
    tmem_ld_32x32b_x32(t_row + 128 + c, u);
    tmem_ld_wait();
    if (c == 96) release();
    const float cinv = p.sw_mode == 2 ? ginv[c >> 5] : inv;
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float y[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        y[k] = swiglu_clamp(__fmul_rn(swiglu_h(g[4 * j + k], u[4 * j + k], alpha), cinv), fmax);
      const uint16_t lo = p.sw_fmt ? cvt_e5m2x2(y[0], y[1]) : cvt_e4m3x2(y[0], y[1]);
      const uint16_t hi = p.sw_fmt ? cvt_e5m2x2(y[2], y[3]) : cvt_e4m3x2(y[2], y[3]);
      w[j] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    const int unit = c / 16;  // two 16-byte units per 32 columns
    st_shared_v4(srow + (((unit) ^ (row & 7)) << 4), w[0], w[1], w[2], w[3]);
    st_shared_v4(srow + (((unit + 1) ^ (row & 7)) << 4), w[4], w[5], w[6], w[7]);
  }
  fence_proxy_async_smem();
  named_bar_sync(bar_id, 128);
  if (wg_tid == 0 && m0 < p.M) {
    tma_store_2d(tmQ, stage, pid_n * 128, m0);
    bulk_commit_group();
  }
}

}  // namespace b2x
