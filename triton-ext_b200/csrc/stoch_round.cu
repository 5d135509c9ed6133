// Stochastic rounding fp32 -> e4m3 / e5m2 / fp16 / bf16 with caller-given
// random bits: the counterpart of the reference's tlx.stoch_round(src, dst_ty,
// rand_bits) (extensions/utlx/tlx/language/tlx/utility.py:113-153), which
// takes one uint32 of entropy per element.
//
// Rounding rule (stochastic rounding in its standard form, with 32 bits of
// resolution): let q * 2^u be |x| truncated to the target's precision at
// |x|'s binade (u = the target's quantum there, subnormal range included) and
// let frac32 be the first 32 bits of the truncated remainder, as a fraction
// of 2^u.  The magnitude rounds up to (q + 1) * 2^u exactly when
// frac32 + r >= 2^32 for the element's random word r, i.e. with probability
// frac32 / 2^32; the sign is kept.  The result is then encoded saturating
// (satfinite): beyond the largest finite value (Inf included) it becomes
// +-max; NaN stays NaN.  Values already representable never change.
//
// Why not `cvt.rs.satfinite`: that instruction takes one 32-bit word of
// entropy per 2 (16-bit targets) or 4 (fp8 targets) results, split into
// per-lane fields (8 bits per fp8 lane), so per-element words would have to be
// folded into it, and the reference's folding lives in Triton's lowering, not
// in the reference.  The reference's test (test_tlx.py:5126-5213) pins only
// properties -- exact values unchanged, no NaN/Inf from finite inputs, results
// next to the input -- which this rule keeps with every element's full word.
//
// Second mode, RS (b2x_stoch_round_rs): the hardware instruction the
// reference's lowering emits, `cvt.rs.satfinite.{e4m3x4,e5m2x4,f16x2,bf16x2}.f32`
// (the reference test asserts it in the PTX, test_tlx.py:5182).  It rounds a
// pack of 4 (fp8) or 2 (16-bit) values with ONE 32-bit entropy word whose
// fields feed the lanes.  Packs are consecutive columns of a row starting at
// column 0, and a pack takes the word of its first element (the other words
// of the pack are not read).  The rounding itself is the instruction's.
//
// The kernel is HBM-bound: 4 + 4 bytes in and 1 (fp8) or 2 bytes out per
// element; a thread handles 8 consecutive elements per step (two 16-byte
// loads of x and of r).
#include <cuda_runtime.h>
#include <cstdint>
#include "b2x_internal.h"

namespace b2x {

struct SrFormat {
  int p;     // stored mantissa bits
  int emin;  // exponent of the smallest normal
};

__device__ __forceinline__ SrFormat sr_format(int t) {
  switch (t) {
    case B2X_E4M3: return {3, -6};
    case B2X_E5M2: return {2, -14};
    case B2X_F16: return {10, -14};
    default: return {7, -126};  // B2X_BF16
  }
}

// |x| (finite, as fp32 bits without sign) stochastically truncated to the
// target precision; returns the exact result as fp32 bits (it may exceed the
// target's range: the encoder saturates).
__device__ __forceinline__ uint32_t sr_magnitude(uint32_t abits, uint32_t r, SrFormat f) {
  const int E = (int)(abits >> 23);
  const uint32_t F = abits & 0x7FFFFFu;
  if (abits == 0) return 0;
  uint32_t M;
  int e2;     // |x| = M * 2^e2
  int eb;     // floor(log2 |x|)
  if (E == 0) {
    M = F;
    e2 = -149;
    eb = -149 + 31 - __clz(F);
  } else {
    M = F | 0x800000u;
    e2 = E - 150;
    eb = E - 127;
  }
  const int u = max(eb, f.emin) - f.p;  // quantum of the target at |x|
  const int s = u - e2;                 // bits of M below the quantum
  if (s <= 0) return abits;             // already representable (range aside)
  uint64_t q;
  uint32_t frac32;
  if (s >= 56) {  // |x| < 2^-31 of the quantum: no 32-bit remainder is left
    q = 0;
    frac32 = 0;
  } else {
    q = (uint64_t)M >> s;
    const uint64_t rem = (uint64_t)M & ((1ull << s) - 1);
    frac32 = s <= 32 ? (uint32_t)(rem << (32 - s)) : (uint32_t)(rem >> (s - 32));
  }
  q += ((uint64_t)frac32 + r) >> 32;  // carry out of the 32-bit add: round up
  if (q == 0) return 0;
  // exact value q * 2^u in fp32 (q < 2^25, 2^u >= 2^-133 for all targets)
  const float pw = u >= -126 ? __uint_as_float((uint32_t)(u + 127) << 23) : __uint_as_float(1u << (u + 149));
  return __float_as_uint((float)q * pw);
}

// Hardware stochastic rounding of a pack: x[0] lands in the lowest byte /
// half of the result (the instruction puts its first operand in the highest).
template <int T>
__device__ __forceinline__ uint32_t cvt_rs_pack(const float* x, uint32_t r) {
  uint32_t o;
  if constexpr (T == B2X_E4M3)
    asm("cvt.rs.satfinite.e4m3x4.f32 %0, {%1, %2, %3, %4}, %5;"
        : "=r"(o) : "f"(x[3]), "f"(x[2]), "f"(x[1]), "f"(x[0]), "r"(r));
  else if constexpr (T == B2X_E5M2)
    asm("cvt.rs.satfinite.e5m2x4.f32 %0, {%1, %2, %3, %4}, %5;"
        : "=r"(o) : "f"(x[3]), "f"(x[2]), "f"(x[1]), "f"(x[0]), "r"(r));
  else if constexpr (T == B2X_BF16)
    asm("cvt.rs.satfinite.bf16x2.f32 %0, %1, %2, %3;" : "=r"(o) : "f"(x[1]), "f"(x[0]), "r"(r));
  else
    asm("cvt.rs.satfinite.f16x2.f32 %0, %1, %2, %3;" : "=r"(o) : "f"(x[1]), "f"(x[0]), "r"(r));
  return o;
}

template <int T>
constexpr int rs_pack() {
  return (T == B2X_E4M3 || T == B2X_E5M2) ? 4 : 2;
}

// Eight consecutive elements starting at a pack boundary (RS mode).
template <int T>
__device__ __forceinline__ void rs8(const float (&x)[8], const uint32_t (&r)[8], void* dst) {
  constexpr int P = rs_pack<T>();
  uint32_t w[8 / P];
#pragma unroll
  for (int k = 0; k < 8 / P; ++k) w[k] = cvt_rs_pack<T>(x + k * P, r[k * P]);
  if constexpr (P == 4)
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  else
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

// One element of column c (RS mode): it is placed in its lane of the pack,
// the other lanes hold zero, and the pack's word is its first element's.
template <int T>
__device__ __forceinline__ void rs1(float x, const uint32_t* r_row, int64_t c, uint8_t* dst) {
  constexpr int P = rs_pack<T>();
  const int lane = (int)(c % P);
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  v[lane] = x;
  const uint32_t o = cvt_rs_pack<T>(v, r_row[c - lane]);
  if constexpr (P == 4)
    *dst = (uint8_t)(o >> (8 * lane));
  else
    *reinterpret_cast<uint16_t*>(dst) = (uint16_t)(o >> (16 * lane));
}

// Round each element, then encode.  The product of a small integer and a
// power of two is exact, so the final converts only saturate.
template <int T>
__device__ __forceinline__ void sr8(const float (&x)[8], const uint32_t (&r)[8], void* dst) {
  const SrFormat f = sr_format(T);
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t b = __float_as_uint(x[i]);
    const uint32_t a = b & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) {
      y[i] = x[i];  // Inf saturates and NaN stays NaN in the encoder
    } else {
      y[i] = __uint_as_float(sr_magnitude(a, r[i], f) | (b & 0x80000000u));
    }
  }
  if constexpr (T == B2X_E4M3 || T == B2X_E5M2) {
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint16_t lo = T == B2X_E4M3 ? cvt_e4m3x2(y[4 * h], y[4 * h + 1]) : cvt_e5m2x2(y[4 * h], y[4 * h + 1]);
      const uint16_t hi = T == B2X_E4M3 ? cvt_e4m3x2(y[4 * h + 2], y[4 * h + 3]) : cvt_e5m2x2(y[4 * h + 2], y[4 * h + 3]);
      w[h] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      if constexpr (T == B2X_BF16)
        asm("cvt.rn.satfinite.bf16x2.f32 %0, %1, %2;" : "=r"(w[h]) : "f"(y[2 * h + 1]), "f"(y[2 * h]));
      else
        asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(w[h]) : "f"(y[2 * h + 1]), "f"(y[2 * h]));
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// One element (ragged column tails).
template <int T>
__device__ __forceinline__ void sr1(float x, uint32_t r, uint8_t* dst) {
  const SrFormat f = sr_format(T);
  const uint32_t b = __float_as_uint(x);
  const uint32_t a = b & 0x7FFFFFFFu;
  const float y = a >= 0x7F800000u ? x : __uint_as_float(sr_magnitude(a, r, f) | (b & 0x80000000u));
  if constexpr (T == B2X_E4M3 || T == B2X_E5M2) {
    const uint16_t v = T == B2X_E4M3 ? cvt_e4m3x2(y, 0.f) : cvt_e5m2x2(y, 0.f);
    *dst = (uint8_t)(v & 0xFF);
  } else {
    uint32_t w;
    if constexpr (T == B2X_BF16)
      asm("cvt.rn.satfinite.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(0.f), "f"(y));
    else
      asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(0.f), "f"(y));
    *reinterpret_cast<uint16_t*>(dst) = (uint16_t)(w & 0xFFFF);
  }
}

struct SrArgs {
  const float* x;
  const uint32_t* r;
  uint8_t* y;
  int64_t rows, cols, ld_x, ld_r, ld_y;  // strides in elements
  int64_t vec_per_row;                   // cols / 8 when every row start is 16-byte aligned, else 0
};

template <int T, int RS>
__global__ void __launch_bounds__(256) stoch_round_kernel(const SrArgs a) {
  constexpr int kOut = (T == B2X_E4M3 || T == B2X_E5M2) ? 1 : 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a.vec_per_row > 0) {
    const int64_t nvec = a.rows * a.vec_per_row;
    for (int64_t v = tid; v < nvec; v += stride) {
      const int64_t row = v / a.vec_per_row;
      const int64_t c = (v - row * a.vec_per_row) * 8;
      const float4* xp = reinterpret_cast<const float4*>(a.x + row * a.ld_x + c);
      const uint4* rp = reinterpret_cast<const uint4*>(a.r + row * a.ld_r + c);
      const float4 x0 = __ldcs(xp), x1 = __ldcs(xp + 1);
      const uint4 r0 = __ldcs(rp), r1 = __ldcs(rp + 1);
      const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      const uint32_t rs[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
      if constexpr (RS)
        rs8<T>(xs, rs, a.y + (row * a.ld_y + c) * kOut);
      else
        sr8<T>(xs, rs, a.y + (row * a.ld_y + c) * kOut);
    }
    // columns past the last full group of 8
    const int64_t tail0 = a.vec_per_row * 8;
    const int64_t ntail = (a.cols - tail0) * a.rows;
    for (int64_t i = tid; i < ntail; i += stride) {
      const int64_t row = i / (a.cols - tail0);
      const int64_t c = tail0 + (i - row * (a.cols - tail0));
      if constexpr (RS)
        rs1<T>(a.x[row * a.ld_x + c], a.r + row * a.ld_r, c, a.y + (row * a.ld_y + c) * kOut);
      else
        sr1<T>(a.x[row * a.ld_x + c], a.r[row * a.ld_r + c], a.y + (row * a.ld_y + c) * kOut);
    }
  } else {
    const int64_t n = a.rows * a.cols;
    for (int64_t i = tid; i < n; i += stride) {
      const int64_t row = i / a.cols;
      const int64_t c = i - row * a.cols;
      if constexpr (RS)
        rs1<T>(a.x[row * a.ld_x + c], a.r + row * a.ld_r, c, a.y + (row * a.ld_y + c) * kOut);
      else
        sr1<T>(a.x[row * a.ld_x + c], a.r[row * a.ld_r + c], a.y + (row * a.ld_y + c) * kOut);
    }
  }
}

cudaError_t launch_stoch_round(const float* x, const uint32_t* r, void* y, b2x_dtype yt, int64_t rows, int64_t cols,
                               int64_t ld_x, int64_t ld_r, int64_t ld_y, int num_sms, cudaStream_t st, int rs) {
  SrArgs a;
  a.x = x;
  a.r = r;
  a.y = reinterpret_cast<uint8_t*>(y);
  a.rows = rows;
  a.cols = cols;
  a.ld_x = ld_x;
  a.ld_r = ld_r;
  a.ld_y = ld_y;
  const int out_bytes = (yt == B2X_E4M3 || yt == B2X_E5M2) ? 1 : 2;
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((uintptr_t)r % 16 == 0) && ((uintptr_t)y % (8 * out_bytes) == 0) &&
                       (ld_x % 4 == 0) && (ld_r % 4 == 0) && ((ld_y * out_bytes) % (8 * out_bytes) == 0);
  a.vec_per_row = aligned ? cols / 8 : 0;
  const int64_t work = aligned ? rows * (cols / 8) + rows * (cols % 8) : rows * cols;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 8;  // 8 resident 256-thread CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (rs) {
    switch (yt) {
      case B2X_E4M3: stoch_round_kernel<B2X_E4M3, 1><<<(int)blocks, 256, 0, st>>>(a); break;
      case B2X_E5M2: stoch_round_kernel<B2X_E5M2, 1><<<(int)blocks, 256, 0, st>>>(a); break;
      case B2X_F16: stoch_round_kernel<B2X_F16, 1><<<(int)blocks, 256, 0, st>>>(a); break;
      default: stoch_round_kernel<B2X_BF16, 1><<<(int)blocks, 256, 0, st>>>(a); break;
    }
  } else {
    switch (yt) {
      case B2X_E4M3: stoch_round_kernel<B2X_E4M3, 0><<<(int)blocks, 256, 0, st>>>(a); break;
      case B2X_E5M2: stoch_round_kernel<B2X_E5M2, 0><<<(int)blocks, 256, 0, st>>>(a); break;
      case B2X_F16: stoch_round_kernel<B2X_F16, 0><<<(int)blocks, 256, 0, st>>>(a); break;
      default: stoch_round_kernel<B2X_BF16, 0><<<(int)blocks, 256, 0, st>>>(a); break;
    }
  }
  note_launch(1);
  return cudaGetLastError();
}

}  // namespace b2x
