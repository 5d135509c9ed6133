/*
 * C restatement of the b2x fp8 path -- TEST INFRASTRUCTURE / TIMED CPU REFERENCE ONLY.
 *
 * Used by tests/ (cross-checked against oracle/fp8_oracle.py) and by bench.py
 * as the timed CPU baseline and the `--impl reference` arm.  Never linked
 * into libb2x.
 *
 * quantize: the recipe of _compute_scale_and_quantize
 *   (extensions/utlx/tlx/language/tlx/mxfp8_utils.py:37-84):
 *   amax (NaN-ignoring) -> scale = amax / FMAX -> [MX: RCEIL to 2^e] ->
 *   inv = scale == 0 ? 0 : 1 / scale -> clamp(x * inv, -FMAX, FMAX), NaN-ignoring
 *   -> fp8 round-to-nearest-even, saturating.
 * gemm: C = sA * sB * (A . B) with fp32 accumulation and a bf16 result, the
 *   arithmetic of matmul_kernel_tma_ws_blackwell (blackwell_gemm_ws.py:1089)
 *   on fp8 operands; B is taken K-major ([N][K]).
 * stoch_round: tlx.stoch_round (extensions/utlx/tlx/language/tlx/utility.py:
 *   113-153) with one uint32 of entropy per element, restated in floating
 *   point (the numpy oracle restates it with integers; tests compare the two).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

#define FMT_E4M3 0
#define FMT_E5M2 1

enum { MODE_NONE = 0, MODE_TENSOR = 1, MODE_BLOCK1x128 = 3, MODE_BLOCK128x128 = 4, MODE_MX1x32 = 5 };

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* fp32 -> fp8 byte, round-to-nearest-even, saturate to the largest finite value. */
static inline uint8_t to_fp8(float x, int fmt) {
  uint32_t u = f2u(x);
  uint8_t sign = (uint8_t)((u >> 24) & 0x80);
  uint32_t ua = u & 0x7FFFFFFFu;
  if (ua > 0x7F800000u) return (uint8_t)(0x7F | sign); /* NaN */
  float a = u2f(ua);
  const int mbits = fmt == FMT_E4M3 ? 3 : 2;
  const int bias = fmt == FMT_E4M3 ? 7 : 15;
  const int min_exp = fmt == FMT_E4M3 ? -6 : -14;
  const uint32_t max_code = fmt == FMT_E4M3 ? 0x7E : 0x7B;
  const float fmax = fmt == FMT_E4M3 ? 448.0f : 57344.0f;
  if (a >= fmax) return (uint8_t)(max_code | sign);
  if (a < ldexpf(1.0f, min_exp)) {
    float v = a * ldexpf(1.0f, mbits - min_exp); /* exact: power-of-two scaling */
    uint32_t c = (uint32_t)nearbyintf(v);       /* default rounding mode: to nearest even */
    return (uint8_t)(c | sign);
  }
  const int drop = 23 - mbits;
  uint32_t lsb = (ua >> drop) & 1u;
  uint32_t r = (ua + ((1u << (drop - 1)) - 1u) + lsb) & ~((1u << drop) - 1u);
  int e = (int)(r >> 23) - 127 + bias;
  uint32_t m = (r >> drop) & ((1u << mbits) - 1u);
  uint32_t c = ((uint32_t)e << mbits) | m;
  if (c > max_code) c = max_code;
  return (uint8_t)(c | sign);
}


/* ---- minimal parallel-for over [0, n) on pthreads (static interleaved chunks) ---- */
typedef void (*range_fn)(void* ctx, int64_t i);
typedef struct { range_fn fn; void* ctx; int64_t n; int tid, nt; } worker_arg;
static void* worker(void* p) {
  worker_arg* w = (worker_arg*)p;
  for (int64_t i = w->tid; i < w->n; i += w->nt) w->fn(w->ctx, i);
  return NULL;
}
static int g_threads = 0;
int oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
static void parallel_for(int64_t n, range_fn fn, void* ctx) {
  int nt = g_threads > 0 ? g_threads : oracle_max_threads();
  if (nt > 256) nt = 256;
  if (nt > n) nt = (int)(n > 0 ? n : 1);
  pthread_t th[256];
  worker_arg args[256];
  for (int t = 0; t < nt; ++t) {
    args[t] = (worker_arg){fn, ctx, n, t, nt};
    if (t) pthread_create(&th[t], NULL, worker, &args[t]);
  }
  worker(&args[0]);
  for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
}

/* Symmetric clamp as a B200 computes tl.clamp(y, -m, m): NaN-ignoring min on
 * |y| with y's sign bit kept, so a NaN becomes +-m by its sign bit. */
static inline float clampf_nan_ignoring(float y, float m) { return copysignf(fminf(fabsf(y), m), y); }
/* The GPU's fp32 multiply returns the canonical positive NaN for NaN results. */
static inline float gpu_mul(float a, float b) {
  volatile float y = a * b;
  return isnan(y) ? NAN : y;
}

static inline float inv_of(float s) { return s == 0.0f ? 0.0f : 1.0f / s; }

static float absmax_range(const float* x, int64_t n) {
  float m = 0.0f;
  for (int64_t i = 0; i < n; ++i) m = fmaxf(m, fabsf(x[i])); /* fmaxf ignores NaN */
  return m;
}

typedef struct {
  const float* x;
  int64_t rows, cols, G, ng, tc;
  int fmt, mode;
  float fm, inv;
  uint8_t* q;
  void* scale;
  float* row_amax;
} quant_ctx;

static void amax_row(void* p, int64_t r) {
  quant_ctx* c = (quant_ctx*)p;
  c->row_amax[r] = absmax_range(c->x + r * c->cols, c->cols);
}

static void cast_row_uniform(void* p, int64_t r) {
  quant_ctx* c = (quant_ctx*)p;
  for (int64_t j = 0; j < c->cols; ++j) {
    float y = c->mode == MODE_NONE ? c->x[r * c->cols + j] : gpu_mul(c->x[r * c->cols + j], c->inv);
    c->q[r * c->cols + j] = to_fp8(clampf_nan_ignoring(y, c->fm), c->fmt);
  }
}

static void cast_row_groups(void* p, int64_t r) {
  quant_ctx* c = (quant_ctx*)p;
  for (int64_t g = 0; g < c->ng; ++g) {
    const int64_t c0 = g * c->G, n = (c0 + c->G <= c->cols) ? c->G : c->cols - c0;
    const float* xs = c->x + r * c->cols + c0;
    volatile float sc = absmax_range(xs, n) / c->fm;
    float inv;
    if (c->mode == MODE_MX1x32) {
      uint32_t e = (f2u(sc) + 0x007FFFFFu) & 0x7F800000u;
      inv = inv_of(u2f(e));
      ((uint8_t*)c->scale)[r * c->ng + g] = (uint8_t)(e >> 23);
    } else {
      inv = inv_of(sc);
      ((float*)c->scale)[r * c->ng + g] = sc;
    }
    for (int64_t i = 0; i < n; ++i) {
      float y = gpu_mul(xs[i], inv);
      c->q[r * c->cols + c0 + i] = to_fp8(clampf_nan_ignoring(y, c->fm), c->fmt);
    }
  }
}

static void cast_tile128(void* p, int64_t t) {
  quant_ctx* c = (quant_ctx*)p;
  const int64_t i = t / c->tc, j = t % c->tc;
  const int64_t r1 = (i * 128 + 128 < c->rows) ? i * 128 + 128 : c->rows;
  const int64_t c1 = (j * 128 + 128 < c->cols) ? j * 128 + 128 : c->cols;
  float m = 0.0f;
  for (int64_t r = i * 128; r < r1; ++r) {
    float v = absmax_range(c->x + r * c->cols + j * 128, c1 - j * 128);
    m = m > v ? m : v;
  }
  volatile float sc = m / c->fm;
  ((float*)c->scale)[i * c->tc + j] = sc;
  const float inv = inv_of(sc);
  for (int64_t r = i * 128; r < r1; ++r)
    for (int64_t cc = j * 128; cc < c1; ++cc) {
      float y = gpu_mul(c->x[r * c->cols + cc], inv);
      c->q[r * c->cols + cc] = to_fp8(clampf_nan_ignoring(y, c->fm), c->fmt);
    }
}

int oracle_quantize(const float* x, int64_t rows, int64_t cols, int fmt, int mode, uint8_t* q, void* scale,
                    int nthreads) {
  g_threads = nthreads;
  quant_ctx c;
  memset(&c, 0, sizeof(c));
  c.x = x, c.rows = rows, c.cols = cols, c.fmt = fmt, c.mode = mode, c.q = q, c.scale = scale;
  c.fm = fmt == FMT_E4M3 ? 448.0f : 57344.0f;
  c.inv = 1.0f;
  if (mode == MODE_NONE || mode == MODE_TENSOR) {
    if (mode == MODE_TENSOR) {
      c.row_amax = (float*)malloc(sizeof(float) * (size_t)(rows > 0 ? rows : 1));
      parallel_for(rows, amax_row, &c);
      float amax = 0.0f;
      for (int64_t r = 0; r < rows; ++r) amax = fmaxf(amax, c.row_amax[r]);
      free(c.row_amax);
      volatile float sc = amax / c.fm;
      ((float*)scale)[0] = sc;
      c.inv = inv_of(sc);
    }
    parallel_for(rows, cast_row_uniform, &c);
    return 0;
  }
  if (mode == MODE_BLOCK1x128 || mode == MODE_MX1x32) {
    c.G = mode == MODE_BLOCK1x128 ? 128 : 32;
    c.ng = (cols + c.G - 1) / c.G;
    parallel_for(rows, cast_row_groups, &c);
    return 0;
  }
  if (mode == MODE_BLOCK128x128) {
    c.tc = (cols + 127) / 128;
    parallel_for(((rows + 127) / 128) * c.tc, cast_tile128, &c);
    return 0;
  }
  return -1;
}

static void decode_table(int fmt, float* t) {
  for (int c = 0; c < 256; ++c) {
    float s = (c & 0x80) ? -1.0f : 1.0f;
    float v;
    if (fmt == FMT_E4M3) {
      int e = (c >> 3) & 15, m = c & 7;
      if (e == 15 && m == 7) v = NAN;
      else if (e == 0) v = ldexpf((float)m, -9);
      else v = ldexpf(1.0f + m / 8.0f, e - 7);
    } else {
      int e = (c >> 2) & 31, m = c & 3;
      if (e == 31) v = m ? NAN : INFINITY;
      else if (e == 0) v = ldexpf((float)m, -16);
      else v = ldexpf(1.0f + m / 4.0f, e - 15);
    }
    t[c] = s * v;
  }
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/*
 * C[m, n] = bf16(sa * sb * sum_k A[m, k] * Bt[n, k]) for rows [m0, m1) and
 * columns [n0, n1) (a bounded sample of the full product when the range is
 * smaller than M x N).  fp32 accumulation.  Returns the FLOPs done.
 */
typedef struct {
  const uint8_t *A, *Bt;
  int64_t lda, ldb, K, ldc, m0, m1, n0, n1;
  float ta[256], tb[256];
  float alpha;
  uint16_t* C;
} gemm_ctx;

#define GEMM_NB 64
static void gemm_colblock(void* p, int64_t blk) {
  gemm_ctx* g = (gemm_ctx*)p;
  const int64_t K = g->K;
  const int64_t nb = g->n0 + blk * GEMM_NB;
  const int64_t ne = nb + GEMM_NB < g->n1 ? nb + GEMM_NB : g->n1;
  float* arow = (float*)malloc(sizeof(float) * (size_t)K);
  float* bcol = (float*)malloc(sizeof(float) * (size_t)K * GEMM_NB);
  for (int64_t n = nb; n < ne; ++n)
    for (int64_t k = 0; k < K; ++k) bcol[(n - nb) * K + k] = g->tb[g->Bt[n * g->ldb + k]];
  for (int64_t m = g->m0; m < g->m1; ++m) {
    for (int64_t k = 0; k < K; ++k) arow[k] = g->ta[g->A[m * g->lda + k]];
    for (int64_t n = nb; n < ne; ++n) {
      const float* b = bcol + (n - nb) * K;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int64_t k = 0;
      for (; k + 8 <= K; k += 8)
        for (int u = 0; u < 8; ++u) acc[u] += arow[k + u] * b[k + u];
      for (; k < K; ++k) acc[0] += arow[k] * b[k];
      float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      g->C[m * g->ldc + n] = f32_to_bf16(s * g->alpha);
    }
  }
  free(arow);
  free(bcol);
}

double oracle_gemm_bf16(const uint8_t* A, int64_t lda, int a_fmt, const uint8_t* Bt, int64_t ldb, int b_fmt,
                        int64_t K, float sa, float sb, uint16_t* C, int64_t ldc, int64_t m0, int64_t m1, int64_t n0,
                        int64_t n1, int nthreads) {
  g_threads = nthreads;
  gemm_ctx* g = (gemm_ctx*)malloc(sizeof(gemm_ctx));
  g->A = A, g->Bt = Bt, g->lda = lda, g->ldb = ldb, g->K = K, g->ldc = ldc;
  g->m0 = m0, g->m1 = m1, g->n0 = n0, g->n1 = n1, g->C = C;
  g->alpha = sa * sb;
  decode_table(a_fmt, g->ta);
  decode_table(b_fmt, g->tb);
  parallel_for((n1 - n0 + GEMM_NB - 1) / GEMM_NB, gemm_colblock, g);
  free(g);
  return 2.0 * (double)(m1 - m0) * (double)(n1 - n0) * (double)K;
}

/* ------------------------------------------------------------------------
 * Stochastic rounding (tlx.stoch_round, extensions/utlx/tlx/language/tlx/
 * utility.py:113-153), restated with floating-point arithmetic instead of the
 * integer formulation of fp8_oracle.py:  t = |x| / q exactly (q the target's
 * quantum at |x|), frac32 = floor((t - floor(t)) * 2^32), round up iff
 * frac32 + r >= 2^32, then a saturating encode.  fmt: 0 e4m3, 1 e5m2,
 * 2 fp16, 3 bf16.  Output: uint8 (fp8) or uint16 (fp16 / bf16) codes.
 */
static uint16_t encode_half(double v, int fp16) {
  /* v is exactly representable in the target or beyond its range (saturate). */
  const int mb = fp16 ? 10 : 7, bias = fp16 ? 15 : 127, emin = fp16 ? -14 : -126;
  const double vmax = fp16 ? 65504.0 : ldexp(2.0 - ldexp(1.0, -7), 127);
  uint16_t sign = signbit(v) ? 0x8000 : 0;
  double a = fabs(v);
  if (a >= vmax) return (uint16_t)(sign | (fp16 ? 0x7BFF : 0x7F7F));
  if (a == 0.0) return sign;
  int e;
  frexp(a, &e); /* a = f * 2^e, f in [0.5, 1) */
  e -= 1;       /* a in [2^e, 2^(e+1)) */
  if (e < emin) return (uint16_t)(sign | (uint16_t)llround(a / ldexp(1.0, emin - mb)));
  uint32_t m = (uint32_t)llround(a / ldexp(1.0, e - mb)) - (1u << mb);
  return (uint16_t)(sign | ((uint32_t)(e + bias) << mb) | m);
}

void oracle_stoch_round(const float* x, const uint32_t* r, int64_t n, int fmt, void* out) {
  static const int P[4] = {3, 2, 10, 7}, EMIN[4] = {-6, -14, -14, -126};
  for (int64_t i = 0; i < n; ++i) {
    const float xi = x[i];
    double y;
    if (isnan(xi)) {
      y = NAN;
    } else if (isinf(xi)) {
      y = xi;
    } else if (xi == 0.0f) {
      y = xi;
    } else {
      const double a = fabs((double)xi);
      int e;
      frexp(a, &e);
      e -= 1;
      const int ue = (e > EMIN[fmt] ? e : EMIN[fmt]) - P[fmt];
      const double t = ldexp(a, -ue); /* exact */
      const double q = floor(t);
      const double f32 = floor((t - q) * 4294967296.0);
      const double up = (f32 + (double)r[i] >= 4294967296.0) ? 1.0 : 0.0;
      y = copysign(ldexp(q + up, ue), (double)xi);
    }
    if (fmt <= 1) {
      ((uint8_t*)out)[i] = isnan(y) ? (uint8_t)(0x7F | (signbit(xi) ? 0x80 : 0)) : to_fp8((float)y, fmt);
    } else {
      ((uint16_t*)out)[i] = isnan(y) ? (uint16_t)0x7FFF : encode_half(y, fmt == 2);
    }
  }
}
