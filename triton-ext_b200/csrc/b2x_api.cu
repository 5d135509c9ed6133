// C ABI of libb2x: argument validation, configuration, TMA descriptors and
// kernel launch.  No exception crosses this boundary; every entry point
// returns a b2x_status and records a message for b2x_last_error().
//
// Counterpart of the host side of matmul() (extensions/utlx/tlx/tutorials/
// blackwell_gemm_ws.py:1352-1483): the shape asserts (:1368-1369), the
// descriptor set-up (:1377-1379, matmul_tma_set_block_size_hook :401-429), the
// persistent grid min(NUM_SMS, tiles) (:1430) and the split-K gating of
// preprocess_configs (:487-497).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <utility>
#include "b2x_internal.h"
#include "b2x_ptx.cuh"

namespace b2x {

static thread_local char t_err[512] = {0};
static std::atomic<uint64_t> g_launches{0};

void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

static b2x_status fail(b2x_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return s;
}

static b2x_status cuda_fail(cudaError_t e, const char* what) {
  return fail(B2X_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

static std::mutex g_mu;
static std::unordered_map<int, int> g_num_sms;
static std::unordered_map<uint64_t, int> g_smem_attr;  // key: (device << 48) ^ func

static int device_num_sms(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_num_sms.find(dev);
  if (it != g_num_sms.end()) return it->second;
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  g_num_sms[dev] = n;
  return n;
}

cudaError_t ensure_smem_attr(const void* func, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  uint64_t key = ((uint64_t)dev << 48) ^ (uint64_t)(uintptr_t)func;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_smem_attr.find(key);
  if (it != g_smem_attr.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_smem_attr[key] = bytes;
  return e;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over a row-major [rows, K] byte matrix viewed as {128-byte K
// chunk x, row, chunk index}: a box {128, box_rows, chunks} lands in smem as
// `chunks` consecutive [box_rows x 128 B] 128B-swizzled tiles.
static bool encode_chunked_3d(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t ld_bytes,
                              uint32_t box_rows, uint32_t chunks) {
  auto fn = get_encode_fn();
  if (!fn || K % 128 != 0) return false;
  cuuint64_t dims[3] = {128, rows, K / 128};
  cuuint64_t strides[2] = {ld_bytes, 128};
  cuuint32_t box[3] = {128, box_rows, chunks};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D tensor map: dims {inner, outer}, row stride in bytes, box {bi, bo}.
static b2x_status encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                            uint64_t row_stride_bytes, uint32_t bi, uint32_t bo, CUtensorMapSwizzle sw,
                            const char* what) {
  auto fn = get_encode_fn();
  if (!fn) return fail(B2X_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {bi, bo};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B2X_ERR_INVALID_ARG, "cuTensorMapEncodeTiled(%s) failed with %d (dims %llu x %llu, stride %llu)",
                what, (int)r, (unsigned long long)inner, (unsigned long long)outer,
                (unsigned long long)row_stride_bytes);
  return B2X_OK;
}

static bool is_fp8(b2x_dtype t) { return t == B2X_E4M3 || t == B2X_E5M2; }
static uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

}  // namespace b2x

using namespace b2x;

extern "C" {

const char* b2x_last_error(void) { return t_err; }
int b2x_abi_version(void) { return B2X_ABI_VERSION; }
uint64_t b2x_launch_count(void) { return g_launches.load(); }

b2x_status b2x_check_device(void) {
  t_err[0] = 0;
  int v = 0;
  b2x_status st = b2x_read_device_status(&v);
  if (st != B2X_OK) return st;
  if (v != 0)
    return fail(B2X_ERR_TIMEOUT, "a kernel gave up a bounded wait (device status 0x%x: %s)", v,
                v == kStatusTimeoutProducer   ? "TMA producer"
                : v == kStatusTimeoutMma      ? "MMA issuer"
                : v == kStatusTimeoutEpilogue ? "epilogue"
                : v == kStatusTimeoutSplitK   ? "split-K finisher"
                : v == kStatusTimeoutAllReduce ? "fused all-reduce peer"
                : v == kStatusTimeoutCast     ? "cast loader"
                                              : "unknown");
  return B2X_OK;
}

b2x_status b2x_debug_inject(int what, uint64_t wait_timeout_ns) {
  t_err[0] = 0;
  if (what < 0 || what > 1) return fail(B2X_ERR_INVALID_ARG, "b2x_debug_inject: what must be 0 or 1 (got %d)", what);
  unsigned long long ns = wait_timeout_ns ? (unsigned long long)wait_timeout_ns : B2X_WAIT_TIMEOUT_NS;
  cudaError_t e = cudaMemcpyToSymbol(g_inject, &what, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "b2x_debug_inject");
  e = cudaMemcpyToSymbol(g_wait_ns, &ns, sizeof(ns));
  if (e != cudaSuccess) return cuda_fail(e, "b2x_debug_inject");
  return B2X_OK;
}

b2x_status b2x_read_device_status(int* status_out) {
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
  e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "clearing the device status word");
  if (status_out) *status_out = v;
  return B2X_OK;
}

// ---------------------------------------------------------------------- cast

static int64_t cast_nsegs(const b2x_cast_args* a) {
  bool flat = a->ld_x == a->cols && a->ld_q == a->cols;
  int64_t cols = flat ? a->rows * a->cols : a->cols;
  int64_t rows = flat ? 1 : a->rows;
  return rows * ((cols + 127) / 128);
}

size_t b2x_cast_workspace_size(const b2x_cast_args* a) {
  if (!a || a->mode != B2X_SCALE_TENSOR) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  return (size_t)cast_num_partials(cast_nsegs(a), device_num_sms(dev)) * sizeof(uint32_t);
}

b2x_status b2x_fp8_cast(const b2x_cast_args* a, void* stream) {
  t_err[0] = 0;
  if (!a) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: args is NULL");
  if (a->x_type != B2X_F32 && a->x_type != B2X_BF16)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_cast: input dtype must be fp32 or bf16 (got %d)", (int)a->x_type);
  if (!is_fp8(a->q_type))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_cast: output dtype must be e4m3 or e5m2 (got %d)", (int)a->q_type);
  if (a->rows < 0 || a->cols < 0) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: negative shape");
  if (a->rows == 0 || a->cols == 0) return B2X_OK;
  if (!a->x || !a->q) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: NULL x or q");
  if (a->ld_x < a->cols || a->ld_q < a->cols)
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: row stride smaller than cols");
  if (a->mode != B2X_SCALE_NONE && !a->scale) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: NULL scale");
  int64_t sc_cols = 0;
  switch (a->mode) {
    case B2X_SCALE_NONE:
    case B2X_SCALE_TENSOR:
    case B2X_SCALE_TENSOR_GIVEN:
      break;
    case B2X_SCALE_BLOCK_1x128:
      sc_cols = (a->cols + 127) / 128;
      break;
    case B2X_SCALE_MX_1x32:
      sc_cols = (a->cols + 31) / 32;
      break;
    case B2X_SCALE_BLOCK_128x128:
      sc_cols = (a->cols + 127) / 128;
      break;
    default:
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: unknown scale mode %d", (int)a->mode);
  }
  if (sc_cols && a->ld_scale < sc_cols)
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_cast: ld_scale %lld < %lld scale columns", (long long)a->ld_scale,
                (long long)sc_cols);
  if (a->mode == B2X_SCALE_TENSOR) {
    size_t need = b2x_cast_workspace_size(a);
    if (!a->workspace || a->workspace_bytes < need)
      return fail(B2X_ERR_WORKSPACE, "b2x_fp8_cast: per-tensor amax needs a %zu-byte workspace (got %zu)", need,
                  a->workspace_bytes);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = launch_cast(*a, device_num_sms(dev), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "b2x_fp8_cast launch");
  return B2X_OK;
}

b2x_status b2x_amax(const void* x, b2x_dtype xt, int64_t rows, int64_t cols, int64_t ld_x, float* out,
                    void* workspace, size_t workspace_bytes, void* stream) {
  t_err[0] = 0;
  if (xt != B2X_F32 && xt != B2X_BF16) return fail(B2X_ERR_UNSUPPORTED, "b2x_amax: dtype must be fp32 or bf16");
  if (!x || !out || rows <= 0 || cols <= 0 || ld_x < cols) return fail(B2X_ERR_INVALID_ARG, "b2x_amax: bad args");
  b2x_cast_args tmp{};
  tmp.rows = rows;
  tmp.cols = cols;
  tmp.ld_x = ld_x;
  tmp.ld_q = ld_x;
  tmp.mode = B2X_SCALE_TENSOR;
  size_t need = b2x_cast_workspace_size(&tmp);
  if (!workspace || workspace_bytes < need)
    return fail(B2X_ERR_WORKSPACE, "b2x_amax: needs a %zu-byte workspace (got %zu)", need, workspace_bytes);
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e =
      launch_amax(x, xt, rows, cols, ld_x, out, (uint32_t*)workspace, device_num_sms(dev), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "b2x_amax launch");
  return B2X_OK;
}

// ---------------------------------------------------------------------- GEMM

static int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

b2x_status b2x_gemm_default_config(const b2x_gemm_args* a, b2x_gemm_config* out) {
  t_err[0] = 0;
  if (!a || !out) return fail(B2X_ERR_INVALID_ARG, "b2x_gemm_default_config: NULL argument");
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_num_sms(dev);
  b2x_gemm_config c = a->config;
  const bool b_mn = a->ldb_n == 1 && a->ldb_k != 1;
  const bool blockscaled = a->scale_mode == B2X_SCALE_BLOCK_1x128;
  c.block_m = 128;
  c.block_k = 128;
  if (blockscaled) {
    // B scales are per 128x128 tile.  Paired CTAs take 256-wide tiles (two
    // scale columns); a single CTA takes 128-wide tiles.
    const bool bs_pair = a->M > 128 && c.num_ctas != 1;
    c.block_n = bs_pair && c.block_n != 128 ? 256 : 128;
    c.num_ctas = bs_pair ? 2 : 1;
    c.split_k = 1;
  }
  if (a->scale_mode == B2X_SCALE_MX_1x32) {
    // MX GEMM (fp8_gemm_mx.cu): 128 x 192 or 128 x 128 tiles on single CTAs
    // (two accumulators and the scale factors must fit 512 TMEM columns).
    if (c.block_n == 0) {
      double best = -1;
      const int bns[2] = {192, 128};
      const double weight[2] = {1.0, 0.92};
      for (int i = 0; i < 2; ++i) {
        int64_t units = (int64_t)ceil_div(a->M, 128) * ceil_div(a->N, bns[i]);
        int64_t waves = (units + sms - 1) / sms;
        double eff = (double)units / (double)(waves * sms) * weight[i];
        if (eff > best + 1e-9) best = eff, c.block_n = bns[i];
      }
    }
    c.num_ctas = 1;
    c.split_k = 1;
  }
  // M <= 64 with a K-major B runs the operand-swapped small-M kernel: 128
  // weight rows per unit (fp8_gemm_smallm.cu).
  const bool mx = a->scale_mode == B2X_SCALE_MX_1x32;
  const bool swap_ab = a->M <= 64 && !b_mn && !blockscaled && !mx && (c.block_n == 0 || c.block_n == 128);
  if (swap_ab) c.block_n = 128;
  if (c.block_n == 0) {
    // Score each tile shape by how well its units fill the last wave, times
    // its per-SM throughput relative to paired 256x256 tiles (pairs read a
    // third less operand data per SM than one CTA's 128x256 tile, which in
    // turn reads less per FLOP than 128x128).
    struct Cand { int bn, ctas; double weight; };
    const Cand cands[3] = {{256, 2, 1.0}, {256, 1, 0.90}, {128, 1, 0.82}};
    double best = -1;
    for (const Cand& cd : cands) {
      if (cd.ctas == 2 && (a->M <= 128 || blockscaled || (c.split_k > 1) || c.num_ctas == 1)) continue;
      if (cd.ctas == 1 && c.num_ctas == 2) continue;
      const int64_t rows = cd.ctas == 2 ? 256 : 128;
      const int64_t slots = cd.ctas == 2 ? sms / 2 : sms;
      int64_t units = (int64_t)ceil_div(a->M, rows) * ceil_div(a->N, cd.bn);
      int64_t waves = (units + slots - 1) / slots;
      double eff = (double)units / (double)(waves * slots) * cd.weight;
      if (eff > best + 1e-9) {
        best = eff;
        c.block_n = cd.bn;
        if (a->config.num_ctas == 0) c.num_ctas = cd.ctas;
      }
    }
    if (a->N <= 64 && !b_mn) c.block_n = 64, c.num_ctas = a->config.num_ctas;
  }
  const int k_tiles = ceil_div(a->K, 128);
  if (c.split_k > 1 && a->config.block_n == 0 && !blockscaled && !swap_ab) {
    // Split-K requested without a tile width: take the width whose units
    // fill the last wave best (decode shapes are bandwidth-bound and want
    // every SM streaming B).
    double best = -1;
    int bns[3] = {256, 128, 64};
    for (int bn : bns) {
      if (b_mn && bn < 128) continue;
      int64_t units = (int64_t)ceil_div(a->M, 128) * ceil_div(a->N, bn) * c.split_k;
      int64_t waves = (units + sms - 1) / sms;
      double eff = (double)units / (double)(waves * sms);
      if (eff > best + 1e-3) best = eff, c.block_n = bn;
    }
  }
  if (c.split_k == 0) {
    // Split-K only when the output tiles cannot fill the GPU, each split
    // keeps >= 4 K blocks (the gating of preprocess_configs :487-497).
    c.split_k = 1;
    int64_t mn = (int64_t)ceil_div(a->M, 128) * ceil_div(a->N, c.block_n);
    if (mn < sms && (a->N % 4) == 0) {
      // Also try narrower tiles: decode shapes are bandwidth-bound and want
      // many small units to spread the B stream over all SMs.
      int best_bn = c.block_n, best_sk = 1;
      double best_eff = 0;
      int bns[3] = {c.block_n, 128, 64};
      for (int bn : bns) {
        if (b_mn && bn < 128) continue;
        if (a->config.block_n && bn != a->config.block_n) continue;
        if (swap_ab && bn != 128) continue;
        int64_t mnb = (int64_t)ceil_div(a->M, 128) * ceil_div(a->N, bn);
        for (int sk = 1; sk <= 16; ++sk) {
          if (k_tiles < sk || k_tiles / sk < 4) break;
          int kps = ceil_div(k_tiles, sk);
          if ((int64_t)(sk - 1) * kps >= k_tiles) continue;  // every split owns >= 1 block
          int64_t units = mnb * sk;
          int64_t waves = (units + sms - 1) / sms;
          double eff = (double)units / (double)(waves * sms);
          double fill = units >= sms ? 1.0 : (double)units / sms;
          double score = eff * fill;
          if (score > best_eff + 1e-6) best_eff = score, best_bn = bn, best_sk = sk;
        }
      }
      c.block_n = best_bn;
      c.split_k = best_sk;
    }
  }
  if (c.group_size_m == 0) {
    // _select_group_size_m (blackwell_gemm_ws.py:344-368) in units of 128-row tiles.
    int num_m_tiles = ceil_div(a->M, 128);
    double ratio = (double)a->M / (double)(a->N > 0 ? a->N : 1);
    if (ratio > 10)
      c.group_size_m = 1;
    else if (ratio < 0.1)
      c.group_size_m = num_m_tiles < 64 ? num_m_tiles : 64;
    else
      c.group_size_m = num_m_tiles < 8 ? num_m_tiles : 8;
    if (c.group_size_m < 1) c.group_size_m = 1;
  }
  if (c.num_tmem_buffers == 0) c.num_tmem_buffers = 2;
  if (c.num_mma_groups == 0) c.num_mma_groups = 1;
  if (c.epilogue_subtile == 0) c.epilogue_subtile = c.block_n / 64 > 0 ? c.block_n / 64 : 1;
  // Paired CTAs (256x256 tiles over two SMs) for large non-split problems:
  // a third less operand traffic per SM.  Needs 256-wide tiles and more
  // than one 128-row block of M.
  const bool pair_ok = c.split_k == 1 && (c.block_n == 256 || blockscaled) && a->M > 128 && !mx;
  if (c.num_ctas == 0) c.num_ctas = pair_ok ? 2 : 1;
  if (c.num_ctas == 2 && !pair_ok) c.num_ctas = 1;
  *out = c;
  return B2X_OK;
}

size_t b2x_gemm_workspace_size(const b2x_gemm_args* a) {
  if (!a) return 0;
  b2x_gemm_config c;
  if (b2x_gemm_default_config(a, &c) != B2X_OK) return 0;
  if (a->scale_mode == B2X_SCALE_MX_1x32 && a->M > 0 && a->N > 0 && a->K > 0)
    return mx_workspace_bytes(a->M, a->N, a->K, c.block_n);
  if (c.split_k == 1 || c.split_k == 0) return 0;  // > 1: split-K; -1: stream-K (small M)
  uint64_t tiles = (uint64_t)ceil_div(a->M, 128) * ceil_div(a->N, c.block_n);
  return (size_t)(align_up((uint64_t)a->M * a->N * 4, 256) + align_up(tiles * 4, 256));
}

// Fused SwiGLU + fp8 quantize output of b2x_fp8_gemm_swiglu.
struct SwArgs {
  void* h;
  int64_t ld_h;
  int fmt, mode;  // fmt 0 e4m3 / 1 e5m2; mode 0 block 1x128 / 1 given per-tensor scale
  float* scale;
  int64_t ld_scale;
  const float* given;
  float* amax;
};

// The GEMM behind b2x_fp8_gemm, b2x_fp8_gemm_allreduce (ar != NULL: the
// paired kernel with the fused all-reduce epilogue) and b2x_fp8_gemm_swiglu
// (sw != NULL: the paired kernel with the SwiGLU + quantize epilogue).
static b2x_status fp8_gemm_impl(const b2x_gemm_args* a, const ArParams* ar, void* stream,
                                const SwArgs* sw = nullptr, bool clc = false) {
  if (!a) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: args is NULL");
  if (!is_fp8(a->a_type) || !is_fp8(a->b_type))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: A and B must be e4m3 or e5m2 (got %d, %d)", (int)a->a_type,
                (int)a->b_type);
  if (a->c_type != B2X_BF16 && a->c_type != B2X_F16)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: C must be bf16 or fp16 (got %d)", (int)a->c_type);
  if (a->M < 0 || a->N < 0 || a->K < 0) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: negative shape");
  if ((a->M == 0 || a->N == 0) && !ar) return B2X_OK;
  if (a->K == 0) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: K == 0 (C would be all zero)");
  if (a->M >= (1LL << 31) || a->N >= (1LL << 31) || a->K >= (1LL << 31))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: dimensions must be < 2^31");
  if (!a->a || !a->b || (!a->c && !sw)) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: NULL A, B or C");
  if (a->lda < a->K) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: lda (%lld) < K (%lld)", (long long)a->lda,
                                 (long long)a->K);
  if ((a->lda % 16) || ((uintptr_t)a->a % 16))
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: A must be 16-byte aligned with lda %% 16 == 0");
  bool b_mn;
  if (a->ldb_k == 1 && a->ldb_n >= a->K) {
    b_mn = false;
    if ((a->ldb_n % 16) || ((uintptr_t)a->b % 16))
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: K-major B needs 16-byte alignment and a row stride %% 16 == 0");
  } else if (a->ldb_n == 1 && a->ldb_k >= a->N) {
    b_mn = true;
    if ((a->ldb_k % 16) || ((uintptr_t)a->b % 16))
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: row-major B needs 16-byte alignment and a row stride %% 16 == 0");
  } else {
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: B strides (%lld, %lld) are not K-major or row-major",
                (long long)a->ldb_k, (long long)a->ldb_n);
  }
  if (!sw && (a->ldc < a->N || (a->ldc % 8) || ((uintptr_t)a->c % 16)))
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: C must be 16-byte aligned with ldc >= N and ldc %% 8 == 0");
  const bool blockscaled = a->scale_mode == B2X_SCALE_BLOCK_1x128;
  switch (a->scale_mode) {
    case B2X_SCALE_NONE:
      break;
    case B2X_SCALE_TENSOR:
    case B2X_SCALE_TENSOR_GIVEN:
      if (!a->scale_a || !a->scale_b) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: NULL scale pointer");
      break;
    case B2X_SCALE_BLOCK_1x128:
      if (!a->scale_a || !a->scale_b) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: NULL scale pointer");
      if (b_mn) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: block-scaled GEMM needs a K-major B");
      break;
    case B2X_SCALE_MX_1x32:
      if (!a->scale_a || !a->scale_b) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: NULL scale pointer");
      if (b_mn) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: MX GEMM needs a K-major B");
      if (a->K % 128)
        return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: MX GEMM needs K %% 128 == 0 (got %lld)", (long long)a->K);
      if (a->sa_stride_m < a->K / 32 || a->sb_stride_n < a->K / 32 || (a->sa_stride_m % 4) || (a->sb_stride_n % 4) ||
          ((uintptr_t)a->scale_a % 4) || ((uintptr_t)a->scale_b % 4))
        return fail(B2X_ERR_INVALID_ARG,
                    "b2x_fp8_gemm: MX scales are uint8 [rows, K/32] with 4-byte aligned rows (sa_stride_m, "
                    "sb_stride_n >= K/32 and %% 4 == 0)");
      break;
    default:
      return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: scale mode %d not supported for GEMM", (int)a->scale_mode);
  }
  const bool mx = a->scale_mode == B2X_SCALE_MX_1x32;

  b2x_gemm_config c;
  b2x_status s = b2x_gemm_default_config(a, &c);
  if (s != B2X_OK) return s;
  if (ar || sw) {  // fused epilogues run on the paired kernel's 256 x 256 tiles
    c.num_ctas = 2;
    c.block_n = 256;
    c.split_k = 1;
  }
  if (clc) {
    if (blockscaled || mx)
      return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_clc: runs the per-tensor / unscaled GEMM only");
    c.num_ctas = 1;  // single-CTA tiles: one CTA per unit, scheduled by cluster launch control
  }
  if (mx) {
    if (c.block_n != 128 && c.block_n != 192)
      return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: MX GEMM runs 128- or 192-wide tiles (got %d)", c.block_n);
    if (c.split_k > 1) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: MX GEMM runs with SPLIT_K = 1");
    const size_t need = mx_workspace_bytes(a->M, a->N, a->K, c.block_n);
    if (!a->workspace || a->workspace_bytes < need || ((uintptr_t)a->workspace % 256))
      return fail(B2X_ERR_WORKSPACE, "b2x_fp8_gemm: MX GEMM needs a %zu-byte workspace (256-byte aligned; got %zu)",
                  need, a->workspace_bytes);
  } else if (c.block_n != 64 && c.block_n != 128 && c.block_n != 256)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: BLOCK_SIZE_N must be 64, 128 or 256 (got %d)", c.block_n);
  if (b_mn && c.block_n < 128)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: row-major B needs BLOCK_SIZE_N >= 128");
  if (blockscaled && (c.split_k > 1 || (c.block_n != 128 && !(c.block_n == 256 && c.num_ctas == 2))))
    return fail(B2X_ERR_UNSUPPORTED,
                "b2x_fp8_gemm: block-scaled GEMM runs with SPLIT_K = 1 and 128-wide tiles (256 on CTA pairs)");
  const int k_tiles = ceil_div(a->K, 128);
  const bool stream_k = c.split_k == -1;
  if (stream_k && !(a->M <= 64 && !b_mn && !blockscaled && !mx && !ar && !sw && !clc && c.block_n == 128))
    return fail(B2X_ERR_UNSUPPORTED,
                "b2x_fp8_gemm: SPLIT_K = -1 (stream-K) is built for the small-M kernel: M <= 64, a K-major B, "
                "per-tensor scales, 128-wide tiles");
  if (c.split_k < 1 && !stream_k) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm: SPLIT_K must be >= 1 (or -1)");
  if (stream_k) {
    if (a->N % 4) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: stream-K needs N %% 4 == 0");
    size_t need = b2x_gemm_workspace_size(a);
    if (!a->workspace || a->workspace_bytes < need || ((uintptr_t)a->workspace % 16))
      return fail(B2X_ERR_WORKSPACE, "b2x_fp8_gemm: stream-K needs a zeroed %zu-byte workspace (got %zu)", need,
                  a->workspace_bytes);
  }
  if (c.split_k > 1) {
    int kps = ceil_div(k_tiles, c.split_k);
    if ((int64_t)(c.split_k - 1) * kps >= k_tiles)
      return fail(B2X_ERR_INVALID_ARG,
                  "b2x_fp8_gemm: SPLIT_K=%d leaves an empty split for %d K blocks of 128", c.split_k, k_tiles);
    if (a->N % 4) return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm: split-K needs N %% 4 == 0");
    size_t need = b2x_gemm_workspace_size(a);
    if (!a->workspace || a->workspace_bytes < need || ((uintptr_t)a->workspace % 16))
      return fail(B2X_ERR_WORKSPACE, "b2x_fp8_gemm: split-K needs a zeroed %zu-byte workspace (got %zu)", need,
                  a->workspace_bytes);
  }

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  GemmLaunch g;
  memset(&g, 0, sizeof(g));
  g.M = a->M;
  g.N = a->N;
  g.K = a->K;
  g.bn = c.block_n;
  g.stages = c.num_smem_buffers;
  g.group_size_m = c.group_size_m;
  g.split_k = c.split_k;
  g.a_fmt = a->a_type == B2X_E4M3 ? 0 : 1;
  g.b_fmt = a->b_type == B2X_E4M3 ? 0 : 1;
  g.b_mn = b_mn ? 1 : 0;
  g.c_half = a->c_type == B2X_F16 ? 1 : 0;
  g.scale_mode = a->scale_mode;
  g.scale_a = a->scale_a;
  g.scale_b = a->scale_b;
  g.sa_stride_m = a->sa_stride_m;
  g.sa_stride_k = a->sa_stride_k;
  g.sb_stride_k = a->sb_stride_k;
  g.sb_stride_n = a->sb_stride_n;
  g.c = a->c;
  g.ldc = a->ldc;
  g.num_sms = device_num_sms(dev);
  if (c.num_sms > 0 && c.num_sms < g.num_sms) g.num_sms = c.num_sms;
  g.pair = c.num_ctas == 2 ? 1 : 0;
  static const int trace_env = [] {
    const char* v = getenv("B2X_TRACE");
    return v && v[0] == '1' ? 1 : 0;
  }();
  g.trace = trace_env;
  // Both operands evict_last: measured best sustained (a streamed B marked
  // evict_first or evict_normal re-reads more under the power cap).
  g.l2_a = 0;
  g.l2_b = 0;
  g.small_m = (!g.pair && !blockscaled && !mx && a->M <= 64) ? 1 : 0;
  g.swap_ab = (!clc && g.small_m && !b_mn && c.block_n == 128) ? 1 : 0;
  g.clc = clc ? 1 : 0;
  if (mx) g.ws = reinterpret_cast<float*>(a->workspace);  // tiled scale atoms (fp8_gemm_mx.cu)
  if (c.split_k > 1 || stream_k) {
    g.ws = reinterpret_cast<float*>(a->workspace);
    g.counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(a->workspace) +
                                        align_up((uint64_t)a->M * a->N * 4, 256));
  }

  s = encode_2d(&g.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, a->a, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda, 128,
                g.swap_ab ? (uint32_t)smallm_tokens_tile(a->M) : (g.small_m ? 64u : 128u),
                CU_TENSOR_MAP_SWIZZLE_128B, "A");
  if (s != B2X_OK) return s;
  if (b_mn)
    s = encode_2d(&g.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, a->b, (uint64_t)a->N, (uint64_t)a->K, (uint64_t)a->ldb_k,
                  128, 128, CU_TENSOR_MAP_SWIZZLE_128B, "B (row-major)");
  else
    s = encode_2d(&g.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, a->b, (uint64_t)a->K, (uint64_t)a->N, (uint64_t)a->ldb_n,
                  128, g.pair ? (uint32_t)c.block_n / 2 : (uint32_t)c.block_n, CU_TENSOR_MAP_SWIZZLE_128B,
                  "B (K-major)");
  if (s != B2X_OK) return s;
  if (sw)  // the fp8 output h [M, N/2]: one 128 x 128-byte box per CTA tile
    s = encode_2d(&g.tmC, CU_TENSOR_MAP_DATA_TYPE_UINT8, sw->h, (uint64_t)(a->N / 2), (uint64_t)a->M,
                  (uint64_t)sw->ld_h, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B, "h");
  else
  s = encode_2d(&g.tmC, a->c_type == B2X_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                a->c, (uint64_t)a->N, (uint64_t)a->M, (uint64_t)a->ldc * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B, "C");
  if (s != B2X_OK) return s;
  if (g.small_m && !b_mn && !g.swap_ab) {
    CUtensorMap a3, b3;
    // K blocks per stage of the small-M kernel (MShape in fp8_gemm.cu).
    const uint32_t kps = c.block_n == 64 ? 4 : (c.block_n == 128 ? 2 : 1);
    if (encode_chunked_3d(&a3, a->a, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda, 64, kps) &&
        encode_chunked_3d(&b3, a->b, (uint64_t)a->K, (uint64_t)a->N, (uint64_t)a->ldb_n, (uint32_t)c.block_n, kps)) {
      g.tmA = a3;
      g.tmB = b3;
      g.chunk3d = 1;
    }
  }

  if (sw) {
    if (!g.pair || blockscaled || mx || b_mn)
      return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_swiglu: this GEMM does not run on the paired kernel");
    g.swiglu = 1;
    g.sw_mode = sw->mode;
    g.sw_fmt = sw->fmt;
    g.sw_scale = sw->scale;
    g.sw_ld_scale = sw->ld_scale;
    g.sw_given = sw->given;
    g.sw_amax = sw->amax;
  }
  if (ar) {
    if (!g.pair || blockscaled || c.split_k != 1 || c.block_n != 256 || b_mn)
      return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_allreduce: this shape does not run on the paired kernel");
    g.ar = *ar;
  }
  if (mx)
    e = launch_fp8_gemm_mx(g, (cudaStream_t)stream);
  else if (blockscaled)
    e = g.pair ? launch_fp8_gemm_blockscaled_pair(g, (cudaStream_t)stream)
               : launch_fp8_gemm_blockscaled(g, (cudaStream_t)stream);
  else if (g.pair)
    e = launch_fp8_gemm_pair(g, (cudaStream_t)stream);
  else if (g.swap_ab)
    e = launch_fp8_gemm_smallm(g, (cudaStream_t)stream);
  else
    e = launch_fp8_gemm(g, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "b2x_fp8_gemm launch");
  return B2X_OK;
}

b2x_status b2x_fp8_gemm(const b2x_gemm_args* a, void* stream) {
  t_err[0] = 0;
  return fp8_gemm_impl(a, nullptr, stream);
}

b2x_status b2x_fp8_gemm_clc(const b2x_gemm_args* a, void* stream) {
  t_err[0] = 0;
  return fp8_gemm_impl(a, nullptr, stream, nullptr, true);
}

b2x_status b2x_fp8_gemm_swiglu(const b2x_gemm_args* args, void* h, int64_t ld_h, b2x_dtype h_type,
                               b2x_scale_mode h_mode, float* h_scale, int64_t ld_h_scale, float* h_amax,
                               void* stream) {
  t_err[0] = 0;
  if (!args) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_swiglu: args is NULL");
  if (h_type != B2X_E4M3 && h_type != B2X_E5M2)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_swiglu: h must be e4m3 or e5m2");
  if (h_mode != B2X_SCALE_BLOCK_1x128 && h_mode != B2X_SCALE_TENSOR_GIVEN && h_mode != B2X_SCALE_MX_1x32)
    return fail(B2X_ERR_UNSUPPORTED,
                "b2x_fp8_gemm_swiglu: h scales are BLOCK_1x128 or MX_1x32 (computed) or TENSOR_GIVEN");
  if (args->scale_mode != B2X_SCALE_NONE && args->scale_mode != B2X_SCALE_TENSOR &&
      args->scale_mode != B2X_SCALE_TENSOR_GIVEN)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_swiglu: the gate+up GEMM takes per-tensor scales or none");
  if (args->M <= 0 || args->N <= 0 || args->N % 256)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_swiglu: N (gate + up rows) must be a positive multiple of 256");
  if (!(args->ldb_k == 1 && args->ldb_n >= args->K))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_swiglu: B must be K-major (interleaved [2I, K] weight)");
  if (args->config.split_k > 1 || args->config.num_ctas == 1 ||
      (args->config.block_n && args->config.block_n != 256))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_swiglu: runs on CTA pairs with 256-wide tiles and SPLIT_K = 1");
  const int64_t I = args->N / 2;
  if (!h || ld_h < I || (ld_h % 16) || ((uintptr_t)h % 16))
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_swiglu: h must be 16-byte aligned with ld_h >= N/2, %% 16 == 0");
  if (!h_scale) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_swiglu: NULL h_scale");
  if (h_mode == B2X_SCALE_BLOCK_1x128 && ld_h_scale < I / 128)
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_swiglu: ld_h_scale must be >= N/256");
  if (h_mode == B2X_SCALE_MX_1x32 && (ld_h_scale < I / 32 || (ld_h_scale % 4) || ((uintptr_t)h_scale % 4)))
    return fail(B2X_ERR_INVALID_ARG,
                "b2x_fp8_gemm_swiglu: MX scales are uint8 [M, N/64] with a 4-byte aligned base and row stride");
  SwArgs sw;
  sw.h = h;
  sw.ld_h = ld_h;
  sw.fmt = h_type == B2X_E4M3 ? 0 : 1;
  sw.mode = h_mode == B2X_SCALE_BLOCK_1x128 ? 0 : (h_mode == B2X_SCALE_MX_1x32 ? 2 : 1);
  sw.scale = h_scale;
  sw.ld_scale = ld_h_scale;
  sw.given = h_scale;
  sw.amax = h_amax;
  b2x_gemm_args a = *args;
  a.c_type = B2X_BF16;
  a.config.block_n = 256;
  a.config.num_ctas = 2;
  a.config.split_k = 1;
  return fp8_gemm_impl(&a, nullptr, stream, &sw);
}

size_t b2x_allreduce_signal_words(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return (size_t)kArArrive0;
  return (size_t)kArArrive0 + (size_t)((M + 127) / 128) * (size_t)((N + 255) / 256);
}

b2x_status b2x_fp8_gemm_allreduce(const b2x_gemm_args* args, const b2x_allreduce_args* r, void* stream) {
  t_err[0] = 0;
  if (!args || !r) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: NULL argument");
  if (r->world < 1 || r->world > B2X_AR_MAX_RANKS || r->rank < 0 || r->rank >= r->world)
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: rank %d / world %d out of range", r->rank, r->world);
  if (args->c_type != B2X_BF16)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_allreduce: C must be bf16");
  if (args->scale_mode == B2X_SCALE_BLOCK_1x128)
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_allreduce: block-scaled operands are not supported");
  if (args->M <= 0 || args->N <= 0 || (args->M % 256) || (args->N % 256))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_allreduce: M and N must be positive multiples of 256 (got %lld, %lld)",
                (long long)args->M, (long long)args->N);
  if (!(args->ldb_k == 1 && args->ldb_n >= args->K))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_allreduce: B must be K-major (an nn.Linear weight viewed as w.t())");
  if (args->config.split_k > 1 || args->config.num_ctas == 1 || (args->config.block_n && args->config.block_n != 256))
    return fail(B2X_ERR_UNSUPPORTED, "b2x_fp8_gemm_allreduce: runs on CTA pairs with 256-wide tiles and SPLIT_K = 1");
  if (r->c_peers[r->rank] != args->c)
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: args->c must be c_peers[rank]");
  const bool mc = r->c_multicast != nullptr;
  if (mc != (r->signal_multicast != nullptr))
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: give both multicast addresses or neither");
  for (int i = 0; i < r->world; ++i) {
    if (!r->signal_peers[i] || ((uintptr_t)r->signal_peers[i] % 16))
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: signal_peers[%d] missing or not 16-byte aligned", i);
    if (!mc && (!r->c_peers[i] || ((uintptr_t)r->c_peers[i] % 16)))
      return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: c_peers[%d] missing or not 16-byte aligned", i);
  }
  if (mc && (((uintptr_t)r->c_multicast % 16) || ((uintptr_t)r->signal_multicast % 16)))
    return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_allreduce: multicast addresses must be 16-byte aligned");
  ArParams ar;
  memset(&ar, 0, sizeof(ar));
  ar.mode = mc ? 1 : 2;
  ar.rank = r->rank;
  ar.world = r->world;
  ar.c_mc = reinterpret_cast<uint8_t*>(r->c_multicast);
  ar.sig_mc = reinterpret_cast<uint32_t*>(r->signal_multicast);
  for (int i = 0; i < r->world; ++i) {
    ar.c_peer[i] = reinterpret_cast<uint8_t*>(r->c_peers[i]);
    ar.sig_peer[i] = reinterpret_cast<uint32_t*>(r->signal_peers[i]);
  }
  const uint32_t units = (uint32_t)(b2x_allreduce_signal_words(args->M, args->N) - kArArrive0);
  ar.units = units;
  ar.device_epoch = r->epoch == 0;
  ar.done_target = r->epoch * units;  // wraps modulo 2^32, compared as a difference
  b2x_gemm_args a = *args;
  a.config.block_n = 256;
  a.config.num_ctas = 2;
  a.config.split_k = 1;
  return fp8_gemm_impl(&a, &ar, stream);
}

static b2x_status stoch_round_impl(const char* who, int rs, const float* x, int64_t rows, int64_t cols, int64_t ld_x,
                                   const uint32_t* rbits, int64_t ld_r, void* y, b2x_dtype y_type, int64_t ld_y,
                                   void* stream) {
  t_err[0] = 0;
  if (y_type != B2X_E4M3 && y_type != B2X_E5M2 && y_type != B2X_F16 && y_type != B2X_BF16)
    return fail(B2X_ERR_UNSUPPORTED, "%s: target must be e4m3, e5m2, fp16 or bf16 (got %d)", who, (int)y_type);
  if (rows < 0 || cols < 0) return fail(B2X_ERR_INVALID_ARG, "%s: negative shape", who);
  if (rows == 0 || cols == 0) return B2X_OK;
  if (!x || !rbits || !y) return fail(B2X_ERR_INVALID_ARG, "%s: NULL pointer", who);
  if (ld_x < cols || ld_r < cols || ld_y < cols)
    return fail(B2X_ERR_INVALID_ARG, "%s: a row stride is smaller than cols", who);
  const int out_bytes = (y_type == B2X_E4M3 || y_type == B2X_E5M2) ? 1 : 2;
  if (((uintptr_t)x % 4) || ((uintptr_t)rbits % 4) || ((uintptr_t)y % out_bytes))
    return fail(B2X_ERR_INVALID_ARG, "%s: misaligned pointer", who);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = launch_stoch_round(x, rbits, y, y_type, rows, cols, ld_x, ld_r, ld_y, device_num_sms(dev), (cudaStream_t)stream, rs);
  if (e != cudaSuccess) return cuda_fail(e, who);
  return B2X_OK;
}

b2x_status b2x_stoch_round(const float* x, int64_t rows, int64_t cols, int64_t ld_x, const uint32_t* rbits,
                           int64_t ld_r, void* y, b2x_dtype y_type, int64_t ld_y, void* stream) {
  return stoch_round_impl("b2x_stoch_round", 0, x, rows, cols, ld_x, rbits, ld_r, y, y_type, ld_y, stream);
}

b2x_status b2x_stoch_round_rs(const float* x, int64_t rows, int64_t cols, int64_t ld_x, const uint32_t* rbits,
                              int64_t ld_r, void* y, b2x_dtype y_type, int64_t ld_y, void* stream) {
  return stoch_round_impl("b2x_stoch_round_rs", 1, x, rows, cols, ld_x, rbits, ld_r, y, y_type, ld_y, stream);
}

b2x_status b2x_trace_read(uint64_t* out, int max_ctas, int* n_ctas) {
  t_err[0] = 0;
  if (!out || max_ctas <= 0) return fail(B2X_ERR_INVALID_ARG, "b2x_trace_read: bad output buffer");
  const int n = max_ctas < kTraceMaxCtas ? max_ctas : kTraceMaxCtas;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_trace, sizeof(unsigned long long) * kTraceSlots * n);
  if (e != cudaSuccess) return cuda_fail(e, "reading the trace counters");
  static unsigned long long zeros[kTraceMaxCtas * kTraceSlots];
  e = cudaMemcpyToSymbol(g_trace, zeros, sizeof(zeros));
  if (e != cudaSuccess) return cuda_fail(e, "clearing the trace counters");
  if (n_ctas) *n_ctas = n;
  return B2X_OK;
}

b2x_status b2x_splitk_reduce(const void* ws, b2x_dtype wt, void* c, b2x_dtype ct, int64_t M, int64_t N, int64_t ldc,
                             int split_k, void* stream) {
  t_err[0] = 0;
  if (!ws || !c) return fail(B2X_ERR_INVALID_ARG, "b2x_splitk_reduce: NULL pointer");
  if (M < 0 || N < 0 || split_k < 1 || ldc < N) return fail(B2X_ERR_INVALID_ARG, "b2x_splitk_reduce: bad shape");
  auto ok_t = [](b2x_dtype t) { return t == B2X_F32 || t == B2X_BF16 || t == B2X_F16; };
  if (!ok_t(wt) || !ok_t(ct)) return fail(B2X_ERR_UNSUPPORTED, "b2x_splitk_reduce: dtypes must be fp32/bf16/fp16");
  if (M == 0 || N == 0) return B2X_OK;
  cudaError_t e = launch_splitk_reduce(ws, wt, c, ct, M, N, ldc, split_k, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "b2x_splitk_reduce launch");
  return B2X_OK;
}

}  // extern "C"
