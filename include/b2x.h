/*
 * b2x — C ABI of the B200-native fp8 GEMM / fp8 cast / split-K library.
 *
 * This is the drop-in boundary that replaces, for one data path, what the
 * reference reaches through Triton plugin machinery:
 *   - the op-level Python entry point `matmul(a, b, config=None, use_heuristic=False)`
 *     (extensions/utlx/tlx/tutorials/blackwell_gemm_ws.py:1352) and the kernel
 *     it launches, `matmul_kernel_tma_ws_blackwell` (:1089-1349);
 *   - the split-K reduction `_reduce_k_kernel` (blackwell_gemm_ws.py:1033-1056);
 *   - the fp8 quantize helper `_compute_scale_and_quantize`
 *     (extensions/utlx/tlx/language/tlx/mxfp8_utils.py:13-86) and the
 *     fp32 -> fp8 cast it ends in (`.to(fp8)`, round-to-nearest-even).
 * The reference's own binary boundary, `tritonGetPluginInfo()`
 * (extensions/utlx/uTLXPlugin.cpp:700-814), is compile-time MLIR plumbing and
 * has no counterpart here: b2x ships finished sm_100a kernels.
 *
 * Conventions
 *   - Plain pointers and sizes; no torch types.  All device pointers belong to
 *     the caller, including workspaces (query their size first).
 *   - Every call is asynchronous on the given stream (cudaStream_t passed as
 *     void*; NULL = legacy default stream) and never synchronises.
 *   - No C++ exception crosses this ABI.  Errors come back as a b2x_status;
 *     b2x_last_error() gives a message for the calling thread's last failure.
 *   - Thread-safe: the only shared state is a per-device cache of kernel
 *     attributes guarded by a mutex.
 *   - Kernels never trap.  Every internal wait is bounded; a wait that gives
 *     up records a code in a per-device status word (b2x_read_device_status)
 *     and the kernel returns early.
 */
#ifndef B2X_H_
#define B2X_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2X_ABI_VERSION 1

#if defined(__GNUC__)
#define B2X_API __attribute__((visibility("default")))
#else
#define B2X_API
#endif

typedef enum {
  B2X_OK = 0,
  B2X_ERR_INVALID_ARG = 1,  /* bad shape / stride / pointer / alignment */
  B2X_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement */
  B2X_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed */
  B2X_ERR_TIMEOUT = 4,      /* a kernel wait gave up (see b2x_read_device_status) */
  B2X_ERR_WORKSPACE = 5     /* workspace missing or too small */
} b2x_status;

typedef enum {
  B2X_F32 = 0,
  B2X_BF16 = 1,
  B2X_F16 = 2,
  B2X_E4M3 = 3, /* float8_e4m3fn: bias 7, max 448, no inf, NaN = S.1111.111 */
  B2X_E5M2 = 4, /* float8_e5m2: bias 15, max 57344, IEEE-style inf/NaN */
  B2X_U8 = 5    /* raw bytes, used for E8M0 scales */
} b2x_dtype;

/* How an fp8 tensor is scaled: x ~= q * scale. */
typedef enum {
  B2X_SCALE_NONE = 0,         /* scale = 1, plain saturating RNE cast */
  B2X_SCALE_TENSOR = 1,       /* one fp32 scale for the tensor, computed from amax */
  B2X_SCALE_TENSOR_GIVEN = 2, /* one fp32 scale supplied by the caller (static) */
  B2X_SCALE_BLOCK_1x128 = 3,  /* fp32 scale per (row, 128-column block) */
  B2X_SCALE_BLOCK_128x128 = 4,/* fp32 scale per (128-row, 128-column) tile */
  B2X_SCALE_MX_1x32 = 5       /* E8M0 (uint8 biased exponent) per (row, 32-column block), RCEIL */
} b2x_scale_mode;

/* ------------------------------------------------------------------ cast */

/*
 * Quantize a 2-D fp32/bf16 tensor x[rows, cols] (row stride ld_x elements,
 * unit column stride) to fp8 q[rows, cols] (row stride ld_q), computing (or,
 * for B2X_SCALE_TENSOR_GIVEN, reading) the scales.
 *
 * Per group of elements sharing one scale (amax is a NaN-ignoring max of |x|):
 *   scale = amax / FMAX                    (IEEE fp32 division; FMAX 448 / 57344)
 *   inv   = scale == 0 ? 0 : 1 / scale     (IEEE fp32 division)
 *   q     = fp8_rne_satfinite(clamp(x * inv, -FMAX, FMAX))
 * and for B2X_SCALE_MX_1x32 the scale is rounded up to a power of two (RCEIL)
 * and stored as its biased exponent byte.
 * Replaces: _compute_scale_and_quantize, mxfp8_utils.py:13-86 (1x32 E8M0) and
 * the per-tensor / 1x128 / 128x128 amax scaling of the same recipe.
 *
 * scale layout (row-major, ld_scale elements per row):
 *   TENSOR / TENSOR_GIVEN: 1 fp32
 *   BLOCK_1x128:           [rows, ceil(cols/128)] fp32
 *   BLOCK_128x128:         [ceil(rows/128), ceil(cols/128)] fp32
 *   MX_1x32:               [rows, ceil(cols/32)] uint8
 */
typedef struct {
  const void* x;
  b2x_dtype x_type; /* B2X_F32 or B2X_BF16 */
  int64_t rows, cols, ld_x;
  void* q;
  b2x_dtype q_type; /* B2X_E4M3 or B2X_E5M2 */
  int64_t ld_q;
  void* scale;
  b2x_scale_mode mode;
  int64_t ld_scale;
  void* workspace; /* B2X_SCALE_TENSOR only: see b2x_cast_workspace_size */
  size_t workspace_bytes;
} b2x_cast_args;

B2X_API size_t b2x_cast_workspace_size(const b2x_cast_args* args);
B2X_API b2x_status b2x_fp8_cast(const b2x_cast_args* args, void* stream);

/* Amax only (NaN-ignoring max |x|) of a 2-D tensor, written as one fp32. */
B2X_API b2x_status b2x_amax(const void* x, b2x_dtype x_type, int64_t rows, int64_t cols, int64_t ld_x, float* amax_out,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Stochastic rounding y = SR(x, r) of an fp32 [rows, cols] tensor to e4m3,
 * e5m2, fp16 or bf16, with one uint32 of caller-given entropy per element
 * (rbits [rows, cols], row stride ld_r).  |x| is truncated to the target's
 * precision at its binade (subnormals included) and rounds up one quantum
 * exactly when frac32 + r >= 2^32, where frac32 is the first 32 bits of the
 * dropped remainder as a fraction of the quantum; so P(up) = frac32 / 2^32
 * and E[y] = x up to 2^-32 of a quantum.  The sign is kept, values already
 * representable are unchanged, results beyond the largest finite value
 * (Inf included) saturate to +-max, NaN stays NaN.  Strides in elements.
 * Replaces tlx.stoch_round(src, dst_ty, rand_bits),
 * extensions/utlx/tlx/language/tlx/utility.py:113-153.
 */
B2X_API b2x_status b2x_stoch_round(const float* x, int64_t rows, int64_t cols, int64_t ld_x, const uint32_t* rbits,
                                   int64_t ld_r, void* y, b2x_dtype y_type, int64_t ld_y, void* stream);

/*
 * Stochastic rounding with the hardware instruction the reference's lowering
 * emits, cvt.rs.satfinite (extensions/utlx/test/test_tlx.py:5182 asserts it;
 * the rounding mode "rs" is chosen in extensions/utlx/ops/NewOps.cpp:249-303).
 * Same arguments as b2x_stoch_round.  The instruction rounds a pack of 4
 * (e4m3 / e5m2) or 2 (fp16 / bf16) values with one 32-bit entropy word split
 * into per-lane fields.  Packs are consecutive columns of a row starting at
 * column 0; a pack takes the rbits word of its first element and ignores the
 * others (how the reference's Triton lowering folds per-element words into a
 * pack is in Triton, outside the reference tree, so a bit-for-bit match with
 * tlx.stoch_round for the same rand_bits is not claimed).  What the
 * reference's tests check holds: representable values are unchanged, finite
 * inputs give finite results next to the input, satfinite saturation, and
 * different entropy gives different roundings.
 * Replaces tlx.stoch_round(src, dst_ty, rand_bits) (utility.py:113-153).
 */
B2X_API b2x_status b2x_stoch_round_rs(const float* x, int64_t rows, int64_t cols, int64_t ld_x, const uint32_t* rbits,
                                      int64_t ld_r, void* y, b2x_dtype y_type, int64_t ld_y, void* stream);

/* ------------------------------------------------------------------ GEMM */

/*
 * Tile / pipeline configuration.  Same keys as the reference's config dict
 * (blackwell_gemm_ws.py:1097-1109); zero means "pick".  NUM_MMA_GROUPS,
 * NUM_CTAS and INTERLEAVE_EPILOGUE are accepted for drop-in compatibility.
 * Each CTA owns 128 rows of the output tile.  num_ctas = 2 runs the paired
 * kernel: two CTAs of a cluster share 256 x 256 tiles through cta_group::2
 * MMAs (each loads its own half of A and of B, no multicast); num_ctas = 1
 * runs single-CTA 128 x block_n tiles; 0 lets the library choose.
 */
typedef struct {
  int block_m, block_n, block_k;
  int group_size_m;
  int num_smem_buffers, num_tmem_buffers;
  int num_mma_groups, epilogue_subtile;
  int num_ctas, split_k, interleave_epilogue; /* split_k = -1: stream-K for M <= 64 (decode): the K blocks of all
                                                  tiles are cut into equal ranges, one per SM; partials are reduced
                                                  like split-K (same workspace) */
  int num_sms; /* NUM_SMS: at most this many SMs for the persistent grid (0 = all); leaves SMs free for concurrent work such as NCCL */
} b2x_gemm_config;

/*
 * C[M,N] = out_cast( sum_k A[m,k] * B[k,n] * scales )
 *   A: fp8 [M,K], row stride lda (elements), K contiguous.
 *   B: fp8, logical [K,N] as in the reference (b.shape == (K, N)); strides
 *      (ldb_k, ldb_n) with exactly one of them equal to 1:
 *        ldb_k == 1  -> B stored "K-major" (an nn.Linear weight [N,K] viewed as w.t())
 *        ldb_n == 1  -> B stored row-major [K,N]
 *   C: bf16 / fp16 / fp32 [M,N], row stride ldc.
 * Scales (fp32, device pointers):
 *   B2X_SCALE_NONE:   none;
 *   B2X_SCALE_TENSOR / _GIVEN: scale_a[0], scale_b[0]   -> C = sA*sB*(A.B)
 *   B2X_SCALE_BLOCK_1x128 (A) with 128x128 (B): scale_a[m, kb] at
 *      scale_a + m*sa_stride_m + kb*sa_stride_k, scale_b[kb, nb] at
 *      scale_b + kb*sb_stride_k + nb*sb_stride_n; promotion per 128-deep
 *      K block: C = sum_kb sA[m,kb]*sB[kb,nb]*(A_kb.B_kb).
 *   B2X_SCALE_MX_1x32: uint8 E8M0 scales, one per 32 K elements: scale_a
 *      [M, K/32] with row stride sa_stride_m bytes, scale_b [N, K/32] (per
 *      row of the [N, K] weight) with row stride sb_stride_n bytes:
 *      C = sum_j 2^(sA[m,j]-127) * 2^(sB[n,j]-127) * (A_j . B_j), applied by
 *      the tensor core (tcgen05 kind::mxf8f6f4.block_scale).  Needs K-major B,
 *      K % 128 == 0, 4-byte aligned scale rows, and a workspace of
 *      b2x_gemm_workspace_size bytes (any content; it receives the scales
 *      re-tiled for the kernel).  Replaces async_dot_scaled with E8M0 scales
 *      (extensions/utlx/python/utlx_plugin/mma_ops.py:163-237).
 * Split-K (config.split_k > 1): fp32 partials are reduced with
 * red.global.add.v4.f32 into a workspace; the last CTA to finish a tile
 * writes C.  The workspace must be all zero on the first call and is left all
 * zero by every successful call (so it can be cached and reused on one
 * stream); see b2x_gemm_workspace_size.
 * Replaces: matmul(a, b, config, use_heuristic) blackwell_gemm_ws.py:1352-1483
 * together with its kernel (:1089-1349) and split-K reduce (:1033-1079).
 */
typedef struct {
  const void* a;
  const void* b;
  void* c;
  int64_t M, N, K;
  int64_t lda;
  int64_t ldb_k, ldb_n;
  int64_t ldc;
  b2x_dtype a_type, b_type, c_type;
  b2x_scale_mode scale_mode;
  const float* scale_a;
  int64_t sa_stride_m, sa_stride_k;
  const float* scale_b;
  int64_t sb_stride_k, sb_stride_n;
  void* workspace;
  size_t workspace_bytes;
  b2x_gemm_config config;
} b2x_gemm_args;

/* Fill in a config for the shape (the counterpart of get_heuristic_config,
 * blackwell_gemm_ws.py:24-341).  Fields the caller set to non-zero are kept. */
B2X_API b2x_status b2x_gemm_default_config(const b2x_gemm_args* args, b2x_gemm_config* out);
B2X_API size_t b2x_gemm_workspace_size(const b2x_gemm_args* args);
B2X_API b2x_status b2x_fp8_gemm(const b2x_gemm_args* args, void* stream);

/*
 * Reference-compatible split-K reduce: c[m,n] = cast(sum_s ws[s*M + m, n]),
 * summed in fp32.  ws is [split_k*M, N] of ws_type (row stride N), c is
 * [M,N] of c_type (row stride ldc).
 * Replaces: _reduce_k_kernel, blackwell_gemm_ws.py:1033-1056.
 */
B2X_API b2x_status b2x_splitk_reduce(const void* ws, b2x_dtype ws_type, void* c, b2x_dtype c_type, int64_t M, int64_t N,
                             int64_t ldc, int split_k, void* stream);

/*
 * Same GEMM as b2x_fp8_gemm (per-tensor or no scales, split-K included) on
 * single-CTA 128 x BLOCK_SIZE_N tiles, scheduled by cluster launch control
 * instead of a persistent grid: the grid has one CTA per output tile (per
 * split), each CTA starts with its own tile and then takes over the tiles of
 * CTAs that have not launched yet (clusterlaunchcontrol.try_cancel), so work
 * moves to the SMs that are free -- the reference's
 * matmul_kernel_tma_ws_blackwell_clc with its host matmul
 * (extensions/utlx/tlx/tutorials/blackwell_gemm_clc.py:62-281, :281; CLC
 * primitives tlx/language/tlx/dynamic_launch.py:35-96).  Block / MX scales
 * give B2X_ERR_UNSUPPORTED.
 */
B2X_API b2x_status b2x_fp8_gemm_clc(const b2x_gemm_args* args, void* stream);

/*
 * Same GEMM as b2x_fp8_gemm, for callers that cannot allocate device memory
 * (a serving loop that reserves all memory up front, a plugin running inside
 * another framework's memory pool, a host with no allocator behind its C
 * interface).  It takes no workspace: split-K partial sums go to a scratch
 * array built into the library (8 MiB per device, held until the process
 * exits), so M*N*4 must stay below about 8 MiB; larger split-K problems are
 * rejected with B2X_ERR_WORKSPACE.  It calls no allocator.  All calls on a
 * device share the scratch: each call clears what it uses first, and calls
 * that overlap on the GPU (unordered streams) race.  The first call on a
 * device looks up the scratch address; make it before any stream capture.
 * No counterpart in the reference (which always allocates its split-K
 * workspace with torch.empty).
 */
B2X_API b2x_status b2x_fp8_gemm_splitk_noalloc(const b2x_gemm_args* args, void* stream);

/* ------------------------------------------------------------ gate+up GEMM with SwiGLU */

/*
 * The gate+up projection of a gated MLP fused with SwiGLU and the fp8
 * quantization of its output:
 *   [g | u] = A . B^T * scales   (B: the K-major [2I, K] weight whose rows are
 *                                 gate rows 128j..128j+127 followed by up rows
 *                                 128j..128j+127, j = 0 .. I/128 - 1)
 *   h       = g / (1 + exp(-g)) * u                       (fp32, [M, I])
 *   q       = fp8_rne_satfinite(clamp(h / s, -FMAX, FMAX)) written to h (row stride ld_h)
 * with s either
 *   B2X_SCALE_BLOCK_1x128:  one fp32 scale per (row, 128 columns of h),
 *                           s = amax / FMAX, written to h_scale [M, I/128]
 *                           (row stride ld_h_scale) -- the A operand scales of
 *                           the block-scaled down projection;
 *   B2X_SCALE_MX_1x32:      one E8M0 byte per (row, 32 columns of h): the
 *                           reference's _to_mxfp8_block recipe (mxfp8_utils.py:
 *                           89-128: amax / FMAX rounded up to a power of two),
 *                           written to h_scale as uint8 [M, I/32] (row stride
 *                           ld_h_scale bytes, a multiple of 4; 4-byte aligned
 *                           base) -- the A operand scales of an MX down
 *                           projection;
 *   B2X_SCALE_TENSOR_GIVEN: *h_scale supplied by the caller (delayed scaling);
 *                           if h_amax is not NULL, max |h| is max-reduced into
 *                           *h_amax (which the caller zeroes before the call).
 * args is the gate+up GEMM as for b2x_fp8_gemm (per-tensor scales or none;
 * args->c and c_type are ignored; N = 2I must be a multiple of 256).  The
 * [M, 2I] product never leaves the chip.  No counterpart in the reference: it
 * composes the GEMM epilogue (blackwell_gemm_ws.py:673-824) with the quantize
 * recipe (mxfp8_utils.py:37-84).
 */
B2X_API b2x_status b2x_fp8_gemm_swiglu(const b2x_gemm_args* args, void* h, int64_t ld_h, b2x_dtype h_type,
                                       b2x_scale_mode h_mode, float* h_scale, int64_t ld_h_scale, float* h_amax,
                                       void* stream);

/* ------------------------------------------------------------ grouped GEMM */

/*
 * Grouped fp8 GEMM: for every group g, C_g = sA_g * sB_g * (A_g . B_g^T) with
 * A_g [M_g, K_g] (row stride lda), B_g the K-major [N_g, K_g] weight (row
 * stride ldb) and C_g [M_g, N_g] bf16/fp16 (row stride ldc), all in one
 * persistent launch.  Per-tensor scales are device pointers (both NULL: 1).
 * Groups with M or N zero are skipped.  The workspace (64-byte aligned,
 * b2x_grouped_gemm_workspace_size bytes) receives the group descriptors,
 * copied from host memory on `stream` before the launch (so a call cannot be
 * captured into a CUDA graph).  block_n: 0 picks 256 unless no group is wider
 * than 128 columns.
 * Replaces the reference's grouped GEMM, grouped_matmul_tlx_kernel with
 * group_gemm_tlx_fn (extensions/utlx/tlx/tutorials/blackwell-grouped-gemm_test.py:366-784).
 */
typedef struct {
  const void* a;
  const void* b;
  void* c;
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  const float* scale_a;
  const float* scale_b;
} b2x_gemm_group;

B2X_API size_t b2x_grouped_gemm_workspace_size(int num_groups);
B2X_API b2x_status b2x_fp8_grouped_gemm(const b2x_gemm_group* groups, int num_groups, b2x_dtype a_type,
                                        b2x_dtype b_type, b2x_dtype c_type, int block_n, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ GEMM + all-reduce */

/*
 * Row-parallel fp8 GEMM fused with the sum over the GPUs of one node:
 *   C = sum over ranks r of ( A_r . B_r * scales_r ),  bf16 [M, N] on every rank,
 * where each rank passes its own K-slice A_r [M, K/world] and B_r.  The ranks'
 * partial tiles are summed while the GEMM runs (each 128 x 256 output unit is
 * reduced by the last rank to finish it, through NVSwitch multicast or peer
 * loads/stores over NVLink), so no separate collective follows.
 *
 * The GEMM arguments are those of b2x_fp8_gemm with these limits: scale mode
 * NONE / TENSOR / TENSOR_GIVEN, K-major B, bf16 C, M and N multiples of 256,
 * ldc a multiple of 8.  `args->c` must be this rank's copy of a buffer every
 * rank can reach (c_peers[rank]); the result overwrites it on every rank.
 * The signal buffer (b2x_allreduce_signal_words 32-bit words per rank, all
 * zero before the first call) carries the arrival and completion counts.
 * Every rank must make the same sequence of calls (same shapes, same
 * buffers).  Calls are counted either by the caller, passing epoch = 1 on the
 * first call after zeroing the signal buffer and one more on each later call
 * (modulo 2^32, skipping 0), or, with epoch = 0 on every call, by the kernel
 * itself in the signal buffer; the second form has no per-call argument, so
 * the launch can be captured once in a CUDA graph and replayed.  The kernel
 * ends when the sum is complete on this rank; a peer that never takes part
 * makes it give up after 10 s with B2X_ERR_TIMEOUT recorded in the device
 * status word, after which the signal buffers must be zeroed on every rank
 * (and caller-kept epochs restarted) before the next call.
 * No counterpart in the reference, which has no multi-GPU code path; it
 * replaces, for the tensor-parallel layer set, a GEMM followed by an NCCL
 * all-reduce of its output.
 */
#define B2X_AR_MAX_RANKS 8
typedef struct {
  int rank, world;                      /* 1 <= world <= B2X_AR_MAX_RANKS */
  void* c_multicast;                    /* multicast address of C's buffer, or NULL for peer mode */
  void* c_peers[B2X_AR_MAX_RANKS];      /* C's buffer on each rank, as mapped in this process */
  void* signal_multicast;               /* multicast address of the signal buffer (with c_multicast) */
  void* signal_peers[B2X_AR_MAX_RANKS]; /* the signal buffer on each rank */
  uint32_t epoch;                       /* 1, 2, 3, ... per call, or 0 on every call: counted on the device */
} b2x_allreduce_args;

B2X_API size_t b2x_allreduce_signal_words(int64_t M, int64_t N);
B2X_API b2x_status b2x_fp8_gemm_allreduce(const b2x_gemm_args* args, const b2x_allreduce_args* ar, void* stream);

/* ------------------------------------------------------------------ misc */

/* Message for the calling thread's last failed call ("" if none). */
B2X_API const char* b2x_last_error(void);
/* Reads and clears the device status word of the current device (blocking). */
B2X_API b2x_status b2x_read_device_status(int* status_out);
/*
 * Reads and clears the device status word (blocking) and returns
 * B2X_ERR_TIMEOUT, with a message naming the role whose wait gave up, when
 * a kernel abandoned a bounded wait since the last read; B2X_OK otherwise.
 * No counterpart in the reference (whose Triton kernels have no bounded
 * waits).
 */
B2X_API b2x_status b2x_check_device(void);
/*
 * Test hook for the bounded-wait failure path (current device; off by
 * default).  what = 1: the next paired-CTA GEMMs have their MMA warp withhold
 * the accumulator-ready signal of its first tile, so the epilogue's wait runs
 * out; the kernel records 0x103 in the status word and returns early, with no
 * fault or trap.  what = 0: normal operation.  wait_timeout_ns sets the limit
 * of every bounded mbarrier wait (0 = the default 2 s).  A test restores
 * (0, 0) when done.  No counterpart in the reference.
 */
B2X_API b2x_status b2x_debug_inject(int what, uint64_t wait_timeout_ns);
/*
 * Wait-cycle trace of the last GEMM launches (diagnostics).  When the
 * environment variable B2X_TRACE=1 is set at the first GEMM call, every GEMM
 * kernel adds, per CTA, clock cycles and counts into 16 counters: [0]
 * producer waiting for a free stage, [1] MMA waiting for loaded data, [2] MMA
 * waiting for a free accumulator, [3]/[4] epilogue warpgroup 0/1 waiting for
 * an accumulator, [5] CTA lifetime, [6] MMA issue (from data ready to
 * commit), [7] tiles or K blocks processed; for b2x_fp8_gemm_allreduce also
 * [8] reducing owned units, [9] waiting for peers' partials, [10]/[11] units
 * reduced inside / after the tile loop, [12] the final wait for every rank's
 * reductions, [13] tile-loop end to end of the remaining reductions.
 * Copies max_ctas x 16 counters to `out` (blocking) and clears them.
 * Counterpart of the reference's clock64-based timing (tlx.clock64,
 * extensions/utlx/tlx/language/tlx/utility.py:108).
 */
B2X_API b2x_status b2x_trace_read(uint64_t* out, int max_ctas, int* n_ctas);
/* ABI version of the loaded library (B2X_ABI_VERSION). */
B2X_API int b2x_abi_version(void);
/* Number of kernels this library launched since load (all devices). */
B2X_API uint64_t b2x_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* B2X_H_ */
