// Device-side primitives for the sm_100a kernels of b2x: mbarriers with
// bounded waits, TMA tiled loads/stores, tcgen05 (TMEM alloc, MMA, commit,
// loads) and the fp8 conversions.
//
// These are the native counterparts of the TLX builtins the reference GEMM is
// written in:
//   alloc_barriers / barrier_expect_bytes / barrier_wait / barrier_arrive
//     (extensions/utlx/python/utlx_plugin/barrier.py:23-161)
//   async_descriptor_load / async_descriptor_store / store_wait
//     (extensions/utlx/python/utlx_plugin/mem_ops.py:750-863)
//   async_dot / tcgen05_commit (extensions/utlx/python/utlx_plugin/mma_ops.py:86-265)
//   local_alloc(storage=tmem) (mem_ops.py:103)
// Every wait is bounded: after B2X_WAIT_TIMEOUT_NS of wall time the waiting
// thread records an error in the device status word and the caller unwinds
// without trapping (no __trap, no assert).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#ifndef B2X_WAIT_TIMEOUT_NS
#define B2X_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: every legitimate wait is < 1 ms
#endif

namespace b2x {

// Device status word: 0 = ok, otherwise a code saying where a wait gave up.
// One per module per device; read back with b2x_read_device_status().
// (libb2x is built as a single translation unit, so this header is the definition.)
__device__ int g_status = 0;

// Wait limit of mbar_wait in ns (B2X_WAIT_TIMEOUT_NS unless a test lowers it
// through b2x_debug_inject), and the test-only fault switch: 1 = the paired
// GEMM's MMA warp withholds the accumulator-ready commit of its first tile, so
// the epilogue's bounded wait runs out (no fault, no trap: the kernel unwinds).
__device__ unsigned long long g_wait_ns = B2X_WAIT_TIMEOUT_NS;
__device__ int g_inject = 0;

enum : int {
  kStatusOk = 0,
  kStatusTimeoutProducer = 0x101,
  kStatusTimeoutMma = 0x102,
  kStatusTimeoutEpilogue = 0x103,
  kStatusTimeoutSplitK = 0x104,
  kStatusTimeoutAllReduce = 0x105,  // a peer GPU never finished its share of a fused all-reduce
  kStatusTimeoutCast = 0x106,       // a staged cast kernel's load never completed
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %laneid;" : "=r"(r));
  return r;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on the phase with the given parity. `abort` is a shared flag
// that any role sets when it gives up, so the other roles stop waiting too.
// Returns false when the wait was abandoned.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer() - start > g_wait_ns) {
        *abort = 1;
        atomicCAS(&g_status, 0, code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- cluster launch control
// Asks the hardware to cancel one not-yet-launched cluster of this grid; the
// 16-byte response lands in `resp` (shared, 16-byte aligned) and completes
// 16 bytes of transaction count on `bar`.  No multicast.
__device__ __forceinline__ void clc_try_cancel(void* resp, uint64_t* bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(
          smem_u32(resp)),
      "r"(smem_u32(bar))
      : "memory");
}

// x index of the first CTA of the cluster a response cancelled, or -1 when
// the request found no cluster left to cancel.
__device__ __forceinline__ int clc_first_ctaid_x(const void* resp) {
  int x, ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b128 r;\n\t"
      "ld.shared.b128 r, [%2];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "selp.u32 %1, 1, 0, p;\n\t"
      "mov.u32 %0, 0xffffffff;\n\t"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, r;\n\t}"
      : "=r"(x), "=r"(ok)
      : "r"(smem_u32(resp))
      : "memory");
  return ok ? x : -1;
}

// ---------------------------------------------------------------- tracing
// Optional per-CTA cycle counters (enabled per launch by B2X_TRACE=1 on the
// host; read back with b2x_trace_read).  Slots:
//   0 producer waiting for a free stage     1 MMA waiting for loaded data
//   2 MMA waiting for a free accumulator    3 epilogue WG0 waiting for data
//   4 epilogue WG1 waiting for data         5 CTA lifetime (thread 0)
//   6 MMA issue (data ready to commit)      7 units processed by the CTA
// and, for the fused GEMM + all-reduce (paired kernel; its reducer warpgroup):
//   8 reducing owned units                  9 waiting for peers' arrivals
//  10 units reduced                        12 final wait for every rank's reductions
//  13 reducer lifetime up to the final wait
constexpr int kTraceSlots = 16;
constexpr int kTraceMaxCtas = 512;
__device__ unsigned long long g_trace[kTraceMaxCtas * kTraceSlots];

__device__ __forceinline__ void trace_add(int on, int slot, unsigned long long v) {
  if (on && blockIdx.x < kTraceMaxCtas) atomicAdd(&g_trace[blockIdx.x * kTraceSlots + slot], v);
}

// Bounded wait that also adds the cycles it spent to trace slot `slot`.
__device__ __forceinline__ bool mbar_wait_traced(uint64_t* bar, uint32_t parity, volatile int* abort, int code,
                                                 int trace, int slot) {
  if (!trace) return mbar_wait(bar, parity, abort, code);
  const long long t0 = clock64();
  const bool ok = mbar_wait(bar, parity, abort, code);
  trace_add(1, slot, (unsigned long long)(clock64() - t0));
  return ok;
}

// Named barrier among `count` threads (multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Two independent fp32 FMAs in one instruction (sm_100 paired FP32):
// a0 = fma(x0, s, a0), a1 = fma(x1, s, a1), each rounded like fmaf.
__device__ __forceinline__ void fma2_scalar(float& a0, float& a1, float x0, float x1, float s) {
  asm("{\n\t.reg .b64 ra, rx, rs;\n\t"
      "mov.b64 ra, {%0, %1};\n\t"
      "mov.b64 rx, {%2, %3};\n\t"
      "mov.b64 rs, {%4, %4};\n\t"
      "fma.rn.f32x2 ra, rx, rs, ra;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(s));
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled load global -> shared, completion counted on `bar` in bytes.
// x is the innermost coordinate (elements); callers keep x*elem_size % 16 == 0.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int32_t x, int32_t y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 3-D tiled load (x innermost), completion counted on `bar` in bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int32_t x, int32_t y,
                                            int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// 2-D tiled store shared -> global (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0),
// completion counted on `bar` in bytes.  No multicast.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                             uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one whole warp; the TMEM base address is
// written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f8f6f4, issued by one thread.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05 ops of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Warp-collective TMEM -> registers: 32 lanes x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Warp-collective TMEM -> registers: 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Orders later uses of r after the preceding tmem_ld_wait(): the registers
// pass through an empty volatile asm, so no read of them can be scheduled
// before the wait (used where several loads are in flight).
__device__ __forceinline__ void tmem_regs_after_wait(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}

// Shared-memory matrix descriptor (sm_100 "version 1" format) for a tile stored
// in the canonical 128-byte-swizzled layout: rows of 128 bytes, 8-row atoms of
// 1024 bytes. `sbo` is the byte distance between 8-row groups (K-major) or
// between 8-column groups (MN-major); `lbo` the byte distance between swizzle
// atoms along the leading dimension (only meaningful for MN-major).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f8f6f4 with an fp32 accumulator.
// fmt: 0 = e4m3, 1 = e5m2. major: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t idesc_f8f6f4(uint32_t a_fmt, uint32_t b_fmt, uint32_t a_major,
                                                    uint32_t b_major, uint32_t M, uint32_t N) {
  return (1u << 4)                 // D format: F32
         | (a_fmt << 7) | (b_fmt << 10) | (a_major << 15) | (b_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}


// ---------------------------------------------------------------- CTA pairs (cluster of 2)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same smem offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Relaxed arrive on a (possibly peer) mbarrier: for releasing TMEM buffers,
// where the only prior work to order is TMEM reads already completed by
// tcgen05.wait::ld and fenced with tcgen05.fence::before_thread_sync.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arrive on an mbarrier given by a shared::cluster address (possibly in the peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D tiled load into this CTA's smem whose completion is counted on an
// mbarrier of either CTA of the pair (cta_group::2 form; no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster_addr,
                                                 int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster_addr), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Paired MMA: issued by one thread of the even CTA; A and B come from the
// same smem offsets in both CTAs (A split along M, B split along N).
__device__ __forceinline__ void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at this smem offset in every CTA of `mask`
// when the issuing thread's paired MMAs complete.
__device__ __forceinline__ void mma_commit_pair_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// ---------------------------------------------------------------- conversions
// Two fp32 -> two fp8 with round-to-nearest-even and saturation to the largest
// finite value; `lo` lands in the low byte.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint16_t cvt_e5m2x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void red_add_f32(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

// Vectorised split-K reduction: four fp32 adds in one global reduction.
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// ---------------------------------------------------------------- cross-GPU (NVLink / NVSwitch)
// Peer pointers are another GPU's memory mapped into this process; multicast
// pointers address the same offset on every GPU of an NVLink multicast group
// (the NVSwitch replicates stores and reduces loads).  Only plain loads,
// stores, atomics and multimem operations touch such memory here; no TMA
// load ever reads it.

// Make this thread's earlier async-proxy (TMA) global writes and generic
// writes visible at system scope before a following release.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ uint32_t atom_add_acq_rel_sys(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.sys.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.add.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Adds v to the word at this multicast address on every GPU of the group.
__device__ __forceinline__ void multimem_red_add_release_sys(uint32_t* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}
// Sum over the group of eight bf16 values (16 bytes) at this multicast
// address, accumulated in fp32 by the switch and returned as bf16.
__device__ __forceinline__ uint4 multimem_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
// Stores 16 bytes at this multicast address on every GPU of the group.
__device__ __forceinline__ void multimem_st_16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Bounded wait until the counter at p reaches `target` (wrap-around compare);
// on timeout records kStatusTimeoutAllReduce and returns false.
__device__ __forceinline__ bool wait_counter_sys(const uint32_t* p, uint32_t target, uint64_t timeout_ns) {
  uint64_t start = globaltimer();
  for (;;) {
    if ((int32_t)(ld_acquire_sys(p) - target) >= 0) return true;
    if (globaltimer() - start > timeout_ns) {
      atomicCAS(&g_status, 0, kStatusTimeoutAllReduce);
      return false;
    }
    __nanosleep(128);
  }
}

}  // namespace b2x
