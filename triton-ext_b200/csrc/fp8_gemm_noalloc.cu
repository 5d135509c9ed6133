// Split-K fp8 GEMM that allocates nothing: the fp32 partial sums and the
// per-tile arrival counters live in a fixed array of device memory that the
// library itself carries, instead of a caller-provided workspace.
//
// Who needs this: code that may not call cudaMalloc (or any allocator) at the
// point where it runs the GEMM -- for example a serving loop that reserves
// all device memory up front and forbids later allocations, a plugin that
// runs inside another framework's memory pool, or a host that calls through
// a plain C interface with no access to an allocator.  The caller still owns
// and passes A, B, C and the scales.
//
// Limits and sharing:
//   * The scratch array holds at most kNoAllocScratchBytes (8 MiB): the split-K
//     sum needs M*N*4 bytes rounded up to 256, plus 4 bytes per output tile
//     rounded up to 256.  Larger requests are rejected with
//     B2X_ERR_WORKSPACE and a message; nothing is launched.
//   * Every device that loads the library keeps the 8 MiB until the process
//     exits.
//   * All calls on a device share the one array.  Each call clears the part it
//     uses (cudaMemsetAsync on the given stream) before the GEMM, so a call
//     never depends on what an earlier call left there.  Calls whose work
//     overlaps on the GPU (different streams, no ordering between them) race
//     on the array and produce wrong results; order them on one stream.
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make that
//     first call before any stream capture begins.
#include <cuda_runtime.h>
#include <mutex>
#include "b2x_internal.h"

namespace b2x {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kNoAllocMaxDevices = 64;

// The scratch array.  Host code must not pass `g_noalloc_scratch` itself to
// a kernel: on the host it names a stand-in object, not device memory.  The
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
static cudaError_t noalloc_scratch_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace b2x

extern "C" B2X_API b2x_status b2x_fp8_gemm_splitk_noalloc(const b2x_gemm_args* args, void* stream) {
  using namespace b2x;
  if (!args) return fail(B2X_ERR_INVALID_ARG, "b2x_fp8_gemm_splitk_noalloc: args is NULL");
  b2x_gemm_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  const size_t need = b2x_gemm_workspace_size(&a);
  if (need > kNoAllocScratchBytes)
    return fail(B2X_ERR_WORKSPACE,
                "b2x_fp8_gemm_splitk_noalloc: this problem needs %zu bytes of split-K scratch; the built-in "
                "scratch holds %zu bytes (M*N*4 must stay below about 8 MiB)",
                need, kNoAllocScratchBytes);
  if (need > 0) {
    void* p = nullptr;
    cudaError_t e = noalloc_scratch_ptr(&p);
    if (e != cudaSuccess) return cuda_fail(e, "b2x_fp8_gemm_splitk_noalloc: cudaGetSymbolAddress");
    e = cudaMemsetAsync(p, 0, need, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "b2x_fp8_gemm_splitk_noalloc: clearing the scratch");
    a.workspace = p;
    a.workspace_bytes = kNoAllocScratchBytes;
  }
  return b2x_fp8_gemm(&a, stream);
}
