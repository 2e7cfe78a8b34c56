// mhc_bwd_noalloc: the fused layer backward (mhc_bwd + mhc_bwd_finalize)
// for callers that cannot allocate device memory, e.g. a plugin boundary
// that passes a kernel only its inputs and outputs.  The per-block partial
// sums go to a file-scope device array instead of a caller workspace.
//
// Contract (also stated in include/mhc_b200.h):
//  - The array is MHC_NOALLOC_SCRATCH_BYTES (16 MiB); every GPU that loads
//    the library holds it until the process exits.  Sizes whose workspace
//    (mhc_bwd_workspace_bytes) exceeds it are rejected with MHC_ERR_WORKSPACE.
//  - Nothing in the array has to start at zero: the backward kernel writes
//    the row count and every partial row it uses before the finalize reads
//    them, in the same call.  Stale contents of a previous call are ignored.
//  - All calls share the array: calls that overlap on the GPU race.
//  - The first call on a device resolves the array's device address with
//    cudaGetSymbolAddress (once per device, with that device current); make
//    that first call before any stream capture.  A first call whose lookup
//    failed returns MHC_ERR_CUDA and can be retried.
//  - No cudaMalloc / cudaFree or allocating library routine is called.
#include <mutex>

#include "mhc_common.cuh"
#include "mhc_internal.h"

namespace mhc {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MHC_NOALLOC_SCRATCH_BYTES];

static constexpr int kMaxDev = 64;
static void* g_scratch_addr[kMaxDev];  // non-null once resolved on that device
static std::mutex g_scratch_mu[kMaxDev];

// Device address of the array on the current device.  In host code
// g_noalloc_scratch names a host-side stand-in, never a device address.
// Only a successful lookup is remembered: a lookup that fails (for example
// one attempted during stream capture) is retried by the next call, and its
// error is cleared from the runtime's last-error slot so that it is not
// reported again by a later, unrelated launch check.
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(MHC_ERR_CUDA, "mhc_bwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDev) return set_error(MHC_ERR_UNSUPPORTED, "mhc_bwd_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu[dev]);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t r = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (r != cudaSuccess || !p) {
      (void)cudaGetLastError();
      return set_error(MHC_ERR_CUDA, "mhc_bwd_noalloc: cudaGetSymbolAddress failed: %s "
                       "(the call can be retried)", cudaGetErrorString(r));
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return MHC_OK;
}

}  // namespace mhc

using namespace mhc;

extern "C" int mhc_bwd_noalloc(const void* x, int x_dtype, const void* d_out, int dout_dtype,
                               const float* M, const float* H_pre_act, const float* H_post_act,
                               const float* rms_weight, void* dx, int dx_dtype, float* dM,
                               float* dH_pre_act, float* dH_post_act, float* d_rms_weight,
                               int64_t T, int n, int C, float eps, void* stream) {
  try {
    if (n < 1 || n > 64) return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: n=%d must be in [1, 64]", n);
    if (C < 1) return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: C=%d must be positive", C);
    if (T < 0) return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: T=%lld must be >= 0", (long long)T);
    if (!dtype_ok(x_dtype) || !dtype_ok(dout_dtype) || !dtype_ok(dx_dtype))
      return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: dtype not one of MHC_F32/F16/BF16");
    if (!M || !H_pre_act || !H_post_act || !rms_weight)
      return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: NULL parameter pointer");
    if (!dM || !dH_pre_act || !dH_post_act || !d_rms_weight)
      return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: NULL gradient pointer");
    if (T > 0 && (!x || !d_out || !dx))
      return set_error(MHC_ERR_INVALID, "mhc_bwd_noalloc: NULL x/d_out/dx");
    const size_t need = bwd_ws_bytes(T, n, C);
    if (need > MHC_NOALLOC_SCRATCH_BYTES)
      return set_error(MHC_ERR_WORKSPACE,
                       "mhc_bwd_noalloc: T=%lld n=%d C=%d needs %zu bytes of partials, above the "
                       "fixed %zu-byte scratch; use mhc_bwd with a caller workspace",
                       (long long)T, n, C, need, (size_t)MHC_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    int r = scratch_address(&scratch);
    if (r != MHC_OK) return r;
    cudaStream_t st = as_stream(stream);
    r = launch_bwd(x, x_dtype, d_out, dout_dtype, M, H_pre_act, H_post_act, rms_weight, dx,
                   dx_dtype, T, n, C, eps, scratch, MHC_NOALLOC_SCRATCH_BYTES, st);
    if (r != MHC_OK) return r;
    return launch_finalize(scratch, n, C, dM, dH_pre_act, dH_post_act, d_rms_weight, nullptr,
                           nullptr, nullptr, nullptr, 0, eps, nullptr, nullptr, nullptr, st);
  } catch (...) {
    return set_error(MHC_ERR_CUDA, "mhc_bwd_noalloc: unexpected C++ exception");
  }
}
