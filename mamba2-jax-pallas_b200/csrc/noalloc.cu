// ssd_combined_fwd_noalloc: the combined SSD forward with its scratch memory in a
// file-scope device array instead of a caller-provided workspace.
//
// For callers that cannot allocate device memory at the point where they run the SSD
// forward: for example a handler registered with a framework that hands it only the
// input/output buffers and a stream (no scratch-buffer slot), or code that runs while
// another component forbids cudaMalloc/cudaFree (which synchronise the device and are
// not allowed inside a stream capture).  They pass inputs and outputs only.
//
// Limits and sharing:
//   - The scratch is SSD_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU, reserved when this code
//     is loaded onto that GPU (at the latest, by the first call there) and held until the
//     process exits.  Calls whose workspace need
//     (ssd_combined_workspace_bytes) exceeds it are rejected with SSD_ERR_WORKSPACE.
//   - Every call on a device uses the same array, which keeps the previous call's
//     contents.  The kernels overwrite every scratch byte they read, and the status word
//     they check is cleared on the stream at the start of each call.  Calls that overlap
//     on the GPU (different streams, no ordering between them) race on the array.
//   - The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current).  Make that first call before any
//     stream capture begins.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "ssd_b200.h"
#include "ssd_kernels.h"

namespace {

// The scratch itself.  In host code this name is only a stand-in for the symbol; the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SSD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices] = {};

thread_local char g_err_local[256];

}  // namespace

extern "C" {

int ssd_combined_fwd_noalloc(const ssd_fwd_params_t* p, ssd_stream_t stream) {
  if (!p) {
    ssd::set_last_error("params is NULL");
    return SSD_ERR_INVALID_ARG;
  }
  const size_t need = ssd_combined_workspace_bytes(p);
  // 0: the params are invalid; the workspace entry point reports why before touching
  // any buffer
  if (need == 0) return ssd_combined_fwd(p, nullptr, 0, stream);
  if (need > (size_t)SSD_NOALLOC_SCRATCH_BYTES) {
    snprintf(g_err_local, sizeof(g_err_local),
             "ssd_combined_fwd_noalloc: these shapes need %zu bytes of scratch, more than the %d-byte "
             "static scratch; use ssd_combined_fwd with a caller-provided workspace",
             need, SSD_NOALLOC_SCRATCH_BYTES);
    ssd::set_last_error(g_err_local);
    return SSD_ERR_WORKSPACE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    ssd::set_last_error("ssd_combined_fwd_noalloc: no current CUDA device");
    return SSD_ERR_CUDA;
  }
  void* ptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ptr[dev]) {
      void* q = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
      if (e != cudaSuccess || !q) {
        snprintf(g_err_local, sizeof(g_err_local), "ssd_combined_fwd_noalloc: cudaGetSymbolAddress: %s",
                 cudaGetErrorString(e));
        ssd::set_last_error(g_err_local);
        return SSD_ERR_CUDA;
      }
      g_ptr[dev] = q;
    }
    ptr = g_ptr[dev];
  }
  return ssd_combined_fwd(p, ptr, (size_t)SSD_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
