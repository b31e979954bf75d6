// m3_scan_bwd_noalloc: the analytic backward with its scratch taken from a
// buffer that lives inside this library instead of from the caller.
//
// Who needs it: callers that cannot allocate device memory at the point where
// they run the backward -- for example a process whose HBM is carved up once at
// start-up by another allocator it has no handle to (an FFI caller of this C
// ABI), or a latency-critical loop that must not call cudaMalloc because it can
// synchronise the device or fail under a fixed memory budget.  Such a caller
// still passes its inputs and outputs; only the backward's partial-sum scratch
// (the workspace m3_scan_bwd normally receives) comes from here.
//
// The buffer is a file-scope device array of M3_NOALLOC_SCRATCH_BYTES.  Every
// GPU that loads this library's module keeps it for the life of the process.
// Host code may not use the array's name as a device address (it is a host-side
// stand-in), so the first call on each device looks the address up with
// cudaGetSymbolAddress while that device is current, checks the result and
// caches it; later calls on the device reuse the cached address.  The cache is
// never invalidated: after a reset of the device's primary context
// (cudaDeviceReset) in the same process the cached address is stale, so the
// entry point must not be used after such a reset.
#include <cuda_runtime.h>

#include <mutex>

#include "m3scan.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[M3_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return M3_ERR_NO_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return M3_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return M3_ERR_LAUNCH;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return M3_OK;
}

}  // namespace

extern "C" int m3_scan_bwd_noalloc(const m3_scan_desc* desc, const void* delta, const void* u,
                                   const void* Bc, const void* Cc, const float* A_real_p,
                                   const float* A_imag_p, const float* track_p, const void* dy,
                                   int32_t dtype_dy, const float* ckpt, void* d_delta, void* d_u,
                                   void* d_Bc, void* d_Cc, float* d_A_real_p,
                                   float* d_A_imag_p, float* d_track_p, void* stream) {
  if (!desc) return M3_ERR_NULL;
  const size_t need = m3_scan_bwd_workspace_bytes(desc);
  if (need == 0) {
    // invalid descriptor or no backward kernel: let the regular entry point
    // report the precise status (it fails before touching any workspace)
    return m3_scan_bwd(desc, delta, u, Bc, Cc, A_real_p, A_imag_p, track_p, dy, dtype_dy, ckpt,
                       d_delta, d_u, d_Bc, d_Cc, d_A_real_p, d_A_imag_p, d_track_p, nullptr, 0,
                       stream);
  }
  if (need > (size_t)M3_NOALLOC_SCRATCH_BYTES) return M3_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != M3_OK) return rc;
  // Nothing in the scratch has to start at zero: the backward writes every
  // partial before it reads it.
  return m3_scan_bwd(desc, delta, u, Bc, Cc, A_real_p, A_imag_p, track_p, dy, dtype_dy, ckpt,
                     d_delta, d_u, d_Bc, d_Cc, d_A_real_p, d_A_imag_p, d_track_p, ws,
                     (size_t)M3_NOALLOC_SCRATCH_BYTES, stream);
}
