// fs_sample_noalloc: fs_sample for callers that cannot allocate device memory. The streaming
// path's scratch is a fixed array in this module's device memory instead of a caller workspace.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "fs_internal.h"
#include "fused_sampling_b200.h"

// The streaming path's per-call candidate lists and counts. Nothing in it has to start at zero:
// every count word is written by its slice CTA before the row merge reads it, and the merge reads
// only the candidate slots those counts cover. One array per device, shared by every call.
static __device__ __align__(256) unsigned char g_static_scratch[FS_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device, looked up once per device.
fs_status static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    fsb::set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    fsb::set_error("device %d is beyond the %d devices this build tracks", dev, kMaxDevices);
    return FS_EUNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      fsb::set_error("cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
      return FS_ELAUNCH;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FS_OK;
}

}  // namespace

extern "C" FS_API fs_status fs_sample_noalloc(const fs_sample_args* args, fs_stream_t stream) {
  if (args == nullptr) {
    fsb::set_error("args is NULL");
    return FS_EINVAL;
  }
  fs_sample_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  const uint64_t need = fs_workspace_size(&a);
  if (need > FS_STATIC_SCRATCH_BYTES) {
    fsb::set_error("this call needs %llu bytes of scratch; the static scratch holds %llu "
                   "(split the batch, or use fs_sample with a workspace)",
                   static_cast<unsigned long long>(need),
                   static_cast<unsigned long long>(FS_STATIC_SCRATCH_BYTES));
    return FS_EWORKSPACE;
  }
  if (need > 0) {
    void* p = nullptr;
    const fs_status st = static_scratch(&p);
    if (st != FS_OK) return st;
    a.workspace = p;
    a.workspace_bytes = FS_STATIC_SCRATCH_BYTES;
  }
  return fs_sample(&a, stream);
}
