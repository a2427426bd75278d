// fs_sample_noalloc: fs_sample for callers that cannot allocate device memory. The scratch of the
// paths that need one (the streaming path's candidate lists, the wide path's key histograms) is
// a fixed array in this module's device memory instead of a caller workspace.
#include <cuda.h>  // CUcontext and CUresult only: the driver is reached through the runtime's entry points
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "fs_internal.h"
#include "fused_sampling_b200.h"

// Scratch of one call. Nothing in it has to start at zero: the streaming path's count words are
// written by their slice CTAs before the row merge reads them, and the merge reads only the slots
// those counts cover; the wide path clears its histogram itself. One array per device (per CUDA
// context), shared by every call.
static __device__ __align__(256) unsigned char g_static_scratch[FS_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxEntries = 64;
struct ScratchEntry {
  int dev;
  unsigned long long ctx;  // the context's unique id (0: not known)
  void* ptr;
};
std::mutex g_scratch_mu;
ScratchEntry g_scratch[kMaxEntries];
int g_scratch_n = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (never reused in the process, unlike the
// handle's address after a cudaDeviceReset), or 0 when there is none or it cannot be read.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_static_scratch in the current device's current context, looked up once per
// (device, context): after a cudaDeviceReset the module is loaded again, at a new address, in a
// context with a new id, so a stale address is never reused.
fs_status static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    fsb::set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  unsigned long long ctx = current_context_id();
  for (int i = 0; i < g_scratch_n; ++i) {
    if (g_scratch[i].dev == dev && g_scratch[i].ctx == ctx) {
      *out = g_scratch[i].ptr;
      return FS_OK;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_static_scratch);  // (creates the device's context when needed)
  if (e != cudaSuccess || p == nullptr) {
    fsb::set_error("cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  ctx = current_context_id();
  int slot = g_scratch_n < kMaxEntries ? g_scratch_n++ : -1;
  if (slot < 0) {  // full: forget the oldest entry
    for (int i = 1; i < kMaxEntries; ++i) g_scratch[i - 1] = g_scratch[i];
    slot = kMaxEntries - 1;
  }
  g_scratch[slot] = ScratchEntry{dev, ctx, p};
  *out = p;
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
