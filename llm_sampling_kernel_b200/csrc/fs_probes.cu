// Floor probes used as a roofline bracket for the fused sampler, plus the C-ABI glue that does
// not belong to one kernel (errors, version, kernel attributes).
//
// The probes follow the reference's measurement design (csrc/probes.cu:8-68): an empty launch
// that writes [B] int64, one full pass per row with one CTA, and one full pass with the row
// split over several CTAs. Here the split pass merges inside a thread-block cluster instead of
// a second launch, so both passes are one launch.
#include <cooperative_groups.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "fs_device.cuh"
#include "fs_internal.h"

namespace cg = cooperative_groups;

namespace fsb {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void fill_attr(const void* fn, int block, int smem, fs_kernel_attr* row) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, fn) != cudaSuccess) {
    cudaGetLastError();
    row->regs = -1;
    return;
  }
  row->regs = a.numRegs;
  row->local_bytes = static_cast<int32_t>(a.localSizeBytes);
  row->static_smem = static_cast<int32_t>(a.sharedSizeBytes);
  int blocks = 0;
  // The occupancy query needs the function's dynamic shared memory limit to cover `smem`; the
  // limit is raised for the query only and put back afterwards, so that the limits the launch
  // paths granted (and remember granting) stay as they were.
  const int granted = a.maxDynamicSharedSizeBytes;
  const bool raise = smem > granted;
  if (raise) cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, block, smem) != cudaSuccess) {
    cudaGetLastError();
    blocks = -1;
  }
  if (raise) cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, granted);
  row->blocks_per_sm = blocks;
}

constexpr int kProbeThreads = 256;

__global__ void fs_noop_kernel(int64_t* __restrict__ out, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = 0;
}

// Packed (key, ~id) max over [lo, hi) of one row, vector loads where aligned.
__device__ __forceinline__ uint64_t scan_max(const uint16_t* __restrict__ row, int lo, int hi,
                                             bool vec) {
  uint64_t best = 0ull;
  int i = lo;
  if (vec) {
    const int vlo = (lo + 7) >> 3, vhi = hi >> 3;
    for (int j = lo + threadIdx.x; j < min(hi, vlo * 8); j += blockDim.x)
      best = max(best, pack(order_key(row[j]), j));
    for (int g = vlo + threadIdx.x; g < vhi; g += blockDim.x) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(row) + g);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        best = max(best, pack(order_key(w[q] & 0xFFFFu), g * 8 + 2 * q));
        best = max(best, pack(order_key(w[q] >> 16), g * 8 + 2 * q + 1));
      }
    }
    i = max(lo, vhi * 8);
  }
  for (int j = i + threadIdx.x; j < hi; j += blockDim.x) best = max(best, pack(order_key(row[j]), j));
  return best;
}

__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t* scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, v, off);
    v = o > v ? o : v;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint64_t w = lane < (blockDim.x >> 5) ? scratch[lane] : 0ull;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, w, off);
      w = o > w ? o : w;
    }
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  return scratch[32];
}

__global__ void __launch_bounds__(kProbeThreads) fs_scan_rowblock_kernel(
    const uint16_t* __restrict__ x, int64_t stride, int vocab, int vec, int64_t* __restrict__ out) {
  __shared__ uint64_t scratch[33];
  const uint16_t* row = x + static_cast<int64_t>(blockIdx.x) * stride;
  const uint64_t best = block_max_u64(scan_max(row, 0, vocab, vec != 0), scratch);
  if (threadIdx.x == 0) out[blockIdx.x] = static_cast<int64_t>(packed_id(best));
}

__global__ void __launch_bounds__(kProbeThreads) fs_scan_split_kernel(
    const uint16_t* __restrict__ x, int64_t stride, int vocab, int vec, int64_t* __restrict__ out) {
  __shared__ uint64_t scratch[33];
  __shared__ uint64_t parts[kMaxSplits];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = static_cast<int>(cluster.num_blocks());
  const int s = static_cast<int>(cluster.block_rank());
  const uint16_t* row = x + static_cast<int64_t>(blockIdx.y) * stride;
  const int per = ((vocab + S - 1) / S + 7) & ~7;
  const int lo = min(vocab, s * per), hi = min(vocab, lo + per);
  const uint64_t best = block_max_u64(scan_max(row, lo, hi, vec != 0), scratch);
  if (threadIdx.x == 0) *cluster.map_shared_rank(&parts[s], 0) = best;
  cluster.sync();
  if (s == 0 && threadIdx.x == 0) {
    uint64_t m = 0ull;
    for (int r = 0; r < S; ++r) m = parts[r] > m ? parts[r] : m;
    out[blockIdx.y] = static_cast<int64_t>(packed_id(m));
  }
}

void append_probe_attrs(std::vector<fs_kernel_attr>& rows) {
  struct Item {
    const char* name;
    const void* fn;
  } items[] = {{"fs_noop_kernel", reinterpret_cast<const void*>(fs_noop_kernel)},
               {"fs_scan_rowblock_kernel", reinterpret_cast<const void*>(fs_scan_rowblock_kernel)},
               {"fs_scan_split_kernel", reinterpret_cast<const void*>(fs_scan_split_kernel)}};
  for (const Item& it : items) {
    fs_kernel_attr r = {};
    std::snprintf(r.name, sizeof(r.name), "%s", it.name);
    r.block = kProbeThreads;
    fill_attr(it.fn, kProbeThreads, 0, &r);
    rows.push_back(r);
  }
}

static fs_status check_probe(const void* logits, int32_t dtype, int64_t batch, int64_t vocab,
                             int64_t stride, const int64_t* out) {
  if (logits == nullptr || out == nullptr) {
    set_error("logits or out is NULL");
    return FS_EINVAL;
  }
  if (dtype != FS_F16 && dtype != FS_BF16) {
    set_error("logits must be float16 or bfloat16");
    return FS_EINVAL;
  }
  if (batch < 1 || batch > 65535 || vocab < 1 || vocab > (1 << 30) || stride < vocab) {
    set_error("invalid probe shape");
    return FS_EINVAL;
  }
  return FS_OK;
}

static fs_status launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

}  // namespace fsb

extern "C" const char* fs_last_error(void) { return fsb::g_last_error.c_str(); }

extern "C" const char* fs_version(void) { return "fused_sampling_b200 1.0 (sm_100a)"; }

extern "C" fs_status fs_probe_noop(int64_t* out, int64_t batch, fs_stream_t stream) {
  if (out == nullptr || batch < 1) {
    fsb::set_error("out is NULL or batch < 1");
    return FS_EINVAL;
  }
  const unsigned blocks = static_cast<unsigned>((batch + 31) / 32);
  fsb::fs_noop_kernel<<<blocks, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(out, batch);
  return fsb::launch_status("probe_noop launch");
}

extern "C" fs_status fs_probe_scan_rowblock(const void* logits, int32_t dtype, int64_t batch,
                                            int64_t vocab, int64_t row_stride, int64_t* out,
                                            fs_stream_t stream) {
  fs_status st = fsb::check_probe(logits, dtype, batch, vocab, row_stride, out);
  if (st != FS_OK) return st;
  const int vec = (reinterpret_cast<uintptr_t>(logits) % 16 == 0 && row_stride % 8 == 0) ? 1 : 0;
  fsb::fs_scan_rowblock_kernel<<<static_cast<unsigned>(batch), fsb::kProbeThreads, 0,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(logits), row_stride, static_cast<int>(vocab), vec, out);
  return fsb::launch_status("probe_scan_rowblock launch");
}

extern "C" fs_status fs_probe_scan_split(const void* logits, int32_t dtype, int64_t batch,
                                         int64_t vocab, int64_t row_stride, int32_t splits,
                                         int64_t* out, fs_stream_t stream) {
  fs_status st = fsb::check_probe(logits, dtype, batch, vocab, row_stride, out);
  if (st != FS_OK) return st;
  if (splits < 1 || splits > fsb::kMaxSplits) {
    fsb::set_error("splits must be in [1, %d]", fsb::kMaxSplits);
    return FS_EINVAL;
  }
  const int vec = (reinterpret_cast<uintptr_t>(logits) % 16 == 0 && row_stride % 8 == 0) ? 1 : 0;
  const void* fn = reinterpret_cast<const void*>(fsb::fs_scan_split_kernel);
  if (splits > 8) cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(batch), 1);
  cfg.blockDim = dim3(fsb::kProbeThreads, 1, 1);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fsb::fs_scan_split_kernel,
                                           static_cast<const uint16_t*>(logits), row_stride,
                                           static_cast<int>(vocab), vec, out);
  if (e != cudaSuccess) {
    fsb::set_error("probe_scan_split launch: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

extern "C" int32_t fs_kernel_attrs(fs_kernel_attr* rows, int32_t cap) {
  std::vector<fs_kernel_attr> all;
  fsb::append_cluster_attrs(all);
  fsb::append_probe_attrs(all);
  if (rows != nullptr) {
    for (int32_t i = 0; i < cap && i < static_cast<int32_t>(all.size()); ++i) rows[i] = all[i];
  }
  return static_cast<int32_t>(all.size());
}
