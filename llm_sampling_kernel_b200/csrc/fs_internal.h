// Host-side internals shared by the translation units of libfs_b200.so.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "fused_sampling_b200.h"

namespace fsb {

struct PlanOut {
  int splits;    // CTAs per row (cluster size)
  int chunks;    // 16-byte vectors per thread
  int threads;   // threads per CTA
  int capacity;  // survivor buffer entries (power of two)
  int mpt;       // maxima per thread
  int mgroup;    // lanes per maximum
  int mcta;      // maxima per CTA
  int slot;      // survivor slots per rank in the leader's buffer
  int smem;      // dynamic shared memory bytes per CTA
  int stream;    // 1: streaming path (slice + row-merge launches), 0: cluster path
  int merge_cap; // streaming: gathered-candidate capacity of the row merge (power of two)
  int merge_smem;
  uint64_t workspace;  // streaming: workspace bytes
  int wide;      // 1: wide path (top_k beyond the survivor buffer; ids and status only)
};

// printf-style message for fs_last_error() on this host thread.
void set_error(const char* fmt, ...);

fs_status make_plan(int64_t B, int64_t V, int64_t K, int32_t splits, int32_t path, PlanOut* out);
fs_status run_cluster(const fs_sample_args* a, int mode, uint64_t* cand_out, cudaStream_t stream);
fs_status run_merge(const fs_sample_args* a, const uint64_t* cand, int parts, cudaStream_t stream);
fs_status run_tp_merge(const fs_sample_args* a, const uint64_t* local_cand, const fs_tp_peers* tp,
                       cudaStream_t stream);

// cudaFuncGetAttributes + occupancy into an fs_kernel_attr row.
void fill_attr(const void* fn, int block, int smem, fs_kernel_attr* row);
void append_cluster_attrs(std::vector<fs_kernel_attr>& rows);
void append_probe_attrs(std::vector<fs_kernel_attr>& rows);

}  // namespace fsb
