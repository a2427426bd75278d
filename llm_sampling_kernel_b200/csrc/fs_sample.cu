// Fused top-k / top-p sampler for B200 (sm_100a): one thread-block cluster per row.
//
// One launch per call; the logits are read from HBM exactly once.
//   * The row is split across the S CTAs of a cluster (S <= 16). Each thread holds its part of
//     the row in registers (C x 16-byte vectors) for the whole kernel.
//   * Phase 1 - maxima: each thread reduces its values to a few sub-chunk maxima with the
//     NaN-propagating packed max (two logits per instruction). The maxima also classify the
//     row (NaN / +inf / all -inf). The start barrier of the cluster is split around the loads.
//   * Phase 2 - exchange: every CTA writes its maxima (as 16-bit order keys) and its row flags
//     into every rank's shared memory over distributed shared memory. One cluster barrier.
//   * Phase 3 - threshold: every CTA runs the same two-level 8-bit radix select over all
//     maxima and gets L, the k-th largest maximum. Those k maxima are distinct elements, so
//     every element of the top-k is >= L.
//   * Phase 4 - filter: every element >= L (packed compare, two logits per instruction) is a
//     survivor; each CTA writes its survivors as packed (key, ~id) words into its own slot range
//     of the leader CTA's buffer, and its count. One cluster barrier. Typically ~1.1k remain.
//   * If a slot range overflows (heavy ties: constant rows, few distinct values), an exact
//     two-level 8-bit radix select over the row finds the k-th key T, and the lowest-id ties at
//     T are chosen by an id-ordered prefix count.
//   * Phases 5..7 in the leader: compaction, sort of the survivors (value desc, id asc) by
//     rank counting across the CTA, FP32 softmax over the top k (expf, no fast-math),
//     cumulative sum accumulated in double and rounded per element, exclusive-prefix top-p cut,
//     inverse-CDF draw against u * Z_p. Other ranks leave right after the survivor barrier.
//   The leader's serial part is written as short rolled loops: it runs once per launch on one
//   SM, so its cost is instruction fetch as much as execution.
//
// Reference algorithm followed (sathviknookala/llm_sampling_kernel):
//   selection semantics  benchmarks/reference.py:47-54 (stable descending sort, first k)
//   softmax/cumsum/cut   benchmarks/reference.py:55-62, csrc/fused_sampling.cu:264-293
//   draw                 csrc/fused_sampling.cu:294-309
//   phase ablation       csrc/fused_sampling.cu:168-214,475-501
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "fs_device.cuh"
#include "fs_internal.h"

namespace cg = cooperative_groups;

namespace fsb {

constexpr int NT = 256;  // threads per CTA (the 8-bit histograms map one thread per bin)
static_assert(NT == 256, "the 8-bit histogram passes map one thread per bin");
constexpr int kMaxMaxima = 4096;   // maxima exchanged per row, all ranks together

struct Params {
  const uint16_t* logits;
  int64_t row_stride;
  int32_t vocab;
  int32_t K;  // bound on k: min(top_k, V)
  uint32_t id_base;
  float top_p;
  const int32_t* k_rows;
  const float* p_rows;
  const float* uniforms;
  uint64_t seed, offset;
  const int64_t* seed_ptr;
  const int64_t* offset_ptr;
  uint64_t offset_intragraph;
  int64_t row_base;
  int64_t* out;
  int64_t* topk_ids;
  uint8_t* keep;
  float* renormed;
  int32_t* status;
  uint64_t* cand_out;  // shard candidates, [B, K + 1]
  int32_t cap;         // survivor capacity, power of two
  int32_t slot;        // survivor slots per rank in the leader's buffer (cap / S)
  int32_t mpt;         // maxima per thread: 1, 2, 4 or 8
  int32_t mgroup;      // lanes per maximum (power of two <= 32), used when mpt == 1
  int32_t mcta;        // maxima per CTA: NT * mpt / mgroup
  int32_t vec;         // 16-byte vector loads allowed
  int32_t stop;        // 0 = full pipeline, else ablation phase
  int32_t mode;        // kModeSample / kModeTopk / kModeShard
  float temperature;   // softmax temperature (1 = none): candidates' logits / T before the softmax
  int32_t early;       // the logits are complete at enqueue: the cluster kernel reads them before the wait
};

constexpr int kModeSample = 0;
constexpr int kModeTopk = 1;
constexpr int kModeShard = 2;

// ctl[] slots (per CTA)
constexpr int kCtlFlags = 14;   // this rank's row flags
// uscr[16 + w]: warp w's row flags, written before the CTA's first barrier (no zeroing needed,
// unlike a shared counter whose zeroing would race with other warps' updates before that barrier)
constexpr int kUscrFlags = 16;
constexpr int kCtlLKey = 0;     // threshold key
constexpr int kCtlStatus = 1;   // row status
constexpr int kCtlLocal = 2;    // this rank's staged survivors
constexpr int kCtlN = 3;        // survivors of the row
constexpr int kCtlScr0 = 5;     // two words of block-search results
constexpr int kCtlHb = 8;       // fallback scratch
constexpr int kCtlAbove = 9;
constexpr int kCtlT = 10;
constexpr int kCtlTmo = 12;     // TP exchange: some flag wait ran out
constexpr int kCtlNgt = 11;

constexpr uint32_t kFlagNaN = 1u, kFlagPosInf = 2u, kFlagAboveNegInf = 4u;

struct alignas(16) Shared {
  uint32_t mkeys[kMaxMaxima]; // every rank's maxima keys; rank r at [r * mcta, (r + 1) * mcta)
  uint32_t flags[kMaxSplits]; // every rank's row flags
  uint32_t cnt[kMaxSplits];   // fallback: per-rank counts above T
  uint32_t cnt2[kMaxSplits];  // fallback: per-rank tie counts
  uint32_t h1[256];           // threshold radix histograms
  uint32_t h2[256];
  uint32_t fh1[256];          // leader: fallback level-1 histogram (key >> 8)
  uint32_t fh2[256];          // leader: fallback level-2 histogram (key & 0xFF inside hb)
  uint32_t lh[256];           // fallback: local histogram before it is pushed
  uint32_t ctl[16];
  int iscr[40];
  uint32_t uscr[40];
  double dscr[40];
};

// the 256-bin histograms are read with 16-byte loads
static_assert(offsetof(Shared, h1) % 16 == 0 && offsetof(Shared, h2) % 16 == 0 && offsetof(Shared, fh1) % 16 == 0 &&
                  offsetof(Shared, fh2) % 16 == 0 && offsetof(Shared, lh) % 16 == 0,
              "histogram alignment");

__host__ __device__ constexpr size_t shared_bytes(int cap) {
  return sizeof(Shared) + static_cast<size_t>(cap) * (sizeof(uint64_t) + 2 * sizeof(float));
}

extern __shared__ __align__(16) unsigned char g_smem[];

__device__ __forceinline__ uint32_t word_of(const uint4& v, int q) {
  return q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
}

// Programmatic dependent launch (griddepcontrol): no-ops when the grid was launched without the
// programmatic-serialization attribute.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Warms L2 with bytes [lo, lo + len) of row b (clipped to the row's 2V bytes), one 128-byte line
// per thread and step. Called before grid_dependency_wait(): while the previous kernel of the
// stream finishes, this grid's reads of its own input are already on their way from DRAM. Only
// prefetches: the loads that use the data still follow the wait, and L2 is where every write of
// the previous kernel lands, so they see its results.
__device__ __forceinline__ void prefetch_row_l2(const uint16_t* __restrict__ logits, int64_t row_stride, int vocab,
                                                int b, int64_t lo, int64_t len, int t, int nthreads) {
  const char* row = reinterpret_cast<const char*>(logits + static_cast<int64_t>(b) * row_stride);
  const int64_t end = min(lo + len, static_cast<int64_t>(vocab) * 2);
  for (int64_t off = (lo & ~static_cast<int64_t>(127)) + static_cast<int64_t>(t) * 128; off < end;
       off += static_cast<int64_t>(nthreads) * 128)
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(row + off));
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// An L2 access policy that evicts the lines it touches first: for data read exactly once
// (logits streamed by the slice kernel), so that it does not push out what later kernels of the
// call read back from L2 (the slices' candidate lists).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}

// 16-byte read-only global load under an L2 access policy.
__device__ __forceinline__ uint4 ldg_policy(const uint4* ptr, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr), "l"(pol));
  return v;
}

// Split cluster barrier: arrive (release) now, wait (acquire) later.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
// Arrive without ordering earlier memory accesses (they are reads whose values were consumed).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// 32-bit distributed-shared-memory addressing: the address of `local` (a shared-memory
// location of this CTA) in the CTA of cluster rank `rank`, and accesses through it.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ uint32_t ld_dsmem(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
// Atomic add on a word in some rank's shared memory (address from dsmem_addr); returns the old value.
__device__ __forceinline__ uint32_t atom_add_dsmem(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;\n" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_dsmem64(uint32_t addr, uint64_t v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;\n" ::"r"(addr), "l"(v) : "memory");
}
// Warp-aggregated shared-memory histogram add: lanes with the same bin elect one adder.
// All 32 lanes must call it.
__device__ __forceinline__ void hist_add_warp(uint32_t* h, uint32_t bin, bool valid) {
  const uint32_t tag = valid ? bin : 0xFFFFFFFFu;
  const unsigned peers = __match_any_sync(0xFFFFFFFFu, tag);
  if (valid && (threadIdx.x & 31) == (__ffs(peers) - 1)) atomicAdd(&h[bin], __popc(peers));
}

// One warp: in the 256-bin histogram h, the bin where the count from the top reaches `want`
// and the count strictly above it (lane l owns bins 255-8l .. 248-8l; h is 16-byte aligned). Returns false when the
// total is below `want`. Results are valid in every lane.
__device__ __forceinline__ bool warp_boundary_256(const uint32_t* h, uint32_t want, uint32_t* bin,
                                                  uint32_t* above) {
  const int lane = threadIdx.x & 31;
  // the lane's 8 bins, 255 - 8 lane - j for j = 0..7, as two 16-byte loads
  const uint4* h4 = reinterpret_cast<const uint4*>(h);
  const uint4 lo = h4[62 - 2 * lane], hi = h4[63 - 2 * lane];
  const uint32_t bins[8] = {hi.w, hi.z, hi.y, hi.x, lo.w, lo.z, lo.y, lo.x};
  uint32_t pre[8], acc = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    acc += bins[j];
    pre[j] = acc;  // inclusive count of this lane's first j+1 bins (from the top)
  }
  const uint32_t inc = warp_incl_scan(acc);
  const uint32_t before = inc - acc;
  const unsigned ball = __ballot_sync(0xFFFFFFFFu, inc >= want);
  if (ball == 0u) return false;
  const int l0 = __ffs(ball) - 1;
  unsigned hit = 0u;
#pragma unroll
  for (int j = 7; j >= 0; --j) hit = (hit << 1) | (before + pre[j] >= want ? 1u : 0u);
  const int j0 = __ffs(hit) - 1;  // first of this lane's bins reaching `want` (valid in lane l0)
  uint32_t ab = before;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j < j0) ab = before + pre[j];
  const uint32_t b = static_cast<uint32_t>(255 - 8 * lane - j0);
  *bin = __shfl_sync(0xFFFFFFFFu, b, l0);
  *above = __shfl_sync(0xFFFFFFFFu, ab, l0);
  return true;
}

// One warp's scan of a 256-bin histogram h (16-byte aligned, top bin h[255]; lane l owns bins
// 255-8l .. 248-8l), loaded once and then searched for any number of wants.
struct WarpHistScan {
  uint32_t pre[8];  // inclusive count of this lane's first j+1 bins (from the top)
  uint32_t inc;     // inclusive count through this lane
  __device__ __forceinline__ explicit WarpHistScan(const uint32_t* h) {
    const int lane = threadIdx.x & 31;
    const uint4* h4 = reinterpret_cast<const uint4*>(h);
    const uint4 lo = h4[62 - 2 * lane], hi = h4[63 - 2 * lane];
    const uint32_t bins[8] = {hi.w, hi.z, hi.y, hi.x, lo.w, lo.z, lo.y, lo.x};
    uint32_t acc = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc += bins[j];
      pre[j] = acc;
    }
    inc = warp_incl_scan(acc);
  }
  // The bin where the count from the top first reaches `want`; false when the total is below it.
  // Every lane calls it and gets the result.
  __device__ __forceinline__ bool find(uint32_t want, uint32_t* bin) const {
    const int lane = threadIdx.x & 31;
    const uint32_t before = inc - pre[7];
    const unsigned ball = __ballot_sync(0xFFFFFFFFu, inc >= want);
    int j0 = 7;
#pragma unroll
    for (int j = 6; j >= 0; --j)
      if (before + pre[j] >= want) j0 = j;
    const int l0 = ball != 0u ? __ffs(ball) - 1 : 0;
    *bin = __shfl_sync(0xFFFFFFFFu, static_cast<uint32_t>(255 - 8 * lane - j0), l0);
    return ball != 0u;
  }
};

// The kk-th largest of the n 16-bit keys keys[0..n) (0 when n < kk): two 8-bit radix levels with
// shared-memory histograms h1 (high byte, filled by every thread) and h2 (low byte inside the
// boundary high bin, filled by warp 0), each boundary found by one warp scan. h1 and h2 must be
// zero on entry. Every thread calls it.
__device__ uint32_t kth_largest_key(const uint32_t* keys, int n, int kk, uint32_t* h1, uint32_t* h2,
                                    uint32_t* result) {
  const int t = threadIdx.x;
  for (int i = t; i < n; i += NT) atomicAdd(&h1[keys[i] >> 8], 1u);
  __syncthreads();
  if (t < 32) {
    uint32_t hb = 0u, above = 0u, L = 0u;
    if (warp_boundary_256(h1, static_cast<uint32_t>(kk), &hb, &above)) {
      for (int i = t; i < n; i += 32) {
        const uint32_t k = keys[i];
        if ((k >> 8) == hb) atomicAdd(&h2[k & 0xFFu], 1u);
      }
      __syncwarp();
      uint32_t lb = 0u, dummy = 0u;
      warp_boundary_256(h2, static_cast<uint32_t>(kk) - above, &lb, &dummy);
      L = (hb << 8) | lb;
    }
    if (t == 0) result[0] = L;
  }
  __syncthreads();
  return result[0];
}

// A lower bound L on the want-th largest of the CTA's 16-bit keys, nk <= 8 per thread in
// registers: one 256-bin histogram anchored at the largest key (bin = (max - key) >> sh, clamped
// to the last bin), the boundary found by one warp scan, L = the lower edge of the boundary bin.
// With sh == 0 and the boundary below the last bin, L is exactly the want-th largest key. At
// least `want` keys are >= L. Returns 0 when the CTA holds fewer than `want` keys.
// When `ladder` is not null, the CTA's last warp also stores there, after the last barrier, the
// same kind of bound for the wants ceil(want/8), ceil(want/4), ceil(want/2) and want, in 16-bit
// fields 0..3; a field is 0 (no bound) unless it lies above `floor`, so that every key counted
// above it is a real element's. h: 256 shared words, zeroed by the caller before the call (the
// call's first barrier publishes that), read by the last warp after the call returns to the
// others: the caller must not write h before the CTA's next barrier. scratch: >= 9 shared words.
// Every thread of the CTA calls it; three barriers.
__device__ uint32_t anchored_threshold(const uint32_t (&keys)[8], int nk, int want, int sh, uint32_t* h,
                                       uint32_t* scratch, uint32_t floor, uint64_t* ladder) {
  const int t = threadIdx.x;
  uint32_t m = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < nk) m = max(m, keys[i]);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if ((t & 31) == 0) scratch[t >> 5] = m;
  __syncthreads();
  uint32_t kmax = 0u;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) kmax = max(kmax, scratch[w]);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < nk) atomicAdd(&h[255u - min(255u, (kmax - keys[i]) >> sh)], 1u);  // top bin = largest key
  __syncthreads();
  const uint32_t w = static_cast<uint32_t>(want);
  // the lower edge of the bin where the count from the top reaches `wi` (0: no bound)
  auto bound = [&](const WarpHistScan& hs, uint32_t wi) -> uint32_t {
    uint32_t idx = 0u;
    if (!hs.find(wi, &idx) || idx == 0u) return 0u;  // idx 0: the last, open-ended bin
    const uint32_t hi = kmax - ((255u - idx) << sh);
    const uint32_t width = (1u << sh) - 1u;
    return hi > width ? hi - width : 0u;
  };
  if (t < 32) {
    const WarpHistScan hs(h);
    const uint32_t L = bound(hs, w);
    if (t == 0) scratch[8] = L;
  }
  __syncthreads();
  const uint32_t L = scratch[8];
  // the ladder, by the last warp while the others go on (h is left alone until they meet again)
  if (ladder != nullptr && t >= NT - 32) {
    const WarpHistScan hs(h);
    const uint32_t l0 = bound(hs, (w + 7u) / 8u), l1 = bound(hs, (w + 3u) / 4u), l2 = bound(hs, (w + 1u) / 2u);
    if (t == NT - 32) {
      *ladder = static_cast<uint64_t>(l0 > floor ? l0 : 0u) | static_cast<uint64_t>(l1 > floor ? l1 : 0u) << 16 |
                static_cast<uint64_t>(l2 > floor ? l2 : 0u) << 32 | static_cast<uint64_t>(L > floor ? L : 0u) << 48;
    }
  }
  return L;
}

// The want-th largest of n 16-bit keys in shared memory by one warp (no block barrier):
// one 256-bin histogram anchored at the largest key (bin = (max - key) >> sh) in the warp's own
// 256 words `h`, one warp scan. Returns the lower edge of the boundary bin (exactly the want-th
// key when sh == 0), or sets *clamped when the boundary falls in the last, open-ended bin (keys
// spread wider than the histogram) and the caller must search another way. 0 when n < want.
__device__ uint32_t warp_anchored_kth(const uint32_t* keys, int n, int want, int sh, uint32_t* h,
                                      bool* clamped) {
  const int lane = threadIdx.x & 31;
  uint32_t m = 0u;
  for (int i = lane; i < n; i += 32) m = max(m, keys[i]);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
#pragma unroll
  for (int j = 0; j < 8; ++j) h[lane * 8 + j] = 0u;
  __syncwarp();
  for (int i = lane; i < n; i += 32) atomicAdd(&h[255u - min(255u, (m - keys[i]) >> sh)], 1u);
  __syncwarp();
  uint32_t idx = 0u, above = 0u, L = 0u;
  *clamped = false;
  if (warp_boundary_256(h, static_cast<uint32_t>(want), &idx, &above)) {
    const uint32_t bin = 255u - idx;
    if (bin < 255u) {
      const uint32_t hi = m - (bin << sh);
      const uint32_t width = (1u << sh) - 1u;
      L = hi > width ? hi - width : 0u;
    } else {
      *clamped = true;
    }
  }
  __syncwarp();
  return L;
}

__device__ __forceinline__ float row_uniform(const Params& p, int b) {
  if (p.uniforms != nullptr) return p.uniforms[b];
  uint64_t seed = p.seed, off = p.offset;
  if (p.seed_ptr != nullptr) {
    seed = static_cast<uint64_t>(*p.seed_ptr);
    off = static_cast<uint64_t>(*p.offset_ptr) + p.offset_intragraph;
  }
  return splitmix_uniform(seed, off, static_cast<uint64_t>(p.row_base + b));
}


// Writes the outputs of a row that cannot be sampled (bad input or parameters). Called by
// `stride` threads numbered t = 0 .. stride-1 (the CTA, or one warp with t = lane).
__device__ void write_invalid_row(const Params& p, int b, int st, int t, int stride) {
  if (t == 0) {
    if (p.out != nullptr) p.out[b] = -1;
    if (p.status != nullptr) p.status[b] = st;
  }
  for (int i = t; i < p.K; i += stride) {
    const size_t o = static_cast<size_t>(b) * p.K + i;
    if (p.topk_ids != nullptr) p.topk_ids[o] = -1;
    if (p.keep != nullptr) p.keep[o] = 0;
    if (p.renormed != nullptr) p.renormed[o] = 0.0f;
  }
  if (p.cand_out != nullptr) {
    uint64_t* co = p.cand_out + static_cast<size_t>(b) * (p.K + 1);
    for (int i = t; i < p.K; i += stride) co[i] = 0ull;
    if (t == 0) co[p.K] = static_cast<uint64_t>(st);
  }
}

__device__ __forceinline__ void write_invalid_row(const Params& p, int b, int st) {
  write_invalid_row(p, b, st, static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x));
}

// Writes the top-K ids or the shard candidates of a sorted candidate list (shared memory).
// Returns true when the mode ends here. Called by `nthreads` threads numbered t = 0 .. nthreads-1.
__device__ bool write_selection(const Params& p, int b, const uint64_t* cand, int kk, int t, int nthreads) {
  if (p.mode == kModeTopk) {
    for (int i = t; i < p.K; i += nthreads)
      p.topk_ids[static_cast<size_t>(b) * p.K + i] = i < kk ? static_cast<int64_t>(packed_id(cand[i])) : -1;
    if (t == 0 && p.status != nullptr) p.status[b] = FS_ROW_OK;
    return true;
  }
  if (p.mode == kModeShard) {
    uint64_t* co = p.cand_out + static_cast<size_t>(b) * (p.K + 1);
    for (int i = t; i < p.K; i += nthreads) co[i] = i < kk ? cand[i] : 0ull;
    if (t == 0) co[p.K] = FS_ROW_OK;
    return true;
  }
  return false;
}

// Stage outputs (top-K ids, keep, renormed) from the sorted candidates and the per-rank
// probabilities / cumulative sums held in shared memory.
__device__ void write_stages(const Params& p, int b, const uint64_t* cand, const float* prob, int kk, int r,
                             float zp, int t, int nthreads) {
  for (int i = t; i < p.K; i += nthreads) {
    const size_t o = static_cast<size_t>(b) * p.K + i;
    if (p.topk_ids != nullptr) p.topk_ids[o] = i < kk ? static_cast<int64_t>(packed_id(cand[i])) : -1;
    if (p.keep != nullptr) p.keep[o] = (i <= r) ? 1 : 0;
    if (p.renormed != nullptr) p.renormed[o] = (i <= r) ? prob[i] / zp : 0.0f;
  }
}

// A candidate's logit as the softmax sees it: its 16-bit value in fp32, divided by the
// temperature (IEEE fp32 division; none when it is 1).
template <int DT>
__device__ __forceinline__ float tail_logit(const Params& p, uint32_t key) {
  const float x = key_to_float<DT>(key);
  return p.temperature == 1.0f ? x : __fdiv_rn(x, p.temperature);
}

// Block-wide tail for more than kWarpPathMax candidates: FP32 softmax over the top kk sorted
// candidates, exclusive-prefix top-p cut, inverse-CDF draw. All NT threads call it.
template <int DT>
__device__ void sample_tail_block(const Params& p, int b, const uint64_t* cand, int kk, float pp,
                                  float* prob, float* cum, double* dscr, int* iscr) {
  const int t = threadIdx.x;
  const float m = tail_logit<DT>(p, packed_key(cand[0]));
  if (m == INFINITY) {  // the scaled maximum overflowed
    write_invalid_row(p, b, FS_ROW_POSINF, t, NT);
    return;
  }
  double part = 0.0;
  for (int i = t; i < kk; i += NT) {
    const float w = expf(tail_logit<DT>(p, packed_key(cand[i])) - m);
    prob[i] = w;
    part += static_cast<double>(w);
  }
  const float z = static_cast<float>(block_sum<double, NT>(part, dscr));
  for (int i = t; i < kk; i += NT) prob[i] = prob[i] / z;
  __syncthreads();

  // inclusive cumulative sum accumulated in double and rounded once per element
  const int ipt = (kk + NT - 1) / NT;
  const int lo = min(kk, t * ipt), hi = min(kk, lo + ipt);
  double run = 0.0;
  for (int i = lo; i < hi; ++i) run += static_cast<double>(prob[i]);
  double total;
  double acc = block_incl_scan<double, NT>(run, dscr, &total) - run;
  for (int i = lo; i < hi; ++i) {
    acc += static_cast<double>(prob[i]);
    cum[i] = static_cast<float>(acc);
  }
  __syncthreads();

  // r = (first i >= 1 with !((c_i - p_i) < p)) - 1, or kk - 1 when p >= 1
  int fail = kk;
  if (pp < 1.0f) {
    for (int i = t; i < kk; i += NT)
      if (i >= 1 && !((cum[i] - prob[i]) < pp)) fail = min(fail, i);
  }
  fail = block_min<NT>(fail, iscr);
  const int r = fail - 1;
  if (p.stop == 6) {
    if (t == 0) p.out[b] = r + 1;
    return;
  }
  const float zp = cum[r];
  const float target = row_uniform(p, b) * zp;
  int pick = r;
  for (int i = t; i <= r; i += NT)
    if (cum[i] >= target) pick = min(pick, i);
  pick = block_min<NT>(pick, iscr);
  if (t == 0) {
    if (p.out != nullptr) p.out[b] = static_cast<int64_t>(packed_id(cand[pick]));
    if (p.status != nullptr) p.status[b] = FS_ROW_OK;
  }
  write_stages(p, b, cand, prob, kk, r, zp, t, NT);
}


// One-warp tail over kk <= 32 * R sorted candidates held in registers (blocked layout: lane l
// owns ranks l*R .. l*R+R-1): FP32 softmax, cumulative sum accumulated in double and rounded per
// element, exclusive-prefix cut, inverse-CDF draw against u * Z_p. One warp sum and one warp scan
// are the only collectives; no block barrier.
template <int DT, int R>
__device__ void sample_tail_warp(const Params& p, int b, const uint64_t* cand, int kk, float pp, float u,
                                 float* prob) {
  const int lane = threadIdx.x & 31;
  uint64_t v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane * R + r;
    v[r] = i < kk ? cand[i] : 0ull;
  }
  const float m = tail_logit<DT>(p, packed_key(__shfl_sync(0xFFFFFFFFu, v[0], 0)));
  if (m == INFINITY) {  // the scaled maximum overflowed
    write_invalid_row(p, b, FS_ROW_POSINF, lane, 32);
    return;
  }
  float pr[R];
  double part = 0.0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    pr[r] = (lane * R + r < kk) ? expf(tail_logit<DT>(p, packed_key(v[r])) - m) : 0.0f;
    part += static_cast<double>(pr[r]);
  }
  const float z = static_cast<float>(warp_sum(part));
  double loc = 0.0, pre[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    pr[r] = pr[r] / z;
    loc += static_cast<double>(pr[r]);
    pre[r] = loc;
  }
  const double excl = warp_incl_scan(loc) - loc;
  float cm[R];
  int fail = kk;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    cm[r] = static_cast<float>(excl + pre[r]);
    const int i = lane * R + r;
    if (pp < 1.0f && i >= 1 && i < kk && !((cm[r] - pr[r]) < pp)) fail = min(fail, i);
  }
  fail = __reduce_min_sync(0xFFFFFFFFu, static_cast<unsigned>(fail));
  const int rc = fail - 1;
  if (p.stop == 6) {
    if (lane == 0) p.out[b] = rc + 1;
    return;
  }
  float csel = 0.0f;
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (lane * R + r == rc) csel = cm[r];
  const float zp = __shfl_sync(0xFFFFFFFFu, csel, rc / R);
  const float target = u * zp;
  int pick = rc;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane * R + r;
    if (i <= rc && cm[r] >= target) pick = min(pick, i);
  }
  pick = static_cast<int>(__reduce_min_sync(0xFFFFFFFFu, static_cast<unsigned>(pick)));
  uint64_t vsel = 0ull;
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (lane * R + r == pick) vsel = v[r];
  const uint64_t win = __shfl_sync(0xFFFFFFFFu, vsel, pick / R);
  if (lane == 0) {
    if (p.out != nullptr) p.out[b] = static_cast<int64_t>(packed_id(win));
    if (p.status != nullptr) p.status[b] = FS_ROW_OK;
  }
  if (p.topk_ids != nullptr || p.keep != nullptr || p.renormed != nullptr) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (lane * R + r < kk) prob[lane * R + r] = pr[r];
    __syncwarp();
    write_stages(p, b, cand, prob, kk, rc, zp, lane, 32);
  }
}

// ctl slots of block_select_top (scratch of the fallback and of the survivor count, dead by then)
constexpr int kCtlSelHb = kCtlHb, kCtlSelAbove = kCtlAbove, kCtlSelT = kCtlT, kCtlSelNgt = kCtlNgt;
constexpr int kCtlSelEq = 5, kCtlSelCgt = 6, kCtlSelCtie = 2;
constexpr int kSelTies = 384;  // ties at the kk-th key that block_select_top ranks (3 KB of Shared)

// The kk largest of the n > kk distinct packed values src[0, n) into dst[0, kk), in no particular
// order. Two 8-bit levels over the 16-bit key (histograms in sh.h1) give the kk-th largest key T
// and the count above it; the values above T go straight to dst (positions from a shared
// counter), the values at T to a buffer in the fallback histograms' space (fh1, fh2, lh: free by
// now), where each is ranked among them by comparisons and the `need` largest (lowest ids) follow.
// More than kSelTies values at T: nothing is written to dst and false is returned (the caller
// sorts everything). All NT threads call it.
__device__ bool block_select_top(const uint64_t* src, int n, int kk, uint64_t* dst, Shared& sh) {
  const int t = threadIdx.x;
  uint32_t* h = sh.h1;
  uint64_t* ties = reinterpret_cast<uint64_t*>(sh.fh1);
  static_assert(offsetof(Shared, fh2) == offsetof(Shared, fh1) + 1024 &&
                    offsetof(Shared, lh) == offsetof(Shared, fh2) + 1024 && kSelTies * 8 <= 3 * 1024,
                "the tie buffer spans fh1, fh2 and lh");
  const uint32_t ukk = static_cast<uint32_t>(kk);
  h[t] = 0u;
  __syncthreads();
  for (int i = t; i < n; i += NT) atomicAdd(&h[packed_key(src[i]) >> 8], 1u);
  __syncthreads();
  if (t < 32) {
    uint32_t hb = 0u, above = 0u;
    warp_boundary_256(h, ukk, &hb, &above);  // n > kk: the boundary exists
    if (t == 0) {
      sh.ctl[kCtlSelHb] = hb;
      sh.ctl[kCtlSelAbove] = above;
    }
  }
  __syncthreads();
  const uint32_t hb = sh.ctl[kCtlSelHb], above = sh.ctl[kCtlSelAbove];
  h[t] = 0u;
  __syncthreads();
  for (int i = t; i < n; i += NT) {
    const uint32_t key = packed_key(src[i]);
    if ((key >> 8) == hb) atomicAdd(&h[key & 0xFFu], 1u);
  }
  __syncthreads();
  if (t < 32) {
    uint32_t lb = 0u, above2 = 0u;
    warp_boundary_256(h, ukk - above, &lb, &above2);
    if (t == 0) {
      sh.ctl[kCtlSelT] = (hb << 8) | lb;
      sh.ctl[kCtlSelNgt] = above + above2;
      sh.ctl[kCtlSelEq] = h[lb];
      sh.ctl[kCtlSelCgt] = 0u;
      sh.ctl[kCtlSelCtie] = 0u;
    }
  }
  __syncthreads();
  const uint32_t T = sh.ctl[kCtlSelT], ngt = sh.ctl[kCtlSelNgt], eq = sh.ctl[kCtlSelEq];
  if (eq > static_cast<uint32_t>(kSelTies)) return false;  // the same decision in every thread
  for (int i = t; i < n; i += NT) {
    const uint64_t x = src[i];
    const uint32_t key = packed_key(x);
    if (key > T) dst[atomicAdd(&sh.ctl[kCtlSelCgt], 1u)] = x;
    else if (key == T) ties[atomicAdd(&sh.ctl[kCtlSelCtie], 1u)] = x;
  }
  __syncthreads();
  const uint32_t need = ukk - ngt;
  for (uint32_t i = static_cast<uint32_t>(t); i < eq; i += NT) {
    const uint64_t x = ties[i];
    uint32_t r = 0u;
    for (uint32_t j = 0; j < eq; ++j) r += ties[j] > x ? 1u : 0u;
    if (r < need) dst[ngt + r] = x;
  }
  __syncthreads();
  return true;
}

// Sorts n packed candidates (value desc, id asc) from `src` into the top kk of `dst`, then
// writes the selection outputs or runs the tail. All NT threads of the CTA call it; `u` is the
// row's uniform (valid in warp 0).
// n <= NT: every candidate's rank is the count of larger ones (packed values are distinct),
// counted by its own thread in unrolled chunks of 16 (src is zero-padded to a multiple of 16;
// zeros are below every candidate). Larger n: bitonic sort in place in `src` (capacity >= next
// power of two of n). `src` may alias prob/cum (it is dead once `dst` holds the sorted
// candidates); `dst` may not.
template <int DT>
__device__ void finish_row(const Params& p, int b, uint64_t* src, int n, uint64_t* dst, int kk, float pp,
                           float u, float* prob, float* cum, Shared& sh) {
  const int t = threadIdx.x;
  if (n <= NT) {
    const int n16 = (n + 15) & ~15;
    for (int i = n + t; i < n16; i += NT) src[i] = 0ull;
    __syncthreads();
    if (t < n) {
      const uint64_t mine = src[t];
      const ulonglong2* s2 = reinterpret_cast<const ulonglong2*>(src);
      int rank = 0;
      for (int base = 0; base < n16; base += 16) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const ulonglong2 w = s2[(base >> 1) + q];
          rank += (w.x > mine) + (w.y > mine);
        }
      }
      if (rank < kk) dst[rank] = mine;
    }
    __syncthreads();
  } else {
    int P = 32;
    while (P < n) P <<= 1;
    int Pk = 32;
    while (Pk < kk) Pk <<= 1;
    // the exact top kk first when that shrinks the sort (dst holds Pk words: the maxima space
    // holds kMaxMaxima / 2 >= Pk when kk <= kMaxMaxima / 2, else dst is a cap-word buffer)
    if (Pk < P && block_select_top(src, n, kk, dst, sh)) {
      if (kk <= NT) {
        // rank counting of the kk selected (distinct values) into src, then back to dst
        if (t < kk) {
          const uint64_t mine = dst[t];
          int rank = 0;
          for (int j = 0; j < kk; ++j) rank += dst[j] > mine ? 1 : 0;
          src[rank] = mine;
        }
        __syncthreads();
        if (t < kk) dst[t] = src[t];
        __syncthreads();
      } else {
        for (int i = kk + t; i < Pk; i += NT) dst[i] = 0ull;
        __syncthreads();
        block_sort_desc<NT>(dst, Pk);
      }
    } else {
      for (int i = n + t; i < P; i += NT) src[i] = 0ull;
      __syncthreads();
      block_sort_desc<NT>(src, P);
      for (int i = t; i < kk; i += NT) dst[i] = src[i];
      __syncthreads();
    }
  }
  if (p.stop == 5) {
    if (t == 0) p.out[b] = static_cast<int64_t>(packed_id(dst[0]));
    return;
  }
  if (write_selection(p, b, dst, kk, t, NT)) return;
  if (kk <= 256) {
    if (t < 32) {
      if (kk <= 32) sample_tail_warp<DT, 1>(p, b, dst, kk, pp, u, prob);
      else if (kk <= 64) sample_tail_warp<DT, 2>(p, b, dst, kk, pp, u, prob);
      else sample_tail_warp<DT, 8>(p, b, dst, kk, pp, u, prob);
    }
  } else {
    sample_tail_block<DT>(p, b, dst, kk, pp, prob, cum, sh.dscr, sh.iscr);
  }
}

// Per-row k and p (a bad per-row value marks the row FS_ROW_BAD_PARAM).
__device__ __forceinline__ void row_params(const Params& p, int b, int* kk, float* pp, bool* bad) {
  *kk = p.K;
  *pp = p.top_p;
  *bad = false;
  if (p.k_rows != nullptr) {
    const int kr = p.k_rows[b];
    if (kr < 1) *bad = true;
    *kk = min(max(kr, 1), p.K);
  }
  if (p.p_rows != nullptr) {
    const float pr = p.p_rows[b];
    if (!(pr > 0.0f && pr <= 1.0f)) *bad = true;
    *pp = pr;
  }
}

// One 16-byte chunk (8 logits) of a row starting at element e0; lanes at or past V read as -inf.
template <int DT>
__device__ __forceinline__ uint4 load_chunk(const uint16_t* __restrict__ row, int e0, int V, int vec) {
  if (vec && e0 + 8 <= V) return __ldg(reinterpret_cast<const uint4*>(row) + (e0 >> 3));
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t lo16 = (e0 + 2 * q < V) ? static_cast<uint32_t>(row[e0 + 2 * q]) : Fmt<DT>::kNegInf;
    const uint32_t hi16 = (e0 + 2 * q + 1 < V) ? static_cast<uint32_t>(row[e0 + 2 * q + 1]) : Fmt<DT>::kNegInf;
    w[q] = lo16 | (hi16 << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Exact top-kk selection of the cluster's row, used when the survivor filter overflows the
// buffer (heavy ties). The k-th key T comes from one counting pass when it lies within four
// keys of the filter threshold L (at least kk keys are >= L): each thread counts its keys at
// L, L + 1, L + 2, L + 3 and at or above L + 4, the per-rank totals go to every rank, and every
// rank finds T and the per-rank counts above and at T from them. Otherwise two 8-bit radix
// levels over the order key give T and the count above it (csrc/fused_sampling.cu:163-209
// computes the same two levels per slice). The ties at T are then ranked in id order - rank
// boundaries follow the (rank, chunk, thread, lane) layout, which is increasing in token id -
// and the lowest `need` are kept. The slice is re-read from global memory (L2) chunk by chunk,
// so this rare path does not hold the row in registers. Every thread of every CTA of the
// cluster calls it; it writes kk packed candidates into the leader's buffer and returns kk.
// exact_select: chunks whose loads one pass issues together (all of them for small C)
__host__ __device__ constexpr int pass_batch(int C) { return C <= 6 ? C : 4; }

// exact_select's counting pass: keys at L + j for j < 4 and at or above L + 4, one 12-bit field
// each in a thread's 64-bit counter (a thread holds at most 8 * C <= 128 keys; the fields are
// taken apart before the warp sums)
constexpr int kBins = 5;
constexpr int kBinBits = 12;
static_assert(kBins * kBinBits <= 64 && 8 * 16 < (1 << kBinBits), "bin counters overflow");
static_assert(kBins * NT / 32 <= 40 && kBins * kMaxSplits <= 256, "bin totals do not fit uscr / lh");

template <int DT, int C>
__device__ __noinline__ int exact_select(Shared& sh, const uint16_t* __restrict__ row, int V, int vec,
                                         uint32_t id_base, int vbase, int kk, uint64_t* lsurv, uint32_t lkey) {
  cg::cluster_group cluster = cg::this_cluster();
  const int S = static_cast<int>(cluster.num_blocks());
  const int s = static_cast<int>(cluster.block_rank());
  const int t = threadIdx.x;
  // fn(e0, chunk) for the CTA's slice chunks in id order, re-read from L1/L2 in batches of
  // pass_batch(C) whose loads are issued together (one round trip per batch, not per chunk)
  constexpr int PB = pass_batch(C);
  auto for_chunks = [&](auto&& fn) {
#pragma unroll 1
    for (int c0 = 0; c0 < C; c0 += PB) {
      uint4 vv[PB];
#pragma unroll
      for (int i = 0; i < PB; ++i)
        if (c0 + i < C) vv[i] = load_chunk<DT>(row, (vbase + (c0 + i) * NT + t) * 8, V, vec);
#pragma unroll
      for (int i = 0; i < PB; ++i)
        if (c0 + i < C) fn((vbase + (c0 + i) * NT + t) * 8, vv[i]);
    }
  };

  static_assert(8 * C < (1 << kBinBits), "bin counters overflow");
  const int lane = t & 31, warp = t >> 5;
  // counting pass: this thread's keys at L + j (j < 4) and at or above L + 4
  uint64_t bins = 0ull;
  for_chunks([&](int e0, const uint4& v) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w = word_of(v, q);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t key = order_key(h ? (w >> 16) : (w & 0xFFFFu));
        if (e0 + 2 * q + h < V && key >= lkey)
          bins += 1ull << (kBinBits * min(key - lkey, static_cast<uint32_t>(kBins - 1)));
      }
    }
  });
  auto bin_of = [&](int j) -> uint32_t {
    return static_cast<uint32_t>(bins >> (kBinBits * j)) & ((1u << kBinBits) - 1u);
  };
  // warp totals, rank totals, then every rank's totals in every rank (lh[kBins * rank + j])
#pragma unroll
  for (int j = 0; j < kBins; ++j) {
    const uint32_t wj = __reduce_add_sync(0xFFFFFFFFu, bin_of(j));
    if (lane == 0) sh.uscr[kBins * warp + j] = wj;
  }
  __syncthreads();
  if (t < kBins * S) {
    const int r = t / kBins, j = t - r * kBins;
    uint32_t tot = 0u;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += sh.uscr[kBins * w + j];
    cluster.map_shared_rank(sh.lh, r)[kBins * s + j] = tot;
  }
  cluster.sync();  // F3: every rank holds every rank's totals
  uint32_t row_bin[kBins], pre_bin[kBins];  // the row's, and the ranks' before this one
#pragma unroll
  for (int j = 0; j < kBins; ++j) row_bin[j] = pre_bin[j] = 0u;
  for (int r = 0; r < S; ++r) {
#pragma unroll
    for (int j = 0; j < kBins; ++j) {
      const uint32_t c = sh.lh[kBins * r + j];
      row_bin[j] += c;
      pre_bin[j] += r < s ? c : 0u;
    }
  }
  // T = L + j for the largest j < 4 with fewer than kk keys above L + j and at least kk at or
  // above it; the same decision in every rank (the same totals)
  uint32_t T = 0u, n_gt = 0u, ngt = 0u, ntie = 0u, gt_base = 0u, tie_base = 0u;
  bool known = false;
  {
    uint32_t above = row_bin[kBins - 1], pabove = pre_bin[kBins - 1], mabove = bin_of(kBins - 1);
#pragma unroll
    for (int j = kBins - 2; j >= 0; --j) {
      if (!known && above < static_cast<uint32_t>(kk) && above + row_bin[j] >= static_cast<uint32_t>(kk)) {
        known = true;
        T = lkey + static_cast<uint32_t>(j);
        n_gt = above;
        ngt = mabove;
        ntie = bin_of(j);
        gt_base = pabove;
        tie_base = pre_bin[j];
      }
      above += row_bin[j];
      pabove += pre_bin[j];
      mabove += bin_of(j);
    }
  }
  uint32_t gt_off, gt_rank;  // this thread's offset among the rank's keys above T; their number
  if (known) {
    gt_off = block_incl_scan<uint32_t, NT>(ngt, sh.uscr, &gt_rank) - ngt;
  } else {
    // T beyond L + 3: two radix levels find it
    __syncthreads();  // every thread has read lh
    // level 1: high byte
    sh.lh[t] = 0u;
    __syncthreads();
    for_chunks([&](int e0, const uint4& v) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w = word_of(v, q);
        hist_add_warp(sh.lh, order_key(w & 0xFFFFu) >> 8, e0 + 2 * q < V);
        hist_add_warp(sh.lh, order_key(w >> 16) >> 8, e0 + 2 * q + 1 < V);
      }
    });
    __syncthreads();
    if (sh.lh[t] != 0u) atomicAdd(cluster.map_shared_rank(&sh.fh1[t], 0), sh.lh[t]);
    cluster.sync();  // F1
    {
      const uint32_t h = *cluster.map_shared_rank(&sh.fh1[255 - t], 0);
      uint32_t total;
      const uint32_t inc = block_incl_scan<uint32_t, NT>(h, sh.uscr, &total);
      if (inc >= static_cast<uint32_t>(kk) && inc - h < static_cast<uint32_t>(kk)) {
        sh.ctl[kCtlHb] = static_cast<uint32_t>(255 - t);
        sh.ctl[kCtlAbove] = inc - h;
      }
      sh.lh[t] = 0u;
      __syncthreads();
    }
    const uint32_t hb = sh.ctl[kCtlHb];
    const uint32_t n_above = sh.ctl[kCtlAbove];

    // level 2: low byte inside bucket hb
    for_chunks([&](int e0, const uint4& v) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w = word_of(v, q);
        const uint32_t k0 = order_key(w & 0xFFFFu), k1 = order_key(w >> 16);
        hist_add_warp(sh.lh, k0 & 0xFFu, e0 + 2 * q < V && (k0 >> 8) == hb);
        hist_add_warp(sh.lh, k1 & 0xFFu, e0 + 2 * q + 1 < V && (k1 >> 8) == hb);
      }
    });
    __syncthreads();
    if (sh.lh[t] != 0u) atomicAdd(cluster.map_shared_rank(&sh.fh2[t], 0), sh.lh[t]);
    cluster.sync();  // F2
    {
      const uint32_t want = static_cast<uint32_t>(kk) - n_above;
      const uint32_t h = *cluster.map_shared_rank(&sh.fh2[255 - t], 0);
      uint32_t total;
      const uint32_t inc = block_incl_scan<uint32_t, NT>(h, sh.uscr, &total);
      if (inc >= want && inc - h < want) {
        sh.ctl[kCtlT] = (hb << 8) | static_cast<uint32_t>(255 - t);
        sh.ctl[kCtlNgt] = n_above + inc - h;
      }
      __syncthreads();
    }
    T = sh.ctl[kCtlT];
    n_gt = sh.ctl[kCtlNgt];

    // counts of keys > T and == T per thread, then per rank
    for_chunks([&](int e0, const uint4& v) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w = word_of(v, q);
        const uint32_t k0 = order_key(w & 0xFFFFu), k1 = order_key(w >> 16);
        if (e0 + 2 * q < V) {
          ngt += k0 > T;
          ntie += k0 == T;
        }
        if (e0 + 2 * q + 1 < V) {
          ngt += k1 > T;
          ntie += k1 == T;
        }
      }
    });
    uint32_t tie_total;
    gt_off = block_incl_scan<uint32_t, NT>(ngt, sh.uscr, &gt_rank) - ngt;
    block_incl_scan<uint32_t, NT>(ntie, sh.uscr, &tie_total);
    if (t < S) {
      cluster.map_shared_rank(sh.cnt, t)[s] = gt_rank;
      cluster.map_shared_rank(sh.cnt2, t)[s] = tie_total;
    }
    cluster.sync();  // F3b
    for (int r = 0; r < s; ++r) {
      gt_base += sh.cnt[r];
      tie_base += sh.cnt2[r];
    }
  }
  const uint32_t need = static_cast<uint32_t>(kk) - n_gt;
  // a rank with no key above T whose first tie ranks past the kept ones contributes nothing
  if (gt_rank == 0u && tie_base >= need) return kk;
  // keys strictly above T, and the ties at T ranked in id order (chunk_base is the same in every
  // thread of the rank, so the scan is skipped by all of them once the kept ties are placed)
  uint32_t slot = gt_base + gt_off;
  uint32_t chunk_base = tie_base;
  for_chunks([&](int e0, const uint4& v) {
    uint32_t mask = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w = word_of(v, q);
      const uint32_t k0 = order_key(w & 0xFFFFu), k1 = order_key(w >> 16);
      if (e0 + 2 * q < V) {
        if (k0 > T) lsurv[slot++] = pack(k0, id_base + e0 + 2 * q);
        if (k0 == T) mask |= 1u << (2 * q);
      }
      if (e0 + 2 * q + 1 < V) {
        if (k1 > T) lsurv[slot++] = pack(k1, id_base + e0 + 2 * q + 1);
        if (k1 == T) mask |= 1u << (2 * q + 1);
      }
    }
    if (chunk_base < need) {
      const uint32_t cnt = __popc(mask);
      uint32_t ctot;
      const uint32_t excl = block_incl_scan<uint32_t, NT>(cnt, sh.uscr, &ctot) - cnt;
      uint32_t rank = chunk_base + excl;
      while (mask != 0u && rank < need) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1;
        lsurv[n_gt + rank] = pack(T, id_base + e0 + j);
        ++rank;
      }
      chunk_base += ctot;
    }
  });
  return kk;
}



// Resident CTAs per SM the register budget must allow: the row slice lives in 4*C registers.
constexpr int min_ctas_for(int C) { return C <= 10 ? 4 : (C <= 12 ? 3 : 2); }

// Cluster-kernel residency: the small-chunk variants serve small batches (at most 32 rows of 16
// CTAs), so they trade residency for registers; C = 10 serves batches up to 127 rows at 8 CTAs.
constexpr int cluster_min_ctas(int C) { return C <= 6 ? 2 : (C <= 10 ? 3 : min_ctas_for(C)); }

template <int DT, int C>
__global__ void __launch_bounds__(NT, cluster_min_ctas(C)) fs_cluster_kernel(const Params p) {
  cg::cluster_group cluster = cg::this_cluster();
  const int S = static_cast<int>(cluster.num_blocks());
  const int s = static_cast<int>(cluster.block_rank());
  const int b = blockIdx.y;
  const int t = threadIdx.x;
  const bool leader = (s == 0);
  const int V = p.vocab;

  Shared& sh = *reinterpret_cast<Shared*>(g_smem);
  uint64_t* surv = reinterpret_cast<uint64_t*>(g_smem + sizeof(Shared));
  float* prob = reinterpret_cast<float*>(surv + p.cap);
  float* cum = prob + p.cap;
  uint64_t* tmp = reinterpret_cast<uint64_t*>(prob);  // prob/cum region viewed as cap words

  cluster_arrive();  // B1 (split): waited for only before the first remote access

  // Programmatic dependent launch: this grid may have started while the previous kernel of the
  // stream was still running. Unless the caller marked the logits complete at enqueue (p.early: no
  // running kernel writes them), L2 is warmed with this CTA's part of the row meanwhile and the
  // reads below wait for that kernel (and its writes); marked logits are read right away, so
  // that their transfer overlaps that kernel, and the next kernel of the stream may start its
  // launch at once (several calls on ready inputs then have their transfers in flight together).
  // Otherwise the next kernel may start its launch once this one has waited.
  if (!p.early) {
    prefetch_row_l2(p.logits, p.row_stride, V, b, static_cast<int64_t>(s) * C * NT * 16, C * NT * 16, t, NT);
    grid_dependency_wait();
  } else {
    grid_launch_dependents();  // the next call may start its own reads now (it waits for this one)
  }

  // ---- issue every load of this thread's slice (one read of the row) ----
  const uint16_t* row = p.logits + static_cast<int64_t>(b) * p.row_stride;
  const int vbase = s * C * NT;
  uint4 v[C];
  if (p.vec && (vbase + C * NT) * 8 <= V) {
    // whole slice in bounds and 16-byte aligned: one straight run of vector loads
    const uint4* rv = reinterpret_cast<const uint4*>(row) + vbase + t;
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = __ldg(rv + c * NT);
  } else {
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = load_chunk<DT>(row, (vbase + c * NT + t) * 8, V, p.vec);
  }
  if (p.early) grid_dependency_wait();
  else grid_launch_dependents();

  int kk;
  float pp;
  bool bad;
  row_params(p, b, &kk, &pp, &bad);
  const float u = (leader && t < 32) ? row_uniform(p, b) : 0.0f;

  sh.h1[t] = 0u;
  sh.h2[t] = 0u;
  if (leader) {
    sh.fh1[t] = 0u;
    sh.fh2[t] = 0u;
  }
  if (t < 16) sh.ctl[t] = 0u;

  // ---- phase 1: sub-chunk maxima ----
  // Per-chunk pair maxima (each half: the max of 4 logits of the chunk): folded, they give 1-2
  // maxima per thread; in phase 4 they tell which chunks hold a survivor. Finer maxima (4 or 8
  // per thread) come from per-word columns.
  uint32_t cp[C];
#pragma unroll
  for (int c = 0; c < C; ++c)
    cp[c] = pair_max_nan<DT>(pair_max_nan<DT>(v[c].x, v[c].y), pair_max_nan<DT>(v[c].z, v[c].w));
  uint32_t m16[8];
  int nm;
  if (p.mpt >= 4) {
    uint32_t mx[4] = {Fmt<DT>::kNegInf2, Fmt<DT>::kNegInf2, Fmt<DT>::kNegInf2, Fmt<DT>::kNegInf2};
#pragma unroll
    for (int c = 0; c < C; ++c) {
#pragma unroll
      for (int q = 0; q < 4; ++q) mx[q] = pair_max_nan<DT>(mx[q], word_of(v[c], q));
    }
    if (p.mpt == 8) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        m16[2 * q] = mx[q] & 0xFFFFu;
        m16[2 * q + 1] = mx[q] >> 16;
      }
      nm = 8;
    } else {
      const uint32_t a = pair_max_nan<DT>(mx[0], mx[2]), c2 = pair_max_nan<DT>(mx[1], mx[3]);
      m16[0] = a & 0xFFFFu;
      m16[1] = a >> 16;
      m16[2] = c2 & 0xFFFFu;
      m16[3] = c2 >> 16;
      nm = 4;
    }
  } else {
    uint32_t a = cp[0];
#pragma unroll
    for (int c = 1; c < C; ++c) a = pair_max_nan<DT>(a, cp[c]);
    if (p.mpt == 2) {
      m16[0] = a & 0xFFFFu;
      m16[1] = a >> 16;
      nm = 2;
    } else {
      uint32_t m1 = half_max_nan<DT>(a & 0xFFFFu, a >> 16);
      for (int off = 1; off < p.mgroup; off <<= 1)
        m1 = half_max_nan<DT>(m1, __shfl_xor_sync(0xFFFFFFFFu, m1, off));
      m16[0] = m1;
      nm = ((t & (p.mgroup - 1)) == 0) ? 1 : 0;
    }
  }
  if (p.stop == 1) {
    cluster_wait();
    if (leader && t == 0) p.out[b] = static_cast<int64_t>(m16[0]);
    return;
  }

  // ---- phase 2: keys of this rank's maxima and its row flags, then copies in every rank ----
  uint32_t flags = 0u;
  const int mbase = s * p.mcta + (t / p.mgroup) * p.mpt;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i >= nm) break;
    const uint32_t bits = m16[i];
    if (Fmt<DT>::is_nan(bits)) {
      flags |= kFlagNaN;
    } else {
      if (bits == Fmt<DT>::kPosInf) flags |= kFlagPosInf;
      if (bits != Fmt<DT>::kNegInf) flags |= kFlagAboveNegInf;
    }
    sh.mkeys[mbase + i] = order_key(bits);
  }
  flags = __reduce_or_sync(0xFFFFFFFFu, flags);
  if ((t & 31) == 0) sh.uscr[kUscrFlags + (t >> 5)] = flags;
  __syncthreads();
  cluster_wait();  // B1: every rank of the cluster is running
  {
    const int own = s * p.mcta;
    const int total = p.mcta * (S - 1);
    for (int i = t; i < total; i += NT) {
      const int ro = i / p.mcta;
      const int j = i - ro * p.mcta;
      const int r = ro < s ? ro : ro + 1;
      st_dsmem(dsmem_addr(&sh.mkeys[own + j], static_cast<uint32_t>(r)), sh.mkeys[own + j]);
    }
    if (t < S) {
      uint32_t f = 0u;
#pragma unroll
      for (int w = 0; w < NT / 32; ++w) f |= sh.uscr[kUscrFlags + w];
      st_dsmem(dsmem_addr(&sh.flags[s], static_cast<uint32_t>(t)), f);
    }
  }
  cluster.sync();  // B2: every rank holds every rank's maxima and flags
  if (p.stop == 2) {
    if (leader && t == 0) p.out[b] = static_cast<int64_t>(sh.flags[0]);
    return;
  }

  // ---- phase 3: the k-th largest maximum, searched locally by every rank ----
  // Up to 512 maxima, warp 0 alone finds it with one anchored histogram; otherwise (or when the
  // maxima spread wider than that histogram) the CTA runs the two-level radix select.
  const int nmax = S * p.mcta;
  constexpr uint32_t kNoKey = 0xFFFFFFFFu;
  if (t < 32) {
    uint32_t f = t < S ? sh.flags[t] : 0u;
    f = __reduce_or_sync(0xFFFFFFFFu, f);
    int st = FS_ROW_OK;
    if (bad) st = FS_ROW_BAD_PARAM;
    else if (f & kFlagNaN) st = FS_ROW_NAN;
    else if (f & kFlagPosInf) st = FS_ROW_POSINF;
    else if (!(f & kFlagAboveNegInf)) st = FS_ROW_ALL_NEGINF;
    if (t == 0) sh.ctl[kCtlStatus] = static_cast<uint32_t>(st);
    uint32_t lk = kNoKey;
    if (nmax <= 512) {
      constexpr int kSh = DT ? 0 : 2;  // bf16: one key per bin; fp16: four (same span in value)
      bool clamped = false;
      const uint32_t kth = warp_anchored_kth(sh.mkeys, nmax, kk, kSh, sh.h1, &clamped);
      if (!clamped) lk = max(kth, order_key(Fmt<DT>::kNegInf));
    }
    if (t == 0) sh.ctl[kCtlLKey] = lk;
  }
  __syncthreads();
  if (sh.ctl[kCtlLKey] == kNoKey) {
    sh.h1[t] = 0u;  // (the warp's histogram may have used it)
    __syncthreads();
    const uint32_t kth = kth_largest_key(sh.mkeys, nmax, kk, sh.h1, sh.h2, &sh.ctl[kCtlScr0]);
    if (t == 0) sh.ctl[kCtlLKey] = max(kth, order_key(Fmt<DT>::kNegInf));
    __syncthreads();
  }
  const int st = static_cast<int>(sh.ctl[kCtlStatus]);
  if (st != FS_ROW_OK) {
    // every remote access of this launch is complete (B2), so ranks may leave independently
    if (leader) write_invalid_row(p, b, st);
    return;
  }
  const uint32_t lkey = sh.ctl[kCtlLKey];
  if (p.stop == 3) {
    if (leader && t == 0) p.out[b] = static_cast<int64_t>(lkey);
    return;
  }

  // ---- phase 4: survivors (every element >= L) into the leader's buffer ----
  // The per-chunk maxima mark the chunks holding an element >= L (one packed compare per chunk).
  // Each lane counts the hits of its marked chunks, a warp scan gives every lane its offset, and
  // one lane per warp reserves the warp's positions with one atomic on the leader's counter (a
  // row made mostly of ties would otherwise send an atomic per chunk to that one counter); then
  // each thread takes its marked chunks out of its registers one at a time and stores the hits,
  // so the leader's survivors are contiguous when the cluster barrier completes.
  const uint32_t lbits = key_to_bits(lkey);
  const uint32_t l2 = lbits | (lbits << 16);
  const uint32_t cap = static_cast<uint32_t>(p.cap);
  const uint32_t surv0 = dsmem_addr(surv, 0);
  const uint32_t ctr = dsmem_addr(&sh.ctl[kCtlN], 0);
  uint32_t cm = 0u;
#pragma unroll
  for (int c = 0; c < C; ++c) cm |= (pair_ge_mask<DT>(cp[c], l2) != 0u ? 1u : 0u) << c;
  // bit 2w + h of chunk_hits(x, e0): half h of word w of the chunk is >= L (past the row end: 0)
  auto chunk_hits = [&](const uint4& x, int e0) -> uint32_t {
    uint32_t hits = 0u;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t m = pair_ge_mask<DT>(word_of(x, w), l2);
      hits |= ((m & 1u) | ((m >> 15) & 2u)) << (2 * w);
    }
    if (e0 + 8 > V) hits &= (e0 < V) ? ((1u << (V - e0)) - 1u) : 0u;
    return hits;
  };
  // chunk c of this thread's slice, out of the registers (predicated selects, no local memory)
  auto chunk_at = [&](int c) -> uint4 {
    uint4 x = v[0];
#pragma unroll
    for (int cc = 1; cc < C; ++cc)
      if (c == cc) x = v[cc];
    return x;
  };
  uint32_t nmine = 0u;
  for (uint32_t m = cm; m != 0u; m &= m - 1u) {
    const int c = __ffs(m) - 1;
    nmine += static_cast<uint32_t>(__popc(chunk_hits(chunk_at(c), (vbase + c * NT + t) * 8)));
  }
  const uint32_t lane_incl = warp_incl_scan(nmine);
  const uint32_t wtot = __shfl_sync(0xFFFFFFFFu, lane_incl, 31);
  uint32_t wbase = 0u;
  if ((t & 31) == 31 && wtot != 0u) wbase = atom_add_dsmem(ctr, wtot);
  uint32_t slot = __shfl_sync(0xFFFFFFFFu, wbase, 31) + lane_incl - nmine;
  while (cm != 0u) {
    const int c = __ffs(cm) - 1;
    cm &= cm - 1u;
    const uint4 x = chunk_at(c);
    const int e0 = (vbase + c * NT + t) * 8;
    uint32_t hits = chunk_hits(x, e0);
    while (hits != 0u) {
      const int bit = __ffs(hits) - 1;
      hits &= hits - 1u;
      const int w = bit >> 1;
      const uint32_t word = w == 0 ? x.x : w == 1 ? x.y : w == 2 ? x.z : x.w;
      if (slot < cap)
        st_dsmem64(surv0 + 8u * slot, pack(order_key((word >> (16 * (bit & 1))) & 0xFFFFu), p.id_base + e0 + bit));
      ++slot;
    }
  }
  cluster.sync();  // B4: the leader's survivors and count are final
  int n = static_cast<int>(leader ? sh.ctl[kCtlN] : ld_dsmem(ctr));
  const bool overflow = n > static_cast<int>(cap);  // the same decision in every rank
  if (overflow) {
    uint64_t* lsurv = cluster.map_shared_rank(surv, 0);
    n = exact_select<DT, C>(sh, row, V, p.vec, p.id_base, vbase, kk, lsurv, lkey);
    cluster.sync();  // F4: the leader holds exactly kk candidates at [0, kk)
  }
  // Ranks other than the leader are done. The leader waits for their arrival before it exits,
  // so its shared memory outlives their last read of it.
  cluster_arrive_relaxed();
  if (!leader) return;

  // ---- phases 5-7 in the leader: sort, tail ----
  if (p.stop == 4) {
    if (t == 0) p.out[b] = static_cast<int64_t>(n);
  } else {
    // the maxima keys are dead: their space holds the sorted top kk (else the survivors move to
    // the probability buffers, which the sort may overwrite, and the top kk goes back to surv)
    uint64_t* src = surv;
    uint64_t* dst = reinterpret_cast<uint64_t*>(sh.mkeys);
    if (kk > kMaxMaxima / 2) {
      for (int i = t; i < n; i += NT) tmp[i] = surv[i];
      __syncthreads();
      src = tmp;
      dst = surv;
    }
    finish_row<DT>(p, b, src, n, dst, kk, pp, u, prob, cum, sh);
  }
  cluster_wait();
}

// ------------------------------------------------------------------------------------------
// Wide path: top-k beyond the survivor buffer, up to k = V (top-p only). Nothing is sorted.
// The probability of an element depends only on its 16-bit key, so the sorted order (value
// desc, id asc) is a sequence of key groups, and every cumulative sum the tail needs is a sum of
// (group size x group probability) over the groups above a point. Five launches in one
// programmatic-dependent-launch chain (a clear of the histograms, then these four), plain CTAs,
// no cluster:
//   fs_wide_hist_kernel  (S x B CTAs) one read of each row slice: the per-key element counts of
//                        the row (a [B, 65536] histogram in the workspace; lanes holding the same
//                        key add once), and the slice's maximum and row flags;
//   fs_wide_row_kernel   (one 1024-thread CTA per row, 64 keys per thread, from the largest key
//                        down) the k-th key T and the `need` lowest-id ties at T that the top-k
//                        takes; Z = sum of n_g * expf(x_g - m) in a fixed order; per key the
//                        probability p_g = fl(w_g / z), held as an integer in units of 2^-62
//                        (exact for every p >= 2^-39, so the masses add exactly and in any order);
//                        the cut: the exclusive-prefix condition !((c_i - p_i) < top_p), with c_i
//                        the float rounding of the exact cumulative sum, holds from some element
//                        on (c is non-decreasing and p non-increasing along the order): the first
//                        group whose last element meets it, then a binary search in the group;
//                        the draw: target = u * c_r and the first element with c_i >= target,
//                        found the same way. Result: the drawn key and its rank j among the
//                        elements holding that key (ids ascending);
//   fs_wide_count_kernel (S x B CTAs) per slice, the elements holding the drawn key;
//   fs_wide_pick_kernel  (S x B CTAs) the slice holding the j-th of them scans its chunks in id
//                        order and writes the token id.
// With p >= 2^-29 for every candidate the cumulative sums are the ones the one-warp tail
// accumulates in double, so the ids equal the other paths' for the same k.
// ------------------------------------------------------------------------------------------

constexpr int kKeys = 65536;                             // 16-bit order keys
constexpr int kRowThreads = 1024;                        // fs_wide_row_kernel
constexpr int kKeysPerThread = kKeys / kRowThreads;      // 64 consecutive keys per thread
constexpr int kWCacheKeys = 32768;  // fs_wide_row_kernel: per-key weights kept in shared memory
constexpr float kTwo62f = 4611686018427387904.0f;        // 2^62: fixed-point unit of a probability
constexpr float kTwoM62f = 2.168404344971008868e-19f;    // 2^-62

// Float rounding of an exact cumulative mass x (units of 2^-62).
__device__ __forceinline__ float fixed_to_float(uint64_t x) { return __fmul_rn(__ull2float_rn(x), kTwoM62f); }
// A probability in units of 2^-62 (exact for pr >= 2^-39).
__device__ __forceinline__ uint64_t prob_to_fixed(float pr) { return __float2ull_rn(__fmul_rn(pr, kTwo62f)); }

// Row slice of the wide path's S x B launches into registers (as the cluster kernel loads it).
template <int DT, int C>
__device__ __forceinline__ void load_slice(const Params& p, int b, int vbase, uint4 (&v)[C]) {
  const uint16_t* row = p.logits + static_cast<int64_t>(b) * p.row_stride;
  const int t = threadIdx.x;
  if (p.vec && (vbase + C * NT) * 8 <= p.vocab) {
    const uint4* rv = reinterpret_cast<const uint4*>(row) + vbase + t;
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = __ldg(rv + c * NT);
  } else {
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = load_chunk<DT>(row, (vbase + c * NT + t) * 8, p.vocab, p.vec);
  }
}

// Order key of element j (0..7) of a 16-byte chunk.
__device__ __forceinline__ uint32_t chunk_key(const uint4& x, int j) {
  return order_key((word_of(x, j >> 1) >> (16 * (j & 1))) & 0xFFFFu);
}

template <int DT, int C>
__global__ void __launch_bounds__(NT, min_ctas_for(C))
    fs_wide_hist_kernel(const Params p, uint32_t* __restrict__ hist, uint32_t* __restrict__ smax,
                        uint32_t* __restrict__ sflag) {
  __shared__ uint32_t wf[NT / 32], wm[NT / 32];
  grid_dependency_wait();  // the stream's previous work (histogram clear, the logits) is done
  grid_launch_dependents();
  const int S = static_cast<int>(gridDim.x);
  const int s = blockIdx.x;
  const int b = blockIdx.y;
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int V = p.vocab;
  const int vbase = s * C * NT;
  uint4 v[C];
  load_slice<DT, C>(p, b, vbase, v);
  uint32_t* hrow = hist + static_cast<size_t>(b) * kKeys;
  uint32_t acc = Fmt<DT>::kNegInf2;
  uint32_t kmin = 0xFFFFu;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    acc = pair_max_nan<DT>(acc, pair_max_nan<DT>(pair_max_nan<DT>(v[c].x, v[c].y), pair_max_nan<DT>(v[c].z, v[c].w)));
    const int e0 = (vbase + c * NT + t) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool valid = e0 + j < V;
      const uint32_t key = chunk_key(v[c], j);
      const unsigned peers = __match_any_sync(0xFFFFFFFFu, valid ? key : 0xFFFFFFFFu);
      if (valid && lane == __ffs(peers) - 1) atomicAdd(&hrow[key], static_cast<uint32_t>(__popc(peers)));
      if (valid) kmin = min(kmin, key);
    }
  }
  const uint32_t mbits = half_max_nan<DT>(acc & 0xFFFFu, acc >> 16);
  uint32_t flags = 0u;
  if (Fmt<DT>::is_nan(mbits)) {
    flags |= kFlagNaN;
  } else {
    if (mbits == Fmt<DT>::kPosInf) flags |= kFlagPosInf;
    if (mbits != Fmt<DT>::kNegInf) flags |= kFlagAboveNegInf;
  }
  const uint32_t f = __reduce_or_sync(0xFFFFFFFFu, flags);
  const uint32_t m = __reduce_max_sync(0xFFFFFFFFu, Fmt<DT>::is_nan(mbits) ? 0u : order_key(mbits));
  const uint32_t mn = __reduce_min_sync(0xFFFFFFFFu, kmin);
  if (lane == 0) {
    wf[t >> 5] = f | (mn << 16);
    wm[t >> 5] = m;
  }
  __syncthreads();
  if (t == 0) {
    uint32_t ff = 0u, mm = 0u, mnn = 0xFFFFu;
    for (int w = 0; w < NT / 32; ++w) {
      ff |= wf[w] & 0xFFFFu;
      mnn = min(mnn, wf[w] >> 16);
      mm = max(mm, wm[w]);
    }
    // row flags in the low half, the slice's smallest key in the high half
    sflag[static_cast<size_t>(b) * S + s] = ff | (mnn << 16);
    smax[static_cast<size_t>(b) * S + s] = mm;
  }
}

// Per-row result of fs_wide_row_kernel: {row status, drawn key, its rank among the elements
// holding that key (ids ascending), 1 when the locate kernels have work}.
constexpr int kWideRes = 4;

// Elements of key `key` in the top-k: all of them above T, `need` at T, none below.
__device__ __forceinline__ uint32_t topk_count(uint32_t key, uint32_t count, uint32_t T, uint32_t need) {
  return key > T ? count : (key == T ? need : 0u);
}

template <int DT>
__global__ void __launch_bounds__(kRowThreads, 1)
    fs_wide_row_kernel(const Params p, const uint32_t* __restrict__ hist, const uint32_t* __restrict__ smax,
                       const uint32_t* __restrict__ sflag, uint32_t* __restrict__ res, int S) {
  __shared__ uint64_t qscr[40];
  __shared__ double dscr[40];
  __shared__ uint32_t uscr[40];
  __shared__ int iscr[40];
  __shared__ uint64_t found[4];
  grid_dependency_wait();  // the histogram launch is complete
  grid_launch_dependents();
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const int lane = t & 31;
  int kk;
  float pp;
  bool bad;
  row_params(p, b, &kk, &pp, &bad);
  // the slices' flags, smallest keys and maxima: each warp reads them a lane per slice
  uint32_t F = 0u, mkey = 0u, kmin = 0xFFFFu;
  for (int r = lane; r < S; r += 32) {
    const uint32_t w = sflag[static_cast<size_t>(b) * S + r];
    F |= w & 0xFFFFu;
    kmin = min(kmin, w >> 16);
    mkey = max(mkey, smax[static_cast<size_t>(b) * S + r]);
  }
  F = __reduce_or_sync(0xFFFFFFFFu, F);
  kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
  mkey = __reduce_max_sync(0xFFFFFFFFu, mkey);
  int st = FS_ROW_OK;
  if (bad) st = FS_ROW_BAD_PARAM;
  else if (F & kFlagNaN) st = FS_ROW_NAN;
  else if (F & kFlagPosInf) st = FS_ROW_POSINF;
  else if (!(F & kFlagAboveNegInf)) st = FS_ROW_ALL_NEGINF;
  const float mf = tail_logit<DT>(p, mkey);
  if (st == FS_ROW_OK && mf == INFINITY) st = FS_ROW_POSINF;  // the scaled maximum overflowed
  uint32_t* rr = res + static_cast<size_t>(b) * kWideRes;
  if (st != FS_ROW_OK) {
    if (t == 0) {
      rr[0] = static_cast<uint32_t>(st);
      rr[3] = 0u;
    }
    write_invalid_row(p, b, st, t, kRowThreads);
    return;
  }

  // The keys holding elements span [kmin, mkey]; thread t takes an equal share of that span
  // (rounded to whole 16-byte vectors), from the top down, so that the per-key work is spread over
  // every thread however narrow the span. each_key(fn) calls fn(key, count) for the thread's
  // keys in descending order (ascending in the sorted order), reading the counts in batches of
  // eight 16-byte loads issued together; fn returns true to stop.
  const uint32_t top = mkey | 3u, bot = min(kmin, mkey) & ~3u;
  const uint32_t span = top - bot + 1u;
  const uint32_t share = (((span + kRowThreads - 1) / kRowThreads) + 3u) & ~3u;
  const uint32_t mine_hi = static_cast<uint32_t>(t) * share < span ? top - static_cast<uint32_t>(t) * share : 0u;
  const uint32_t mine_lo = mine_hi >= bot + share - 1u ? mine_hi - share + 1u : bot;
  const int nvec = static_cast<uint32_t>(t) * share < span ? static_cast<int>((mine_hi - mine_lo + 1u) / 4u) : 0;
  const uint4* h4 = reinterpret_cast<const uint4*>(hist + static_cast<size_t>(b) * kKeys + mine_lo);
  // (the vectors of a batch are visited by a rolled loop, each picked out of the registers by
  // predicated selects: fn is instantiated 4 times per pass, not 32, which keeps the passes in
  // the instruction cache)
  auto each_key = [&](auto&& fn) {
#pragma unroll 1
    for (int v0 = nvec - 1; v0 >= 0; v0 -= 8) {
      uint4 w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = v0 - i >= 0 ? h4[v0 - i] : make_uint4(0u, 0u, 0u, 0u);
      const int nb = min(8, v0 + 1);
#pragma unroll 1
      for (int i = 0; i < nb; ++i) {
        uint4 x = w[0];
#pragma unroll
        for (int c = 1; c < 8; ++c)
          if (i == c) x = w[c];
        const uint32_t cnt[4] = {x.w, x.z, x.y, x.x};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t key = mine_lo + 4u * static_cast<uint32_t>(v0 - i) + 3u - static_cast<uint32_t>(j);
          if (fn(key, cnt[j])) return;
        }
      }
    }
  };

  // ---- the k-th key T and the ties `need` at T (k >= V: every element, T = 0) ----
  const uint32_t ukk = static_cast<uint32_t>(kk);
  uint32_t T = 0u, need = 0u;
  if (kk < p.vocab) {
    uint32_t csum = 0u;
    each_key([&](uint32_t, uint32_t n) {
      csum += n;
      return false;
    });
    uint32_t ctot = 0u;
    const uint32_t cbase = block_incl_scan<uint32_t, kRowThreads>(csum, uscr, &ctot) - csum;
    if (cbase < ukk && ukk <= cbase + csum) {
      uint32_t run = cbase;
      each_key([&](uint32_t key, uint32_t n) {
        if (run + n >= ukk) {
          uscr[36] = key;
          uscr[37] = ukk - run;
          return true;
        }
        run += n;
        return false;
      });
    }
    __syncthreads();
    T = uscr[36];
    need = uscr[37];
  }

  // ---- Z over the top-k, in a fixed order ----
  // The weights expf(x_g - m) are kept in shared memory (indexed by key - bot) when the span fits
  // kWCacheKeys, so the later passes read them back instead of evaluating them again; each
  // thread reads back only what it wrote itself (the owner's warp reads the owner's, after the
  // block barriers of the scans below).
  float* wc = reinterpret_cast<float*>(g_smem);
  const bool cache = span <= static_cast<uint32_t>(kWCacheKeys);
  double part = 0.0;
  each_key([&](uint32_t key, uint32_t cnt) {
    const uint32_t n = topk_count(key, cnt, T, need);
    if (n != 0u) {
      const float w = expf(tail_logit<DT>(p, key) - mf);
      if (cache) wc[key - bot] = w;
      part += static_cast<double>(n) * static_cast<double>(w);
    }
    return false;
  });
  auto weight = [&](uint32_t key) -> float { return cache ? wc[key - bot] : expf(tail_logit<DT>(p, key) - mf); };
  part = warp_sum(part);
  if (lane == 0) dscr[t >> 5] = part;
  __syncthreads();
  if (t == 0) {
    double zs = 0.0;
    for (int w = 0; w < kRowThreads / 32; ++w) zs += dscr[w];
    dscr[32] = zs;
  }
  __syncthreads();
  const float z = static_cast<float>(dscr[32]);

  // ---- the fixed-point mass above this thread's keys, and the probability of its last group ----
  uint64_t msum = 0ull;
  float last_pr = 0.0f;
  bool has = false;
  each_key([&](uint32_t key, uint32_t cnt) {
    const uint32_t n = topk_count(key, cnt, T, need);
    if (n != 0u) {
      last_pr = __fdiv_rn(weight(key), z);
      msum += static_cast<uint64_t>(n) * prob_to_fixed(last_pr);
      has = true;
    }
    return false;
  });
  uint64_t mtot = 0ull;
  const uint64_t mbase = block_incl_scan<uint64_t, kRowThreads>(msum, qscr, &mtot) - msum;
  const uint64_t mend = mbase + msum;  // the exact mass through this thread's last element

  // Both the cut and the draw conditions hold from some element of the sorted order on, so the
  // element is in the first thread whose last element meets the condition (the owner). The
  // owner's warp searches the owner's keys (at most 64): lane l takes the keys of ranks 2l and
  // 2l + 1 within the owner's share, a warp scan of their masses gives each group's start, and
  // the first lane holding a group whose last element meets the condition reports it (that lane
  // then finds the position inside the group by binary search). Returns that lane, -1 if none.
  constexpr int kNone = 0x7FFFFFFF;
  auto owner_group = [&](int owner, int mode, float target, uint64_t* start, uint32_t* n_out,
                         uint64_t* pf_out, float* pr_out, uint32_t* key_out) -> int {
    const int ol = owner & 31;
    const uint64_t ob = __shfl_sync(0xFFFFFFFFu, mbase, ol);
    const uint32_t ohi = __shfl_sync(0xFFFFFFFFu, mine_hi, ol);
    const int onk = 4 * __shfl_sync(0xFFFFFFFFu, nvec, ol);
    const uint32_t* hrow = hist + static_cast<size_t>(b) * kKeys;
    uint32_t n[2];
    float pr[2];
    uint64_t pf[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = 2 * lane + j;
      const uint32_t key = ohi - static_cast<uint32_t>(i);
      n[j] = i < onk ? topk_count(key, hrow[key], T, need) : 0u;
      pr[j] = n[j] != 0u ? __fdiv_rn(weight(key), z) : 0.0f;
      pf[j] = prob_to_fixed(pr[j]);
    }
    const uint64_t m0 = static_cast<uint64_t>(n[0]) * pf[0], m1 = static_cast<uint64_t>(n[1]) * pf[1];
    const uint64_t run0 = ob + warp_incl_scan<uint64_t>(m0 + m1) - (m0 + m1);
    const uint64_t ends[2] = {run0 + m0, run0 + m0 + m1};
    int hit = -1;
#pragma unroll
    for (int j = 1; j >= 0; --j) {
      const float c = fixed_to_float(ends[j]);
      if (n[j] != 0u && (mode == 0 ? !((c - pr[j]) < pp) : c >= target)) hit = j;
    }
    const int f = __ffs(__ballot_sync(0xFFFFFFFFu, hit >= 0)) - 1;
    if (lane == f) {
      *start = hit == 0 ? run0 : run0 + m0;
      *n_out = n[hit];
      *pf_out = pf[hit];
      *pr_out = pr[hit];
      *key_out = ohi - static_cast<uint32_t>(2 * lane + hit);
    }
    return f;
  };

  // ---- the cut: xr = the exact mass through r ----
  uint64_t xr = mtot;
  if (pp < 1.0f) {
    const bool meets = has && !((fixed_to_float(mend) - last_pr) < pp);
    const int owner = block_min<kRowThreads>(meets ? t : kNone, iscr);
    if (owner != kNone && (t >> 5) == (owner >> 5)) {
      uint64_t start = 0ull, pf = 0ull;
      uint32_t n = 0u, key = 0u;
      float pr = 0.0f;
      const int f = owner_group(owner, 0, 0.0f, &start, &n, &pf, &pr, &key);
      if (lane == f) {
        // the first position j of the group that meets the condition (it holds at j = n - 1)
        uint32_t lo = 0u, hi = n - 1u;
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (!((fixed_to_float(start + static_cast<uint64_t>(mid + 1u) * pf) - pr) < pp)) hi = mid;
          else lo = mid + 1u;
        }
        found[0] = start + static_cast<uint64_t>(lo) * pf;
      }
      if (f < 0 && lane == 0) found[0] = mtot;  // (not reached: the owner's last element meets it)
    }
    __syncthreads();
    if (owner != kNone) xr = found[0];
  }
  const float zp = fixed_to_float(xr);
  const float target = __fmul_rn(row_uniform(p, b), zp);

  // ---- the draw: the first element with c_i >= target ----
  const int owner = block_min<kRowThreads>(has && fixed_to_float(mend) >= target ? t : kNone, iscr);
  if (owner != kNone && (t >> 5) == (owner >> 5)) {
    uint64_t start = 0ull, pf = 0ull;
    uint32_t n = 0u, key = 0u;
    float pr = 0.0f;
    const int f = owner_group(owner, 1, target, &start, &n, &pf, &pr, &key);
    if (lane == f) {
      uint32_t lo = 0u, hi = n - 1u;
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (fixed_to_float(start + static_cast<uint64_t>(mid + 1u) * pf) >= target) hi = mid;
        else lo = mid + 1u;
      }
      rr[0] = static_cast<uint32_t>(FS_ROW_OK);
      rr[1] = key;
      rr[2] = lo;
      rr[3] = 1u;
    }
    if (f < 0 && lane == 0) {
      rr[0] = static_cast<uint32_t>(FS_ROW_OK);
      rr[3] = 0u;
    }
  }
  if (owner == kNone && t == 0) {  // (not reached: the last element meets the draw)
    rr[0] = static_cast<uint32_t>(FS_ROW_OK);
    rr[3] = 0u;
  }
}

template <int DT, int C>
__global__ void __launch_bounds__(NT, min_ctas_for(C))
    fs_wide_count_kernel(const Params p, const uint32_t* __restrict__ res, uint32_t* __restrict__ cnt) {
  __shared__ uint32_t scr[40];
  grid_dependency_wait();  // the row launch is complete
  grid_launch_dependents();
  const int S = static_cast<int>(gridDim.x);
  const int s = blockIdx.x;
  const int b = blockIdx.y;
  const int t = threadIdx.x;
  const uint32_t* rr = res + static_cast<size_t>(b) * kWideRes;
  if (rr[3] == 0u) {
    if (t == 0) cnt[static_cast<size_t>(b) * S + s] = 0u;
    return;
  }
  const uint32_t gkey = rr[1];
  const int vbase = s * C * NT;
  uint4 v[C];
  load_slice<DT, C>(p, b, vbase, v);
  uint32_t mine = 0u;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int e0 = (vbase + c * NT + t) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) mine += (e0 + j < p.vocab && chunk_key(v[c], j) == gkey) ? 1u : 0u;
  }
  const uint32_t total = block_sum<uint32_t, NT>(mine, scr);
  if (t == 0) cnt[static_cast<size_t>(b) * S + s] = total;
}

template <int DT, int C>
__global__ void __launch_bounds__(NT, min_ctas_for(C))
    fs_wide_pick_kernel(const Params p, const uint32_t* __restrict__ res, const uint32_t* __restrict__ cnt) {
  __shared__ uint32_t scr[40];
  grid_dependency_wait();  // the count launch (and, through it, the row launch) is complete
  grid_launch_dependents();
  const int S = static_cast<int>(gridDim.x);
  const int s = blockIdx.x;
  const int b = blockIdx.y;
  const int t = threadIdx.x;
  const uint32_t* rr = res + static_cast<size_t>(b) * kWideRes;
  if (rr[3] == 0u) return;
  const uint32_t gkey = rr[1], jpick = rr[2];
  uint32_t before = 0u;
  for (int r = 0; r < s; ++r) before += cnt[static_cast<size_t>(b) * S + r];
  const uint32_t here = cnt[static_cast<size_t>(b) * S + s];
  if (!(jpick >= before && jpick < before + here)) return;  // (the same in every thread)
  const int vbase = s * C * NT;
  uint4 v[C];
  load_slice<DT, C>(p, b, vbase, v);
  // chunks in id order: chunk c of every thread, threads in order, lanes in order
  uint32_t chunk_base = before;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int e0 = (vbase + c * NT + t) * 8;
    uint32_t hits = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (e0 + j < p.vocab && chunk_key(v[c], j) == gkey) hits |= 1u << j;
    const uint32_t n = static_cast<uint32_t>(__popc(hits));
    uint32_t ctot = 0u;
    const uint32_t excl = block_incl_scan<uint32_t, NT>(n, scr, &ctot) - n;
    if (jpick >= chunk_base + excl && jpick < chunk_base + excl + n) {
      for (uint32_t r = chunk_base + excl; r < jpick; ++r) hits &= hits - 1u;
      if (p.out != nullptr) p.out[b] = static_cast<int64_t>(p.id_base) + e0 + (__ffs(hits) - 1);
      if (p.status != nullptr) p.status[b] = FS_ROW_OK;
    }
    chunk_base += ctot;
  }
}

// ---- asynchronous copies (row merge) ------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

// Per-thread 16-byte global -> shared copy through L2 only (both addresses 16-byte aligned); the
// thread's copies are complete after cp_async_wait_all.
__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// Streaming path for large batches: two launches, no cross-CTA waiting.
//   fs_slice_kernel: one CTA per (slice, row). The slice is read once into registers; the CTA
//     keeps every element >= L_s, a lower bound on its own kk-th largest element (the kk-th
//     largest of about 4kk of its sub-chunk maxima, from one anchored histogram), and writes them
//     as packed candidates to cand[b][s][0..n) with n | flags << 24 in cnt[b][s]. A slice whose
//     survivors would not fit its M slots writes its exact top-kk instead. The union over the
//     slices holds the row's top-kk.
//   fs_rowmerge_kernel: four warps per row. They gather the slices' candidates (L2-resident),
//     keep those at or above a row bound from the slices' threshold ladders, rank them, and run
//     the same tail as the cluster kernel.
// ------------------------------------------------------------------------------------------

constexpr uint32_t kCountMask = 0xFFFFFFu;

// slice kernel: per-warp staging of marked chunks in dynamic shared memory after Shared
constexpr int kMarkedPerWarp = 64;                         // chunks per warp
constexpr int kMarkedBytesPerWarp = kMarkedPerWarp * 16;    // their data; then as many index words
constexpr int kSliceStageBytes = (NT / 32) * kMarkedPerWarp * (16 + 4);

// Exact top-kk of the span of `nchunks` CTA chunks starting at vector vbase (heavy ties), written
// to slots[0..) (global or shared memory): two 8-bit radix levels over the span (re-read from
// L1/L2) give the kk-th key T; the elements above T and the lowest-id ties at T (ranked in id
// order: chunk, thread, lane) are written. Returns min(kk, valid elements). Every thread of the
// CTA calls it.
template <int DT>
__device__ __noinline__ int span_exact_topk(Shared& sh, const uint16_t* __restrict__ row, int V, int vec,
                                            uint32_t id_base, int vbase, int nchunks, int kk, uint64_t* slots) {
  const int t = threadIdx.x;
  const int valid = max(0, min(V - vbase * 8, nchunks * NT * 8));
  const int want = min(kk, valid);
  if (want == 0) return 0;
  sh.h1[t] = 0u;
  sh.h2[t] = 0u;
  if (t == 0) sh.ctl[kCtlLocal] = 0u;
  __syncthreads();
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int e0 = (vbase + c * NT + t) * 8;
    const uint4 v = load_chunk<DT>(row, e0, V, vec);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w = word_of(v, q);
      if (e0 + 2 * q < V) atomicAdd(&sh.h1[order_key(w & 0xFFFFu) >> 8], 1u);
      if (e0 + 2 * q + 1 < V) atomicAdd(&sh.h1[order_key(w >> 16) >> 8], 1u);
    }
  }
  __syncthreads();
  if (t < 32) {
    uint32_t hb = 0u, above = 0u;
    warp_boundary_256(sh.h1, static_cast<uint32_t>(want), &hb, &above);
    if (t == 0) {
      sh.ctl[kCtlHb] = hb;
      sh.ctl[kCtlAbove] = above;
    }
  }
  __syncthreads();
  const uint32_t hb = sh.ctl[kCtlHb];
  const uint32_t n_above = sh.ctl[kCtlAbove];
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int e0 = (vbase + c * NT + t) * 8;
    const uint4 v = load_chunk<DT>(row, e0, V, vec);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w = word_of(v, q);
      const uint32_t k0 = order_key(w & 0xFFFFu), k1 = order_key(w >> 16);
      if (e0 + 2 * q < V && (k0 >> 8) == hb) atomicAdd(&sh.h2[k0 & 0xFFu], 1u);
      if (e0 + 2 * q + 1 < V && (k1 >> 8) == hb) atomicAdd(&sh.h2[k1 & 0xFFu], 1u);
    }
  }
  __syncthreads();
  if (t < 32) {
    uint32_t lb = 0u, above2 = 0u;
    warp_boundary_256(sh.h2, static_cast<uint32_t>(want) - n_above, &lb, &above2);
    if (t == 0) {
      sh.ctl[kCtlT] = (hb << 8) | lb;
      sh.ctl[kCtlNgt] = n_above + above2;
    }
  }
  __syncthreads();
  const uint32_t T = sh.ctl[kCtlT];
  const uint32_t n_gt = sh.ctl[kCtlNgt];
  const uint32_t need = static_cast<uint32_t>(want) - n_gt;
  uint32_t chunk_base = 0u;
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int e0 = (vbase + c * NT + t) * 8;
    const uint4 v = load_chunk<DT>(row, e0, V, vec);
    uint32_t mask = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w = word_of(v, q);
      const uint32_t k0 = order_key(w & 0xFFFFu), k1 = order_key(w >> 16);
      if (e0 + 2 * q < V) {
        if (k0 > T) slots[atomicAdd(&sh.ctl[kCtlLocal], 1u)] = pack(k0, id_base + e0 + 2 * q);
        if (k0 == T) mask |= 1u << (2 * q);
      }
      if (e0 + 2 * q + 1 < V) {
        if (k1 > T) slots[atomicAdd(&sh.ctl[kCtlLocal], 1u)] = pack(k1, id_base + e0 + 2 * q + 1);
        if (k1 == T) mask |= 1u << (2 * q + 1);
      }
    }
    const uint32_t cnt = __popc(mask);
    uint32_t ctot;
    const uint32_t excl = block_incl_scan<uint32_t, NT>(cnt, sh.uscr, &ctot) - cnt;
    uint32_t rank = chunk_base + excl;
    while (mask != 0u && rank < need) {
      const int j = __ffs(mask) - 1;
      mask &= mask - 1;
      slots[n_gt + rank] = pack(T, id_base + e0 + j);
      ++rank;
    }
    chunk_base += ctot;
  }
  return want;
}

template <int DT, int C>
__global__ void __launch_bounds__(NT, min_ctas_for(C)) fs_slice_kernel(const Params p, uint64_t* __restrict__ cand,
                                                                      uint64_t* __restrict__ lad,
                                                                      uint32_t* __restrict__ cnt) {
  const int S = static_cast<int>(gridDim.x);
  const int s = blockIdx.x;
  const int b = blockIdx.y;
  const int t = threadIdx.x;
  const int V = p.vocab;
  const uint32_t M = static_cast<uint32_t>(p.slot);
  Shared& sh = *reinterpret_cast<Shared*>(g_smem);

  // programmatic dependent launch: wait for the stream's previous kernel before reading, and let
  // the row merge launch once every slice CTA has started (it waits for this grid to finish)
  grid_dependency_wait();
  grid_launch_dependents();
  int kk;
  float pp;
  bool bad;
  row_params(p, b, &kk, &pp, &bad);

  const uint16_t* row = p.logits + static_cast<int64_t>(b) * p.row_stride;
  const int vbase = s * C * NT;
  uint4 v[C];
  const bool full = p.vec && (vbase + C * NT) * 8 <= V;
  if (full) {
    const uint4* rv = reinterpret_cast<const uint4*>(row) + vbase + t;
    const uint64_t pol = l2_evict_first_policy();
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = ldg_policy(rv + c * NT, pol);
  } else {
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = load_chunk<DT>(row, (vbase + c * NT + t) * 8, V, p.vec);
  }
  sh.h1[t] = 0u;
  if (t < 16) sh.ctl[t] = 0u;

  // Per-chunk pair maxima (each half: the max of 4 logits of the chunk) and their fold over the
  // thread's chunks; they give the sub-chunk maxima for 1 or 2 per thread, and later tell which
  // chunks hold a candidate. Finer maxima (4 or 8 per thread) come from per-word columns.
  uint32_t cp[C];
#pragma unroll
  for (int c = 0; c < C; ++c)
    cp[c] = pair_max_nan<DT>(pair_max_nan<DT>(v[c].x, v[c].y), pair_max_nan<DT>(v[c].z, v[c].w));
  uint32_t acc = cp[0];
#pragma unroll
  for (int c = 1; c < C; ++c) acc = pair_max_nan<DT>(acc, cp[c]);
  uint32_t m16[8];
  int nm;
  if (p.mpt >= 4) {
    uint32_t mx[4] = {Fmt<DT>::kNegInf2, Fmt<DT>::kNegInf2, Fmt<DT>::kNegInf2, Fmt<DT>::kNegInf2};
#pragma unroll
    for (int c = 0; c < C; ++c) {
#pragma unroll
      for (int q = 0; q < 4; ++q) mx[q] = pair_max_nan<DT>(mx[q], word_of(v[c], q));
    }
    if (p.mpt == 8) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        m16[2 * q] = mx[q] & 0xFFFFu;
        m16[2 * q + 1] = mx[q] >> 16;
      }
      nm = 8;
    } else {
      const uint32_t a = pair_max_nan<DT>(mx[0], mx[2]), c2 = pair_max_nan<DT>(mx[1], mx[3]);
      m16[0] = a & 0xFFFFu;
      m16[1] = a >> 16;
      m16[2] = c2 & 0xFFFFu;
      m16[3] = c2 >> 16;
      nm = 4;
    }
  } else if (p.mpt == 2) {
    m16[0] = acc & 0xFFFFu;
    m16[1] = acc >> 16;
    nm = 2;
  } else {
    m16[0] = half_max_nan<DT>(acc & 0xFFFFu, acc >> 16);
    nm = 1;
  }
  uint32_t flags = 0u;
  uint32_t mk[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i >= nm) break;
    const uint32_t bits = m16[i];
    if (Fmt<DT>::is_nan(bits)) {
      flags |= kFlagNaN;
    } else {
      if (bits == Fmt<DT>::kPosInf) flags |= kFlagPosInf;
      if (bits != Fmt<DT>::kNegInf) flags |= kFlagAboveNegInf;
    }
    mk[i] = order_key(bits);
  }
  flags = __reduce_or_sync(0xFFFFFFFFu, flags);
  if ((t & 31) == 0) sh.uscr[kUscrFlags + (t >> 5)] = flags;

  // L_s: at most kk of this slice's elements lie above the kk-th largest of its maxima (the
  // threshold's first barrier also publishes the zeroed histogram and counters, and the flags)
  constexpr int kSh = DT ? 0 : 2;  // bf16: one key per bin; fp16: four (same span in value)
  const uint32_t kth = anchored_threshold(mk, nm, kk, kSh, sh.h1, sh.uscr, order_key(Fmt<DT>::kNegInf),
                                          lad + static_cast<size_t>(b) * S + s);
  const uint32_t lkey = max(kth, order_key(Fmt<DT>::kNegInf));
  const uint32_t lbits = key_to_bits(lkey);
  const uint32_t l2 = lbits | (lbits << 16);

  // Filter: the per-chunk maxima mark the chunks of each thread that hold an element >= L (one
  // packed compare per chunk). The warp stages its marked chunks in shared memory (a scan of the
  // lanes' counts, predicated 16-byte stores) and hands one to each lane, which compares its 8
  // logits with L; one shared atomic per warp reserves the hits' slots. A warp with more marked
  // chunks than its staging room (heavy ties) takes them out of its registers one at a time.
  uint64_t* slots = cand + (static_cast<size_t>(b) * S + s) * M;
  uint32_t cm = 0u;
#pragma unroll
  for (int c = 0; c < C; ++c) cm |= (pair_ge_mask<DT>(cp[c], l2) != 0u ? 1u : 0u) << c;
  const int lane = t & 31;
  const uint32_t nmine = static_cast<uint32_t>(__popc(cm));
  const uint32_t incl = warp_incl_scan(nmine);
  const uint32_t wtotal = __shfl_sync(0xFFFFFFFFu, incl, 31);
  // the row's hits of one 8-logit chunk (bit 2w + h: half h of word w is >= L), past-the-end
  // elements cleared
  auto chunk_hits = [&](const uint4& x, int e0) -> uint32_t {
    uint32_t hits = 0u;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t m = pair_ge_mask<DT>(word_of(x, w), l2);
      hits |= ((m & 1u) | ((m >> 15) & 2u)) << (2 * w);
    }
    if (e0 + 8 > V) hits &= (e0 < V) ? ((1u << (V - e0)) - 1u) : 0u;
    return hits;
  };
  auto write_hits = [&](const uint4& x, int e0, uint32_t hits, uint32_t j) {
    while (hits != 0u) {
      const int bit = __ffs(hits) - 1;
      hits &= hits - 1u;
      const int w = bit >> 1;
      const uint32_t word = w == 0 ? x.x : w == 1 ? x.y : w == 2 ? x.z : x.w;
      if (j < M) slots[j] = pack(order_key((word >> (16 * (bit & 1))) & 0xFFFFu), p.id_base + e0 + bit);
      ++j;
    }
  };
  if (wtotal <= static_cast<uint32_t>(kMarkedPerWarp)) {
    uint4* stg = reinterpret_cast<uint4*>(g_smem + sizeof(Shared)) + (t >> 5) * kMarkedPerWarp;
    uint32_t* sidx = reinterpret_cast<uint32_t*>(g_smem + sizeof(Shared) + kMarkedBytesPerWarp * (NT / 32)) +
                     (t >> 5) * kMarkedPerWarp;
    uint32_t o = incl - nmine;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      if (cm & (1u << c)) {
        stg[o] = v[c];
        sidx[o] = static_cast<uint32_t>(c * NT + t);
        ++o;
      }
    }
    __syncwarp();
    for (uint32_t i0 = 0; i0 < wtotal; i0 += 32u) {
      const uint32_t i = i0 + static_cast<uint32_t>(lane);
      uint4 x = make_uint4(0u, 0u, 0u, 0u);
      int e0 = 0;
      uint32_t hits = 0u;
      if (i < wtotal) {
        x = stg[i];
        e0 = (vbase + static_cast<int>(sidx[i])) * 8;
        hits = chunk_hits(x, e0);
      }
      const uint32_t nh = static_cast<uint32_t>(__popc(hits));
      const uint32_t hincl = warp_incl_scan(nh);
      const uint32_t htot = __shfl_sync(0xFFFFFFFFu, hincl, 31);
      uint32_t hbase = 0u;
      if (lane == 31 && htot != 0u) hbase = atomicAdd(&sh.ctl[kCtlLocal], htot);
      hbase = __shfl_sync(0xFFFFFFFFu, hbase, 31);
      write_hits(x, e0, hits, hbase + hincl - nh);
    }
  } else {
    while (cm != 0u) {
      const int c = __ffs(cm) - 1;
      cm &= cm - 1u;
      uint4 x = v[0];
#pragma unroll
      for (int cc = 1; cc < C; ++cc)
        if (c == cc) x = v[cc];
      const int e0 = (vbase + c * NT + t) * 8;
      const uint32_t hits = chunk_hits(x, e0);
      if (hits == 0u) continue;
      write_hits(x, e0, hits, atomicAdd(&sh.ctl[kCtlLocal], static_cast<uint32_t>(__popc(hits))));
    }
  }
  __syncthreads();
  const uint32_t total = sh.ctl[kCtlLocal];
  uint32_t written = total;
  if (total > M) {
    __syncthreads();  // every thread has read the count before the fallback resets it
    written = static_cast<uint32_t>(span_exact_topk<DT>(sh, row, V, p.vec, p.id_base, vbase, C, kk, slots));
  }
  if (t == 0) {
    uint32_t f = 0u;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) f |= sh.uscr[kUscrFlags + w];
    cnt[static_cast<size_t>(b) * S + s] = written | (f << 24);
  }
}

// Row merge: kMergeRowWarps warps per row, merge_rows_per_cta rows per CTA; a row's warps meet at
// the row group's own named barrier, never at a block barrier. Per-row shared memory: a control
// word (the compaction counter), a 256-bin histogram and 256 bin cursors, the row's candidate
// slots as copied (capn), the compacted survivors (capn), the sorted top kk and the
// probabilities of the tail.
constexpr int kMergeRowWarps = 4;
constexpr int kMergeRowThreads = 32 * kMergeRowWarps;

__host__ __device__ constexpr size_t merge_row_bytes(int capn, int K) {
  return (16 + 2048 + 2 * static_cast<size_t>(capn) * 8 + static_cast<size_t>(K) * 8 +
          static_cast<size_t>(K) * 4 + 15) &
         ~static_cast<size_t>(15);
}

// Rows per row-merge CTA that fit the shared memory budget (at least 1: capn <= kMaxMaxima and
// K <= 256 need at most 71 KB per row).
__host__ __device__ constexpr int merge_rows_per_cta(int capn, int K) {
  return (200u * 1024u) / merge_row_bytes(capn, K) >= 2 ? 2 : 1;
}

// The need-th largest low word (0xFFFFFFFF - id: the need-th smallest id) among the n gathered
// candidates whose key is E: four 8-bit radix levels (one warp).
__device__ __noinline__ uint32_t warp_tie_cut(const uint64_t* g, uint32_t n, uint32_t E, uint32_t need,
                                              uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0u;
  for (int level = 3; level >= 0; --level) {
    const int sh = 8 * level;
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0u;
    __syncwarp();
    for (uint32_t d = lane; d < n; d += 32) {
      const uint64_t x = g[d];
      const uint32_t lo = static_cast<uint32_t>(x);
      const bool match = packed_key(x) == E && (level == 3 || (lo >> (sh + 8)) == (prefix >> (sh + 8)));
      if (match) atomicAdd(&hist[(lo >> sh) & 0xFFu], 1u);
    }
    __syncwarp();
    uint32_t bin = 0u, above = 0u;
    warp_boundary_256(hist, need, &bin, &above);
    prefix |= bin << sh;
    need -= above;
    __syncwarp();
  }
  return prefix;
}

// The top kk of the n distinct packed values g[0..n) in descending order into dst (one warp):
// each value's rank is the count of larger ones. For n <= 32 R, R values per lane are ranked
// together against pairs of the list (16-byte loads; g[n] is padded with 0, below every packed
// candidate, whose low word 0xFFFFFFFF - id is never 0); larger n rank one value at a time.
// g must be 16-byte aligned with room for g[n].
template <int R>
__device__ __forceinline__ void warp_rank_top_regs(uint64_t* g, uint32_t n, uint32_t kk, uint64_t* dst) {
  const int lane = threadIdx.x & 31;
  if ((n & 1u) && lane == 0) g[n] = 0ull;
  __syncwarp();
  uint64_t x[R];
  uint32_t r[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    x[i] = lane + 32u * i < n ? g[lane + 32u * i] : 0ull;
    r[i] = 0u;
  }
  const ulonglong2* g2 = reinterpret_cast<const ulonglong2*>(g);
  const uint32_t np = (n + 1u) >> 1;
#pragma unroll 4
  for (uint32_t j = 0; j < np; ++j) {
    const ulonglong2 y = g2[j];
#pragma unroll
    for (int i = 0; i < R; ++i) r[i] += (y.x > x[i] ? 1u : 0u) + (y.y > x[i] ? 1u : 0u);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < R; ++i)
    if (lane + 32u * i < n && r[i] < kk) dst[r[i]] = x[i];
}

__device__ __forceinline__ void warp_rank_top(uint64_t* g, uint32_t n, uint32_t kk, uint64_t* dst) {
  const int lane = threadIdx.x & 31;
  if (n <= 96u) {
    warp_rank_top_regs<3>(g, n, kk, dst);
  } else if (n <= 192u) {
    warp_rank_top_regs<6>(g, n, kk, dst);
  } else {
    for (uint32_t i = lane; i < n; i += 32) {
      const uint64_t x = g[i];
      uint32_t rank = 0u;
      for (uint32_t j = 0; j < n; ++j) rank += g[j] > x ? 1u : 0u;
      if (rank < kk) dst[rank] = x;
    }
  }
  __syncwarp();
}

// Top kk of the n (>= 1) distinct packed values g[0..n) in descending order into dst, by a
// counting sort on the 16-bit key (one warp): bins from the largest key down, the values
// scattered into t[0..n) grouped by bin, and each value of a bin that starts below kk ranked
// among the bin's values. Returns false, having written nothing, when the keys span more than
// 256 values or a bin holds more than 64 (heavy ties); the caller then ranks another way.
// hist, cursor: 256 shared words each, 16-byte aligned; t must not overlap g.
__device__ bool warp_count_rank_top(const uint64_t* g, uint32_t n, uint32_t kk, uint32_t* hist, uint32_t* cursor,
                                    uint64_t* t, uint64_t* dst) {
  const int lane = threadIdx.x & 31;
  uint32_t kmax = 0u, kmin = 0xFFFFu;
  for (uint32_t d = lane; d < n; d += 32) {
    const uint32_t k = packed_key(g[d]);
    kmax = max(kmax, k);
    kmin = min(kmin, k);
  }
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
  if (kmax - kmin > 255u) return false;
  uint4* h4 = reinterpret_cast<uint4*>(hist);
  h4[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
  h4[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
  __syncwarp();
  for (uint32_t d = lane; d < n; d += 32) atomicAdd(&hist[kmax - packed_key(g[d])], 1u);
  __syncwarp();
  // exclusive prefix over the bins from the largest key (lane l owns bins 8l .. 8l+7)
  const uint4 a = h4[2 * lane], b = h4[2 * lane + 1];
  const uint32_t cnt[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t acc = 0u, big = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    acc += cnt[j];
    big = max(big, cnt[j]);
  }
  if (__reduce_max_sync(0xFFFFFFFFu, big) > 64u) return false;
  uint32_t run = warp_incl_scan(acc) - acc;
  uint32_t st[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    st[j] = run;
    run += cnt[j];
  }
  uint4* c4 = reinterpret_cast<uint4*>(cursor);
  c4[2 * lane] = make_uint4(st[0], st[1], st[2], st[3]);
  c4[2 * lane + 1] = make_uint4(st[4], st[5], st[6], st[7]);
  __syncwarp();
  for (uint32_t d = lane; d < n; d += 32) {
    const uint64_t x = g[d];
    t[atomicAdd(&cursor[kmax - packed_key(x)], 1u)] = x;
  }
  __syncwarp();
  // cursor[bin] is now the bin's end and hist[bin] its size
  for (uint32_t q = lane; q < n; q += 32) {
    const uint64_t x = t[q];
    const uint32_t bin = kmax - packed_key(x);
    const uint32_t e = cursor[bin], s0 = e - hist[bin];
    if (s0 >= kk) continue;
    uint32_t r = s0;
    for (uint32_t j = s0; j < e; ++j) r += t[j] > x ? 1u : 0u;
    if (r < kk) dst[r] = x;
  }
  __syncwarp();
  return true;
}

// The top kk of the n survivors g[0, n) into dst[0, kk), by one warp: a counting sort on the key
// (t: room for n more candidates) when the keys span <= 256 values and no bin holds more than
// 64; else, for at most 192 of them, a rank by comparisons; else two 8-bit radix levels for the
// kk-th key E, the keys above E and the lowest-id ties at E compacted in place in g, then a rank.
__device__ __noinline__ void warp_select_top(uint64_t* g, uint32_t n, int kk, uint32_t* hist, uint32_t* cursor,
                                             uint64_t* t, uint64_t* dst) {
  const int lane = threadIdx.x & 31;
  const uint32_t ukk = static_cast<uint32_t>(kk);
  if (n >= ukk) {
    if (warp_count_rank_top(g, n, ukk, hist, cursor, t, dst)) return;
    if (n <= 192u) {
      warp_rank_top(g, n, ukk, dst);
      return;
    }
  }
  // the histogram path: high byte, then low byte inside the boundary bin
#pragma unroll
  for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0u;
  __syncwarp();
  for (uint32_t d = lane; d < n; d += 32) atomicAdd(&hist[packed_key(g[d]) >> 8], 1u);
  __syncwarp();
  uint32_t hb = 0u, above = 0u;
  warp_boundary_256(hist, ukk, &hb, &above);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0u;
  __syncwarp();
  for (uint32_t d = lane; d < n; d += 32) {
    const uint32_t key = packed_key(g[d]);
    if ((key >> 8) == hb) atomicAdd(&hist[key & 0xFFu], 1u);
  }
  __syncwarp();
  uint32_t lb = 0u, above2 = 0u;
  warp_boundary_256(hist, ukk - above, &lb, &above2);
  const uint32_t E = (hb << 8) | lb;
  const uint32_t need = ukk - (above + above2);  // ties to take at E
  const uint32_t eq = hist[lb];
  // more than 32 surplus ties at E: keep only the `need` lowest ids among them
  const bool cut = eq > need + 32u;
  const uint32_t tcut = cut ? warp_tie_cut(g, n, E, need, hist) : 0u;
  // compact in place (a kept candidate never moves up): keys above E and the kept ties
  uint32_t nsel = 0u;
  for (uint32_t d0 = 0; d0 < n; d0 += 32) {
    const uint32_t d = d0 + lane;
    const uint64_t x = d < n ? g[d] : 0ull;
    const uint32_t key = packed_key(x);
    const bool take = d < n && (key > E || (key == E && (!cut || static_cast<uint32_t>(x) >= tcut)));
    const unsigned ball = __ballot_sync(0xFFFFFFFFu, take);
    if (take) g[nsel + __popc(ball & ((1u << lane) - 1u))] = x;
    nsel += __popc(ball);
  }
  __syncwarp();
  // rank sort (packed values are distinct; nsel <= kk + 32): the top kk in order
  warp_rank_top(g, nsel, ukk, dst);
}

// Row merge of the streaming path, kMergeRowWarps warps per row.
//  1. The row's threads start 16-byte async copies of the row's S * M candidate slots into shared
//     memory (one L2 round trip for the whole row); every warp loads the slices' count words and
//     threshold ladders meanwhile (lanes 0..S-1).
//  2. A row-wide lower bound L* on the kk-th largest, computed by every warp from the same words:
//     slice s has at least n_j elements at or above its ladder key l_sj (n_j = ceil(kk/8),
//     ceil(kk/4), ceil(kk/2), kk), so any t with sum_s max{n_j : l_sj >= t} >= kk has kk elements
//     at or above it. L* is the largest such t among the ladder keys; L* >= every slice's own
//     bound l_s3, so every element of the row's top kk is in the lists and >= L*.
//  3. Warp w compacts the listed candidates >= L* of slices w, w + 4, ... into the survivor array
//     (usually a few dozen in all), reserving slots with one shared atomic per ballot step.
//  4. With kk <= n <= 256 survivors every thread ranks its survivors against all of them (packed
//     values are distinct, so the order the warps wrote them in does not matter); otherwise warp 0
//     selects (warp_select_top). Then warp 0 runs the tail shared with the cluster kernel.
// Every branch before the last barrier depends only on values all the row's warps computed
// alike, so they all take the same barriers.
template <int DT>
__global__ void __launch_bounds__(NT) fs_rowmerge_kernel(const Params p, const uint64_t* __restrict__ cand,
                                                         const uint64_t* __restrict__ lad,
                                                         const uint32_t* __restrict__ cnt, int S, int B) {
  const int lane = threadIdx.x & 31;
  const int rg = static_cast<int>(threadIdx.x) / kMergeRowThreads;  // row group in the CTA
  const int rt = static_cast<int>(threadIdx.x) - rg * kMergeRowThreads;  // thread in the row group
  const int w = rt >> 5;                                                 // warp in the row group
  const int rows = static_cast<int>(blockDim.x) / kMergeRowThreads;
  const int b = static_cast<int>(blockIdx.x) * rows + rg;
  // the slices' lists are complete only when the slice grid is: wait for it, then let the next
  // kernel of the stream start launching
  grid_dependency_wait();
  grid_launch_dependents();
  if (b >= B) return;  // the whole row group
  const uint32_t bar = 1u + static_cast<uint32_t>(rg);  // barrier 0 is the block's
  auto row_sync = [bar]() { asm volatile("bar.sync %0, %1;\n" ::"r"(bar), "r"(kMergeRowThreads) : "memory"); };
  const uint32_t M = static_cast<uint32_t>(p.slot);
  const int capn = p.cap;
  unsigned char* base = g_smem + merge_row_bytes(capn, p.K) * rg;
  uint32_t* ctl = reinterpret_cast<uint32_t*>(base);
  uint32_t* hist = ctl + 4;
  uint32_t* cursor = hist + 256;
  uint64_t* g = reinterpret_cast<uint64_t*>(cursor + 256);
  uint64_t* sv = g + capn;  // survivors
  uint64_t* dst = sv + capn;
  float* prob = reinterpret_cast<float*>(dst + p.K);

  // 1. the row's S * M slots -> g (capn >= S * M), 16-byte async copies spread over the row group
  const size_t row0 = static_cast<size_t>(b) * S;
  {
    const uint4* src = reinterpret_cast<const uint4*>(cand + row0 * M);
    uint4* g4 = reinterpret_cast<uint4*>(g);
    const uint32_t pairs = static_cast<uint32_t>(S) * M / 2u;
    for (uint32_t q = static_cast<uint32_t>(rt); q < pairs; q += kMergeRowThreads) cp_async_16(g4 + q, src + q);
  }
  const uint32_t wv = lane < S ? __ldcg(cnt + row0 + lane) : 0u;
  const uint64_t lw = lane < S ? __ldcg(lad + row0 + lane) : 0ull;

  int kk;
  float pp;
  bool bad;
  row_params(p, b, &kk, &pp, &bad);
  const uint32_t c = min(wv & kCountMask, M);  // (never above M; the clamp keeps reads in range)
  const uint32_t f = __reduce_or_sync(0xFFFFFFFFu, wv >> 24);

  // 2. L* from the ladders (every warp)
  const uint32_t ukk = static_cast<uint32_t>(kk);
  const uint32_t n0 = (ukk + 7u) / 8u, n1 = (ukk + 3u) / 4u, n2 = (ukk + 1u) / 2u;
  uint32_t lstar = 0u;
  for (int e0 = 0; e0 < 4 * S; e0 += 32) {
    const int e = e0 + lane;
    const uint64_t own = __shfl_sync(0xFFFFFFFFu, lw, (e >> 2) & 31);
    const uint32_t t = e < 4 * S ? static_cast<uint32_t>(own >> (16 * (e & 3))) & 0xFFFFu : 0u;
    uint32_t sum = 0u;
    for (int r = 0; r < S; ++r) {
      const uint64_t x = __shfl_sync(0xFFFFFFFFu, lw, r);
      const uint32_t l0 = static_cast<uint32_t>(x) & 0xFFFFu, l1 = static_cast<uint32_t>(x >> 16) & 0xFFFFu;
      const uint32_t l2 = static_cast<uint32_t>(x >> 32) & 0xFFFFu, l3 = static_cast<uint32_t>(x >> 48);
      sum += (l3 != 0u && l3 >= t)   ? ukk
             : (l2 != 0u && l2 >= t) ? n2
             : (l1 != 0u && l1 >= t) ? n1
             : (l0 != 0u && l0 >= t) ? n0
                                     : 0u;
    }
    if (t != 0u && sum >= ukk) lstar = max(lstar, t);
  }
  lstar = __reduce_max_sync(0xFFFFFFFFu, lstar);

  if (rt == 0) ctl[0] = 0u;
  // the copies land (each thread waits for its own, the barrier publishes them) before anything
  // reads g, and the counter is zeroed before anything adds to it
  cp_async_wait_all();
  row_sync();
  int st = FS_ROW_OK;
  if (bad) st = FS_ROW_BAD_PARAM;
  else if (f & kFlagNaN) st = FS_ROW_NAN;
  else if (f & kFlagPosInf) st = FS_ROW_POSINF;
  else if (!(f & kFlagAboveNegInf)) st = FS_ROW_ALL_NEGINF;
  if (st != FS_ROW_OK) {
    if (w == 0) write_invalid_row(p, b, st, lane, 32);
    return;  // every warp of the row (st is the same for all)
  }

  // 3. survivors >= L*: warp w takes slices w, w + kMergeRowWarps, ...
  const ulonglong2* g2 = reinterpret_cast<const ulonglong2*>(g);
  const unsigned lt = (1u << lane) - 1u;
  for (int r = w; r < S; r += kMergeRowWarps) {
    const uint32_t cr = __shfl_sync(0xFFFFFFFFu, c, r);
    for (uint32_t j0 = 0; j0 < cr; j0 += 64u) {
      const uint32_t j = j0 + 2u * lane;
      ulonglong2 x = make_ulonglong2(0ull, 0ull);
      if (j < cr) x = g2[(static_cast<uint32_t>(r) * M + j) >> 1];
      const bool k0 = j < cr && packed_key(x.x) >= lstar;
      const bool k1 = j + 1u < cr && packed_key(x.y) >= lstar;
      const unsigned b0 = __ballot_sync(0xFFFFFFFFu, k0), b1 = __ballot_sync(0xFFFFFFFFu, k1);
      const uint32_t nb = static_cast<uint32_t>(__popc(b0) + __popc(b1));
      uint32_t at = 0u;
      if (lane == 0 && nb != 0u) at = atomicAdd(&ctl[0], nb);
      at = __shfl_sync(0xFFFFFFFFu, at, 0);
      if (k0) sv[at + __popc(b0 & lt)] = x.x;
      if (k1) sv[at + __popc(b0) + __popc(b1 & lt)] = x.y;
    }
  }
  row_sync();
  const uint32_t n = ctl[0];

  // 4. the survivors' top kk
  if (n >= ukk && n <= 2u * kMergeRowThreads) {
    const ulonglong2* s2 = reinterpret_cast<const ulonglong2*>(sv);
    const uint32_t np = n >> 1;
    for (uint32_t i = static_cast<uint32_t>(rt); i < n; i += kMergeRowThreads) {
      const uint64_t x = sv[i];
      uint32_t r = 0u;
#pragma unroll 4
      for (uint32_t j = 0; j < np; ++j) {
        const ulonglong2 y = s2[j];
        r += (y.x > x ? 1u : 0u) + (y.y > x ? 1u : 0u);
      }
      if (n & 1u) r += sv[n - 1u] > x ? 1u : 0u;
      if (r < ukk) dst[r] = x;
    }
    row_sync();
    if (w != 0) return;
  } else {
    if (w != 0) return;
    warp_select_top(sv, n, kk, hist, cursor, g, dst);  // g is free: room for n candidates
  }
  __syncwarp();
  const float u = row_uniform(p, b);
  if (write_selection(p, b, dst, kk, lane, 32)) return;
  if (kk <= 32) sample_tail_warp<DT, 1>(p, b, dst, kk, pp, u, prob);
  else if (kk <= 64) sample_tail_warp<DT, 2>(p, b, dst, kk, pp, u, prob);
  else sample_tail_warp<DT, 8>(p, b, dst, kk, pp, u, prob);
}

// Merge of per-shard candidate blocks [parts, B, K + 1] for vocab-sharded tensor parallelism:
// one CTA per row, exact top-k over parts*K packed candidates, then the same tail.
template <int DT>
__global__ void __launch_bounds__(NT) fs_merge_kernel(const Params p, const uint64_t* __restrict__ cand,
                                                      int parts, int64_t B) {
  Shared& sh = *reinterpret_cast<Shared*>(g_smem);
  uint64_t* surv = reinterpret_cast<uint64_t*>(g_smem + sizeof(Shared));
  float* prob = reinterpret_cast<float*>(surv + p.cap);
  float* cum = prob + p.cap;
  uint64_t* tmp = reinterpret_cast<uint64_t*>(prob);
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  int kk;
  float pp;
  bool bad;
  row_params(p, b, &kk, &pp, &bad);
  const float u = t < 32 ? row_uniform(p, b) : 0.0f;
  const int n = parts * p.K;
  for (int i = t; i < n; i += NT) {
    const int part = i / p.K, j = i - part * p.K;
    tmp[i] = cand[(static_cast<size_t>(part) * B + b) * (p.K + 1) + j];
  }
  // Combined row status: NaN or +inf in any shard; all -inf only if every shard is.
  if (t == 0) {
    int nan = 0, inf = 0, neg = 0;
    for (int part = 0; part < parts; ++part) {
      const uint64_t w = cand[(static_cast<size_t>(part) * B + b) * (p.K + 1) + p.K];
      nan |= w == FS_ROW_NAN;
      inf |= w == FS_ROW_POSINF;
      neg += w == FS_ROW_ALL_NEGINF;
    }
    const int st = bad ? FS_ROW_BAD_PARAM
                       : nan ? FS_ROW_NAN : inf ? FS_ROW_POSINF : (neg == parts ? FS_ROW_ALL_NEGINF : FS_ROW_OK);
    sh.ctl[kCtlStatus] = static_cast<uint32_t>(st);
  }
  __syncthreads();
  const int st = static_cast<int>(sh.ctl[kCtlStatus]);
  if (st != FS_ROW_OK) {
    write_invalid_row(p, b, st);
    return;
  }
  // A shard padded with 0 when it held fewer than K values; kk never exceeds the real count
  // because every shard holds at least K values (checked on the host).
  finish_row<DT>(p, b, tmp, n, surv, kk, pp, u, prob, cum, sh);
}

// ------------------------------------------------------------------------------------------
// Vocab-sharded tensor parallelism without a collective library: every rank pushes its [B, K+1]
// candidate block straight into every peer's receive buffer over NVLink (CUDA IPC mappings, plain
// stores), then raises one flag per (row, source rank) in every peer with a system-scope release
// store; each rank waits for its own flags (acquire loads, bounded) and merges locally.
// Receive buffers and flags are double-buffered by call parity: a rank can only be one call
// ahead of a peer (its merge needs the peer's push of the same call, and the peer pushes a call
// only after its previous merge has finished), so a slot is never overwritten while being read.
// The call's epoch is either a launch argument or, with a device counter, read from the counter
// at launch and written back (advanced) by the launch's last CTA: then the host passes nothing
// per call and the launches can be captured in a CUDA graph and replayed.
// ------------------------------------------------------------------------------------------

struct TpPeers {
  int32_t world, rank;
  int64_t max_batch;
  uint32_t epoch;                  // this call's number (>= 1); its slot is epoch & 1
  uint32_t* ectr;                  // optional device counter {last epoch, CTAs done}: overrides `epoch`
  long long wait_polls;            // bound on the polls of one flag
  uint64_t* recv;                  // local [2][world][max_batch][K + 1]
  uint32_t* flags;                 // local [2][world][max_batch]
  uint64_t* const* peer_recv;      // device array: every rank's recv (this rank's included)
  uint32_t* const* peer_flags;     // device array: every rank's flags
};

__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

// The epoch after `e` on the device counter: never 0 (flags start at 0) and always of the other
// parity (the slot alternates): after 2^32 - 1 it wraps to 2.
__device__ __forceinline__ uint32_t next_epoch(uint32_t e) { return e == 0xFFFFFFFFu ? 2u : e + 1u; }

// The exchange, wait and merge of one row; returns when the row's outputs are written.
template <int DT>
__device__ void tp_merge_row(const Params& p, const uint64_t* __restrict__ local_cand, const TpPeers& tp,
                             uint32_t epoch) {
  Shared& sh = *reinterpret_cast<Shared*>(g_smem);
  uint64_t* surv = reinterpret_cast<uint64_t*>(g_smem + sizeof(Shared));
  float* prob = reinterpret_cast<float*>(surv + p.cap);
  float* cum = prob + p.cap;
  uint64_t* tmp = reinterpret_cast<uint64_t*>(prob);
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const int W = tp.world;
  const int K1 = p.K + 1;
  const uint32_t slot = epoch & 1u;
  // 1. push this rank's row to every rank, then raise the row's flag there
  for (int i = t; i < K1; i += NT) {
    const uint64_t x = local_cand[static_cast<size_t>(b) * K1 + i];
    for (int r = 0; r < W; ++r)
      tp.peer_recv[r][((static_cast<size_t>(slot) * W + tp.rank) * tp.max_batch + b) * K1 + i] = x;
  }
  // the CTA's stores are ordered before the flag by the barrier and one system-scope fence in
  // each flag-raising thread (fences are cumulative), not by a fence in every thread
  __syncthreads();
  if (t < W) {
    __threadfence_system();
    st_release_sys(&tp.peer_flags[t][(static_cast<size_t>(slot) * W + tp.rank) * tp.max_batch + b], epoch);
  }
  // 2. wait for every rank's row (bounded)
  if (t < 32) {
    bool ok = true;
    if (t < W) {
      const uint32_t* f = &tp.flags[(static_cast<size_t>(slot) * W + t) * tp.max_batch + b];
      ok = false;
      for (long long i = 0; i < tp.wait_polls; ++i) {
        if (ld_acquire_sys(f) == epoch) {
          ok = true;
          break;
        }
        __nanosleep(32);
      }
    }
    const bool all = __all_sync(0xFFFFFFFFu, ok);
    if (t == 0) sh.ctl[kCtlTmo] = all ? 0u : 1u;
  }
  __syncthreads();
  if (sh.ctl[kCtlTmo] != 0u) {
    write_invalid_row(p, b, FS_ROW_TIMEOUT);
    return;
  }
  __threadfence();
  // 3. merge: exact top-k over the W * K gathered candidates, then the common tail
  int kk;
  float pp;
  bool bad;
  row_params(p, b, &kk, &pp, &bad);
  const float u = t < 32 ? row_uniform(p, b) : 0.0f;
  const uint64_t* rows = tp.recv + static_cast<size_t>(slot) * W * tp.max_batch * K1;
  const int n = W * p.K;
  for (int i = t; i < n; i += NT) {
    const int part = i / p.K, j = i - part * p.K;
    tmp[i] = __ldcg(rows + (static_cast<size_t>(part) * tp.max_batch + b) * K1 + j);
  }
  if (t == 0) {
    int nan = 0, inf = 0, neg = 0;
    for (int part = 0; part < W; ++part) {
      const uint64_t w = __ldcg(rows + (static_cast<size_t>(part) * tp.max_batch + b) * K1 + p.K);
      nan |= w == FS_ROW_NAN;
      inf |= w == FS_ROW_POSINF;
      neg += w == FS_ROW_ALL_NEGINF;
    }
    const int st = bad ? FS_ROW_BAD_PARAM
                       : nan ? FS_ROW_NAN : inf ? FS_ROW_POSINF : (neg == W ? FS_ROW_ALL_NEGINF : FS_ROW_OK);
    sh.ctl[kCtlStatus] = static_cast<uint32_t>(st);
  }
  __syncthreads();
  const int st = static_cast<int>(sh.ctl[kCtlStatus]);
  if (st != FS_ROW_OK) {
    write_invalid_row(p, b, st);
    return;
  }
  finish_row<DT>(p, b, tmp, n, surv, kk, pp, u, prob, cum, sh);
}

template <int DT>
__global__ void __launch_bounds__(NT) fs_tp_merge_kernel(const Params p, const uint64_t* __restrict__ local_cand,
                                                         const TpPeers tp) {
  // programmatic dependent launch: this grid may have been placed while the shard top-k kernel
  // still runs; wait for it (and, through it, for the previous step) before reading anything
  grid_dependency_wait();
  grid_launch_dependents();
  // with a device counter every CTA reads the last epoch before any CTA writes it back: the
  // write-back comes from the CTA that finishes last, after every CTA has started
  uint32_t epoch = tp.epoch;
  if (tp.ectr != nullptr) epoch = next_epoch(*reinterpret_cast<volatile const uint32_t*>(&tp.ectr[0]));
  tp_merge_row<DT>(p, local_cand, tp, epoch);
  if (tp.ectr != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(&tp.ectr[1], 1u) == gridDim.x - 1u) {
        tp.ectr[1] = 0u;
        *reinterpret_cast<volatile uint32_t*>(&tp.ectr[0]) = epoch;
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------

using KernelFn = void (*)(const Params);

constexpr int kChunkOptions[] = {1, 2, 3, 4, 5, 6, 8, 10, 12, 16};

template <int DT>
KernelFn cluster_kernel_for(int C) {
  switch (C) {
    case 1: return fs_cluster_kernel<DT, 1>;
    case 2: return fs_cluster_kernel<DT, 2>;
    case 3: return fs_cluster_kernel<DT, 3>;
    case 4: return fs_cluster_kernel<DT, 4>;
    case 5: return fs_cluster_kernel<DT, 5>;
    case 6: return fs_cluster_kernel<DT, 6>;
    case 8: return fs_cluster_kernel<DT, 8>;
    case 10: return fs_cluster_kernel<DT, 10>;
    case 12: return fs_cluster_kernel<DT, 12>;
    case 16: return fs_cluster_kernel<DT, 16>;
    default: return nullptr;
  }
}

static int pow2_ceil(int64_t x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}
static int pow2_floor(int64_t x) {
  int p = 1;
  while (static_cast<int64_t>(p) * 2 <= x) p <<= 1;
  return p;
}

constexpr int kMaxCap = 8192;
constexpr int64_t kStreamMaxK = 256;     // streaming path: top-K bound

// Cluster path: CTAs per row, measured best on B200 (bench.py --sweep; bf16, cold L2) for
// [vocabulary class][batch bucket][k bucket]. Vocabulary class 0: rows that 4 CTAs can hold in
// registers (V <= 131072; measured at 128256), 1: larger (measured at 151936, where 8 and 16 are
// the choices). Batch buckets: 1, 4, 16, 32, 64, 96, 128, 256 rows (the largest not above B);
// k buckets: 1, <= 128, <= 512, larger. A value the row cannot use is raised to the smallest
// split that holds it (or lowered to one chunk per CTA for small rows).
constexpr int kSplitBatch[8] = {1, 4, 16, 32, 64, 96, 128, 256};
constexpr unsigned char kClusterSplits[2][8][4] = {
    {{16, 16, 16, 8}, {8, 8, 16, 16}, {8, 8, 8, 4}, {8, 8, 4, 4}, {4, 4, 4, 4}, {4, 4, 4, 4}, {4, 4, 4, 4},
     {4, 4, 4, 4}},
    {{16, 16, 16, 16}, {16, 16, 16, 16}, {8, 8, 8, 8}, {8, 8, 8, 8}, {8, 8, 8, 8}, {8, 8, 8, 8}, {8, 8, 8, 8},
     {8, 8, 8, 8}},
};

static int split_bucket_b(int64_t B) {
  int i = 0;
  while (i + 1 < 8 && B >= kSplitBatch[i + 1]) ++i;
  return i;
}
static int split_bucket_k(int64_t K) { return K <= 1 ? 0 : K <= 128 ? 1 : K <= 512 ? 2 : 3; }

// AUTO takes the streaming path from this many rows (measured crossover with the cluster path at
// its measured split): k <= 128 from 96 rows; 128 < k <= 256 from 64 rows when the row needs 8
// or more CTAs, else from 96.
static bool auto_stream(int64_t B, int64_t K, int64_t min_s) {
  if (K <= 128) return B >= 96;
  if (K <= kStreamMaxK) return B >= (min_s > 4 ? 64 : 96);
  return false;
}

// Plan of one call: cluster size, chunks per thread, survivor capacity, maxima granularity.
static fs_status make_plan_uncached(int64_t B, int64_t V, int64_t K, int32_t splits, int32_t path, PlanOut* out);

// make_plan with a small per-thread cache: a serving loop asks for the same few plans on every
// call, and the plan is on the host's critical path of a B=1 call (about as long as the kernel).
fs_status make_plan(int64_t B, int64_t V, int64_t K, int32_t splits, int32_t path, PlanOut* out) {
  struct Entry {
    int64_t B, V, K;
    int32_t splits, path;
    bool valid;
    PlanOut plan;
  };
  constexpr int kEntries = 8;
  thread_local Entry cache[kEntries] = {};
  thread_local int next = 0;
  for (const Entry& e : cache) {
    if (e.valid && e.B == B && e.V == V && e.K == K && e.splits == splits && e.path == path) {
      *out = e.plan;
      return FS_OK;
    }
  }
  const fs_status st = make_plan_uncached(B, V, K, splits, path, out);
  if (st == FS_OK) {
    cache[next] = Entry{B, V, K, splits, path, true, *out};
    next = (next + 1) % kEntries;
  }
  return st;
}

static fs_status make_plan_uncached(int64_t B, int64_t V, int64_t K, int32_t splits, int32_t path, PlanOut* out) {
  if (path < FS_PATH_AUTO || path > FS_PATH_WIDE) {
    set_error("path must be one of FS_PATH_AUTO, FS_PATH_CLUSTER, FS_PATH_STREAM, FS_PATH_WIDE; got %d", path);
    return FS_EINVAL;
  }
  const int64_t per_cta_chunk = static_cast<int64_t>(NT) * 8;  // elements per chunk per CTA
  constexpr int kMaxChunks = 16;
  const int64_t min_s = std::max<int64_t>(1, (V + per_cta_chunk * kMaxChunks - 1) / (per_cta_chunk * kMaxChunks));
  int S;
  if (splits > 0) {
    // a requested split that cannot hold the row in registers is raised to the smallest that can
    S = static_cast<int>(std::min<int64_t>(kMaxSplits, std::max<int64_t>(splits, min_s)));
    S = std::min(kMaxSplits, pow2_ceil(S));  // powers of two keep the slot arithmetic to shifts
  } else {
    S = kClusterSplits[min_s > 4 ? 1 : 0][split_bucket_b(B)][split_bucket_k(K)];
    // small rows need fewer CTAs
    const int64_t one_chunk = (V + per_cta_chunk - 1) / per_cta_chunk;
    S = static_cast<int>(std::min<int64_t>(S, std::max<int64_t>(1, one_chunk)));
    S = static_cast<int>(std::min<int64_t>(kMaxSplits, std::max<int64_t>(S, min_s)));
    S = std::min(kMaxSplits, pow2_ceil(S));
  }
  // smallest chunk option that covers the row
  int C = 0;
  for (int opt : kChunkOptions) {
    if (static_cast<int64_t>(opt) * per_cta_chunk * S >= V) {
      C = opt;
      break;
    }
  }
  if (C == 0) {
    set_error("vocabulary of %lld does not fit %d CTAs x %d threads x 128 values",
              static_cast<long long>(V), S, NT);
    return FS_EUNSUPPORTED;
  }
  const int threads_total = S * NT;
  int mpt = 1, mgroup = 1;
  const int64_t target = 4 * K;  // about four maxima per wanted candidate
  if (target <= threads_total) {
    mgroup = std::min(32, pow2_floor(threads_total / target));
  } else {
    mpt = static_cast<int>(std::min<int64_t>(8, pow2_ceil((target + threads_total - 1) / threads_total)));
  }
  while (static_cast<int64_t>(threads_total) * mpt / mgroup > kMaxMaxima) {
    if (mpt > 1) mpt /= 2;
    else mgroup *= 2;
  }
  int cap = std::max(1024, pow2_ceil(4 * K));
  cap = std::min(cap, kMaxCap);
  // top_k beyond the survivor buffer takes the wide path (token ids and row status only)
  const bool wide = path == FS_PATH_WIDE || (path == FS_PATH_AUTO && K > kMaxCap);
  if (!wide && cap < K) {
    set_error("top_k of %lld exceeds the %d-candidate capacity of the cluster and streaming paths "
              "(FS_PATH_AUTO or FS_PATH_WIDE take any top_k for token ids)",
              static_cast<long long>(K), kMaxCap);
    return FS_EUNSUPPORTED;
  }
  out->splits = S;
  out->chunks = C;
  out->threads = NT;
  out->mpt = mpt;
  out->mgroup = mgroup;
  out->capacity = cap;
  out->slot = cap / S;
  out->mcta = NT * out->mpt / out->mgroup;
  out->smem = static_cast<int>(shared_bytes(out->capacity));
  out->stream = 0;
  out->merge_cap = 0;
  out->merge_smem = 0;
  out->workspace = 0;
  out->wide = wide ? 1 : 0;
  if (wide) {
    // per-key counts [B][65536], slice maxima and flags [B][S] x 2, locate counts [B][S], row
    // results [B][4]
    out->smem = 0;
    out->workspace = static_cast<uint64_t>(B) * kKeys * 4 + static_cast<uint64_t>(B) * S * 12 +
                     static_cast<uint64_t>(B) * kWideRes * 4 + 256;
    return FS_OK;
  }

  // streaming path: slices keep their own top-K in M slots; the row merge gathers S * M. The
  // fewest slices that hold the row measured fastest at every batch (a requested split is kept)
  const int M = std::max(64, pow2_ceil(2 * K));
  int Ss = splits > 0 ? S : std::min(kMaxSplits, pow2_ceil(min_s));
  // fewer, longer slices when S * M candidates would not fit the row merge's key buffer
  while (Ss > 1 && static_cast<int64_t>(Ss) * M > kMaxMaxima) Ss /= 2;
  int Cs = 0;
  for (int opt : kChunkOptions) {
    if (static_cast<int64_t>(opt) * per_cta_chunk * Ss >= V) {
      Cs = opt;
      break;
    }
  }
  // (the slice launch puts rows on grid.y, at most 65535)
  const bool stream_fits = K <= kStreamMaxK && static_cast<int64_t>(Ss) * M <= kMaxMaxima && Cs > 0 && B <= 65535;
  const bool want_stream = path == FS_PATH_STREAM || (path == FS_PATH_AUTO && auto_stream(B, K, min_s));
  if (path == FS_PATH_STREAM && !stream_fits) {
    set_error("the streaming path supports top_k <= %lld with splits * slots <= %d and batch <= 65535",
              static_cast<long long>(kStreamMaxK), kMaxMaxima);
    return FS_EUNSUPPORTED;
  }
  if (want_stream && stream_fits) {
    S = Ss;
    out->splits = Ss;
    out->chunks = Cs;
    out->stream = 1;
    out->mpt = static_cast<int>(std::min<int64_t>(8, pow2_ceil((4 * K + NT - 1) / NT)));
    out->mgroup = 1;
    out->mcta = NT * out->mpt;
    out->slot = M;
    out->smem = static_cast<int>(sizeof(Shared)) + kSliceStageBytes;
    out->merge_cap = std::max(256, pow2_ceil(static_cast<int64_t>(S) * M));
    out->merge_smem = static_cast<int>(merge_rows_per_cta(out->merge_cap, static_cast<int>(K)) *
                                       merge_row_bytes(out->merge_cap, static_cast<int>(K)));
    // candidates [B][S][M], ladders [B][S], count words [B][S]
    out->workspace = static_cast<uint64_t>(B) * S * M * sizeof(uint64_t) + static_cast<uint64_t>(B) * S * 8 +
                     static_cast<uint64_t>(B) * S * 4 + 256;
  }
  return FS_OK;
}

// Kernel attribute state of one (kernel, device) pair: the dynamic shared memory limit already
// granted and whether non-portable cluster sizes were enabled. Function attributes are per
// device, so a process that drives several GPUs keeps one record per device; each is set once
// per kernel and size, not on every launch.
struct KernelState {
  const void* fn;
  int dev;
  int smem_granted;
  bool nonportable;
};

constexpr int kMaxKernelStates = 512;

// The record of (fn, dev), created on first use; null when the table is full.
KernelState* kernel_state(const void* fn, int dev) {
  static KernelState states[kMaxKernelStates];
  static int n_states = 0;
  for (int i = 0; i < n_states; ++i)
    if (states[i].fn == fn && states[i].dev == dev) return &states[i];
  if (n_states == kMaxKernelStates) return nullptr;
  states[n_states] = KernelState{fn, dev, 0, false};
  return &states[n_states++];
}

static fs_status prepare_kernel(KernelFn fn, int S, int smem) {
  static std::mutex mu;
  const void* f = reinterpret_cast<const void*>(fn);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  // the calling thread's last kernel already prepared for at least this much: no lock (grants
  // only ever grow, so a remembered grant stays valid)
  thread_local const void* last_fn = nullptr;
  thread_local int last_dev = -1, last_smem = 0;
  thread_local bool last_nonportable = false;
  if (f == last_fn && dev == last_dev && smem <= last_smem && (S <= 8 || last_nonportable)) return FS_OK;
  std::lock_guard<std::mutex> lock(mu);
  KernelState* ks = kernel_state(f, dev);
  if (ks == nullptr) {
    set_error("kernel state table full (%d kernel x device pairs)", kMaxKernelStates);
    return FS_ELAUNCH;
  }
  if (smem > ks->smem_granted) {
    e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(max dynamic smem %d): %s", smem, cudaGetErrorString(e));
      return FS_ELAUNCH;
    }
    ks->smem_granted = smem;
  }
  if (S > 8 && !ks->nonportable) {
    e = cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(non-portable cluster): %s", cudaGetErrorString(e));
      return FS_ELAUNCH;
    }
    ks->nonportable = true;
  }
  last_fn = f;
  last_dev = dev;
  last_smem = ks->smem_granted;
  last_nonportable = ks->nonportable;
  return FS_OK;
}

static fs_status launch_cluster(int dtype, const PlanOut& plan, int64_t B, const Params& prm,
                                cudaStream_t stream) {
  KernelFn fn = dtype == FS_BF16 ? cluster_kernel_for<1>(plan.chunks) : cluster_kernel_for<0>(plan.chunks);
  if (fn == nullptr) {
    set_error("no kernel for %d chunks", plan.chunks);
    return FS_EUNSUPPORTED;
  }
  fs_status st = prepare_kernel(fn, plan.splits, plan.smem);
  if (st != FS_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.splits, static_cast<unsigned>(B), 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = plan.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // may start while the stream's previous kernel finishes (the kernel waits for it before it
  // reads anything), which hides most of the launch latency of back-to-back calls
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, prm);
  if (e != cudaSuccess) {
    set_error("cluster launch (splits=%d chunks=%d smem=%d B=%lld): %s", plan.splits, plan.chunks,
              plan.smem, static_cast<long long>(B), cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

// Clears the wide path's [B, 65536] per-key histograms with 16-byte stores. It waits for the
// stream's previous kernel first (the workspace may be memory that kernel still reads) and then
// lets the histogram launch be placed while it runs.
__global__ void __launch_bounds__(NT) fs_wide_zero_kernel(uint4* __restrict__ h, size_t n16) {
  grid_dependency_wait();
  grid_launch_dependents();
  const size_t step = static_cast<size_t>(gridDim.x) * NT;
  for (size_t i = static_cast<size_t>(blockIdx.x) * NT + threadIdx.x; i < n16; i += step) h[i] = make_uint4(0u, 0u, 0u, 0u);
}

template <int DT, int C>
struct WideKernels {
  static fs_status launch(const fs_sample_args* a, const PlanOut& plan, const Params& prm, uint32_t* hist,
                          uint32_t* smax, uint32_t* sflag, uint32_t* cnt, uint32_t* res, cudaStream_t stream) {
    const dim3 grid(plan.splits, static_cast<unsigned>(a->batch), 1);
    fs_status st = prepare_kernel(reinterpret_cast<KernelFn>(fs_wide_row_kernel<DT>), 1, kWCacheKeys * 4);
    if (st != FS_OK) return st;
    // programmatic dependent launch: each kernel waits for its predecessor before it reads
    // anything, so the next one may be launched (and placed) while the current one runs
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    auto cfg = [&](dim3 g, unsigned block, size_t smem) {
      cudaLaunchConfig_t c = {};
      c.gridDim = g;
      c.blockDim = dim3(block, 1, 1);
      c.dynamicSmemBytes = smem;
      c.stream = stream;
      c.attrs = pdl;
      c.numAttrs = 1;
      return c;
    };
    const char* what = "wide histogram launch";
    cudaLaunchConfig_t c1 = cfg(grid, NT, 0);
    cudaError_t e = cudaLaunchKernelEx(&c1, fs_wide_hist_kernel<DT, C>, prm, hist, smax, sflag);
    if (e == cudaSuccess) {
      what = "wide row launch";
      cudaLaunchConfig_t c2 = cfg(dim3(static_cast<unsigned>(a->batch), 1, 1), kRowThreads, kWCacheKeys * 4);
      e = cudaLaunchKernelEx(&c2, fs_wide_row_kernel<DT>, prm, static_cast<const uint32_t*>(hist),
                             static_cast<const uint32_t*>(smax), static_cast<const uint32_t*>(sflag), res,
                             plan.splits);
    }
    if (e == cudaSuccess) {
      what = "wide count launch";
      cudaLaunchConfig_t c3 = cfg(grid, NT, 0);
      e = cudaLaunchKernelEx(&c3, fs_wide_count_kernel<DT, C>, prm, static_cast<const uint32_t*>(res), cnt);
    }
    if (e == cudaSuccess) {
      what = "wide pick launch";
      cudaLaunchConfig_t c4 = cfg(grid, NT, 0);
      e = cudaLaunchKernelEx(&c4, fs_wide_pick_kernel<DT, C>, prm, static_cast<const uint32_t*>(res),
                             static_cast<const uint32_t*>(cnt));
    }
    if (e != cudaSuccess) {
      set_error("%s: %s", what, cudaGetErrorString(e));
      return FS_ELAUNCH;
    }
    return FS_OK;
  }
};

template <int DT>
static fs_status launch_wide_dt(const fs_sample_args* a, const PlanOut& plan, const Params& prm, uint32_t* hist,
                                uint32_t* smax, uint32_t* sflag, uint32_t* cnt, uint32_t* res, cudaStream_t st) {
  switch (plan.chunks) {
    case 1: return WideKernels<DT, 1>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 2: return WideKernels<DT, 2>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 3: return WideKernels<DT, 3>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 4: return WideKernels<DT, 4>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 5: return WideKernels<DT, 5>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 6: return WideKernels<DT, 6>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 8: return WideKernels<DT, 8>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 10: return WideKernels<DT, 10>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 12: return WideKernels<DT, 12>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    case 16: return WideKernels<DT, 16>::launch(a, plan, prm, hist, smax, sflag, cnt, res, st);
    default:
      set_error("no wide-path kernels for %d chunks", plan.chunks);
      return FS_EUNSUPPORTED;
  }
}

// The wide path's launches: the histogram is cleared first (the workspace needs no
// initialisation from the caller), then the four kernels, stream-ordered.
static fs_status launch_wide(const fs_sample_args* a, const PlanOut& plan, const Params& prm, cudaStream_t stream) {
  if (a->workspace == nullptr || a->workspace_bytes < plan.workspace) {
    set_error("the wide path needs %llu bytes of workspace (got %llu)",
              static_cast<unsigned long long>(plan.workspace),
              static_cast<unsigned long long>(a->workspace == nullptr ? 0 : a->workspace_bytes));
    return FS_EWORKSPACE;
  }
  const uintptr_t base = (reinterpret_cast<uintptr_t>(a->workspace) + 255) & ~static_cast<uintptr_t>(255);
  const size_t B = static_cast<size_t>(a->batch), S = static_cast<size_t>(plan.splits);
  uint32_t* hist = reinterpret_cast<uint32_t*>(base);
  uint32_t* smax = hist + B * kKeys;
  uint32_t* sflag = smax + B * S;
  uint32_t* cnt = sflag + B * S;
  uint32_t* res = cnt + B * S;
  // the histograms start at zero: a clearing kernel in the same launch chain as the four below
  const size_t n16 = B * kKeys * sizeof(uint32_t) / 16;
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t zc = {};
  zc.gridDim = dim3(static_cast<unsigned>(std::min<size_t>((n16 + NT - 1) / NT, 148 * 8)), 1, 1);
  zc.blockDim = dim3(NT, 1, 1);
  zc.stream = stream;
  zc.attrs = pdl;
  zc.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&zc, fs_wide_zero_kernel, reinterpret_cast<uint4*>(hist), n16);
  if (e != cudaSuccess) {
    set_error("wide path histogram clear: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  const fs_status st = a->dtype == FS_BF16 ? launch_wide_dt<1>(a, plan, prm, hist, smax, sflag, cnt, res, stream)
                                           : launch_wide_dt<0>(a, plan, prm, hist, smax, sflag, cnt, res, stream);
  if (st != FS_OK) return st;
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("wide path launch (splits=%d chunks=%d B=%lld): %s", plan.splits, plan.chunks,
              static_cast<long long>(a->batch), cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

static fs_status check_common(const fs_sample_args* a, bool need_logits) {
  if (a == nullptr) {
    set_error("args is NULL");
    return FS_EINVAL;
  }
  if (a->dtype != FS_F16 && a->dtype != FS_BF16) {
    set_error("logits must be float16 or bfloat16");
    return FS_EINVAL;
  }
  if (a->batch < 1 || a->batch > 65535) {
    set_error("batch must be in [1, 65535], got %lld", static_cast<long long>(a->batch));
    return FS_EINVAL;
  }
  if (need_logits) {
    if (a->logits == nullptr) {
      set_error("logits is NULL");
      return FS_EINVAL;
    }
    if (a->vocab < 1 || a->vocab > (1 << 19)) {
      set_error("vocab must be in [1, 524288], got %lld", static_cast<long long>(a->vocab));
      return FS_EINVAL;
    }
    if (a->row_stride < a->vocab) {
      set_error("row_stride %lld is smaller than vocab %lld", static_cast<long long>(a->row_stride),
                static_cast<long long>(a->vocab));
      return FS_EINVAL;
    }
    if (a->id_base < 0 || a->id_base + a->vocab > 0xFFFFFFFFll) {
      set_error("id_base + vocab must fit in 32 bits");
      return FS_EINVAL;
    }
  }
  if (a->top_k < 1) {
    set_error("top_k must be >= 1");
    return FS_EINVAL;
  }
  return FS_OK;
}

static fs_status check_top_p(const fs_sample_args* a) {
  if (a->top_p_rows == nullptr && !(a->top_p > 0.0f && a->top_p <= 1.0f)) {
    set_error("top_p must be in (0, 1]");
    return FS_EINVAL;
  }
  if (!(a->temperature >= 0.0f && a->temperature <= 3.0e38f)) {
    set_error("temperature must be a finite value >= 0 (0 or 1: none)");
    return FS_EINVAL;
  }
  return FS_OK;
}

static Params base_params(const fs_sample_args* a, int64_t K) {
  Params prm = {};
  prm.logits = static_cast<const uint16_t*>(a->logits);
  prm.row_stride = a->row_stride;
  prm.temperature = a->temperature == 0.0f ? 1.0f : a->temperature;
  prm.vocab = static_cast<int32_t>(a->vocab);
  prm.K = static_cast<int32_t>(K);
  prm.id_base = static_cast<uint32_t>(a->id_base);
  prm.top_p = a->top_p;
  prm.k_rows = a->top_k_rows;
  prm.p_rows = a->top_p_rows;
  prm.uniforms = a->rng.uniforms;
  prm.seed = a->rng.seed;
  prm.offset = a->rng.offset;
  prm.seed_ptr = a->rng.seed_ptr;
  prm.offset_ptr = a->rng.offset_ptr;
  prm.offset_intragraph = a->rng.offset_intragraph;
  prm.row_base = a->rng.row_base;
  prm.out = a->out_ids;
  prm.topk_ids = a->topk_ids;
  prm.keep = a->keep;
  prm.renormed = a->renormed;
  prm.status = a->row_status;
  prm.early = (a->input_flags & FS_INPUT_READY) != 0u ? 1 : 0;
  prm.vec = 0;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(a->logits);
  if (addr % 16 == 0 && a->row_stride % 8 == 0) prm.vec = 1;
  return prm;
}

template <int DT>
KernelFn slice_kernel_for(int C) {
  switch (C) {
    case 1: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 1>);
    case 2: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 2>);
    case 3: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 3>);
    case 4: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 4>);
    case 5: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 5>);
    case 6: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 6>);
    case 8: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 8>);
    case 10: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 10>);
    case 12: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 12>);
    case 16: return reinterpret_cast<KernelFn>(fs_slice_kernel<DT, 16>);
    default: return nullptr;
  }
}

using SliceFn = void (*)(const Params, uint64_t*, uint64_t*, uint32_t*);
using RowMergeFn = void (*)(const Params, const uint64_t*, const uint64_t*, const uint32_t*, int, int);

static fs_status launch_stream(const fs_sample_args* a, const PlanOut& plan, const Params& prm,
                               cudaStream_t stream) {
  if (a->workspace == nullptr || a->workspace_bytes < plan.workspace) {
    set_error("the streaming path needs %llu bytes of workspace (got %llu)",
              static_cast<unsigned long long>(plan.workspace),
              static_cast<unsigned long long>(a->workspace == nullptr ? 0 : a->workspace_bytes));
    return FS_EWORKSPACE;
  }
  const uintptr_t base = (reinterpret_cast<uintptr_t>(a->workspace) + 255) & ~static_cast<uintptr_t>(255);
  uint64_t* cand = reinterpret_cast<uint64_t*>(base);
  uint64_t* lad = cand + static_cast<size_t>(a->batch) * plan.splits * plan.slot;
  uint32_t* cnt = reinterpret_cast<uint32_t*>(lad + static_cast<size_t>(a->batch) * plan.splits);
  SliceFn sfn = reinterpret_cast<SliceFn>(a->dtype == FS_BF16 ? slice_kernel_for<1>(plan.chunks)
                                                               : slice_kernel_for<0>(plan.chunks));
  RowMergeFn mfn = a->dtype == FS_BF16 ? fs_rowmerge_kernel<1> : fs_rowmerge_kernel<0>;
  if (sfn == nullptr) {
    set_error("no slice kernel for %d chunks", plan.chunks);
    return FS_EUNSUPPORTED;
  }
  fs_status st = prepare_kernel(reinterpret_cast<KernelFn>(sfn), 1, plan.smem);
  if (st != FS_OK) return st;
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t scfg = {};
  scfg.gridDim = dim3(plan.splits, static_cast<unsigned>(a->batch), 1);
  scfg.blockDim = dim3(NT, 1, 1);
  scfg.dynamicSmemBytes = plan.smem;
  scfg.stream = stream;
  scfg.attrs = pdl;
  scfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&scfg, sfn, prm, cand, lad, cnt);
  if (e != cudaSuccess) {
    set_error("slice launch: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  st = prepare_kernel(reinterpret_cast<KernelFn>(mfn), 1, plan.merge_smem);
  if (st != FS_OK) return st;
  Params mp = prm;
  mp.cap = plan.merge_cap;
  const int mr = merge_rows_per_cta(plan.merge_cap, static_cast<int>(prm.K));
  const unsigned mgrid = static_cast<unsigned>((a->batch + mr - 1) / mr);
  cudaLaunchConfig_t mcfg = {};
  mcfg.gridDim = dim3(mgrid, 1, 1);
  mcfg.blockDim = dim3(kMergeRowThreads * mr, 1, 1);
  mcfg.dynamicSmemBytes = plan.merge_smem;
  mcfg.stream = stream;
  mcfg.attrs = pdl;
  mcfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&mcfg, mfn, static_cast<const Params>(mp), static_cast<const uint64_t*>(cand),
                         static_cast<const uint64_t*>(lad), static_cast<const uint32_t*>(cnt), plan.splits,
                         static_cast<int>(a->batch));
  if (e != cudaSuccess) {
    set_error("row-merge launch: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

fs_status run_cluster(const fs_sample_args* a, int mode, uint64_t* cand_out, cudaStream_t stream) {
  const int64_t K = std::min<int64_t>(a->top_k, a->vocab);
  PlanOut plan;
  // the ablation probe instruments the cluster kernel's phases
  const int32_t path = a->stop_phase != 0 ? FS_PATH_CLUSTER : a->path;
  fs_status st = make_plan(a->batch, a->vocab, K, a->splits, path, &plan);
  if (st != FS_OK) return st;
  Params prm = base_params(a, K);
  prm.cand_out = cand_out;
  prm.cap = plan.capacity;
  prm.mpt = plan.mpt;
  prm.mgroup = plan.mgroup;
  prm.mcta = plan.mcta;
  prm.slot = plan.slot;
  prm.stop = a->stop_phase;
  prm.mode = mode;
  if (plan.wide) {
    if (mode != kModeSample || a->topk_ids != nullptr || a->keep != nullptr || a->renormed != nullptr ||
        a->stop_phase != 0) {
      set_error("the wide path (top_k > %d, or FS_PATH_WIDE) produces token ids and row status only: no top-k "
                "ids, keep, renormed, shard candidates or phase probes",
                kMaxCap);
      return FS_EUNSUPPORTED;
    }
    return launch_wide(a, plan, prm, stream);
  }
  if (plan.stream) return launch_stream(a, plan, prm, stream);
  return launch_cluster(a->dtype, plan, a->batch, prm, stream);
}

uint64_t workspace_size(const fs_sample_args* a) {
  if (a == nullptr || a->batch < 1 || a->vocab < 1 || a->top_k < 1) return 0;
  PlanOut plan;
  const int32_t path = a->stop_phase != 0 ? FS_PATH_CLUSTER : a->path;
  if (make_plan(a->batch, a->vocab, std::min<int64_t>(a->top_k, a->vocab), a->splits, path, &plan) != FS_OK)
    return 0;
  return (plan.stream || plan.wide) ? plan.workspace : 0;
}

fs_status run_merge(const fs_sample_args* a, const uint64_t* cand, int parts, cudaStream_t stream) {
  const int64_t K = a->top_k;
  const int64_t n = static_cast<int64_t>(parts) * K;
  int cap = std::max(256, pow2_ceil(n));
  if (cap > kMaxCap) {
    set_error("parts * top_k = %lld exceeds the merge capacity %d", static_cast<long long>(n), kMaxCap);
    return FS_EUNSUPPORTED;
  }
  Params prm = base_params(a, K);
  prm.vec = 0;
  prm.cap = cap;
  prm.mode = a->topk_ids != nullptr && a->out_ids == nullptr ? kModeTopk : kModeSample;
  const int smem = static_cast<int>(shared_bytes(cap));
  auto fn = a->dtype == FS_BF16 ? fs_merge_kernel<1> : fs_merge_kernel<0>;
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(merge smem %d): %s", smem, cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  fn<<<static_cast<unsigned>(a->batch), NT, smem, stream>>>(prm, cand, parts, a->batch);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("merge launch: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

fs_status run_tp_merge(const fs_sample_args* a, const uint64_t* local_cand, const fs_tp_peers* tpa,
                       cudaStream_t stream) {
  const int64_t K = a->top_k;
  const int64_t n = static_cast<int64_t>(tpa->world) * K;
  int cap = std::max(256, pow2_ceil(n));
  if (cap > kMaxCap) {
    set_error("world * top_k = %lld exceeds the merge capacity %d", static_cast<long long>(n), kMaxCap);
    return FS_EUNSUPPORTED;
  }
  Params prm = base_params(a, K);
  prm.vec = 0;
  prm.cap = cap;
  prm.mode = kModeSample;
  TpPeers tp;
  tp.world = tpa->world;
  tp.rank = tpa->rank;
  tp.max_batch = tpa->max_batch;
  tp.epoch = tpa->epoch;
  tp.ectr = tpa->epoch_counter;
  tp.wait_polls = tpa->wait_polls > 0 ? tpa->wait_polls : (1LL << 22);
  tp.recv = tpa->recv;
  tp.flags = tpa->flags;
  tp.peer_recv = tpa->peer_recv;
  tp.peer_flags = tpa->peer_flags;
  const int smem = static_cast<int>(shared_bytes(cap));
  auto fn = a->dtype == FS_BF16 ? fs_tp_merge_kernel<1> : fs_tp_merge_kernel<0>;
  fs_status st = prepare_kernel(reinterpret_cast<KernelFn>(fn), 1, smem);
  if (st != FS_OK) return st;
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a->batch), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, prm, local_cand, tp);
  if (e != cudaSuccess) {
    set_error("tp merge launch: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

void append_cluster_attrs(std::vector<fs_kernel_attr>& rows) {
  for (int dt = 0; dt < 2; ++dt) {
    for (int C : kChunkOptions) {
      KernelFn fn = dt ? cluster_kernel_for<1>(C) : cluster_kernel_for<0>(C);
      fs_kernel_attr r = {};
      std::snprintf(r.name, sizeof(r.name), "fs_cluster_kernel<%s>", dt ? "bf16" : "fp16");
      r.param = C;
      r.block = NT;
      fill_attr(reinterpret_cast<const void*>(fn), NT, static_cast<int>(shared_bytes(1024)), &r);
      rows.push_back(r);
    }
    for (int C : kChunkOptions) {
      KernelFn fn = dt ? slice_kernel_for<1>(C) : slice_kernel_for<0>(C);
      fs_kernel_attr r = {};
      std::snprintf(r.name, sizeof(r.name), "fs_slice_kernel<%s>", dt ? "bf16" : "fp16");
      r.param = C;
      r.block = NT;
      fill_attr(reinterpret_cast<const void*>(fn), NT, static_cast<int>(sizeof(Shared)), &r);
      rows.push_back(r);
    }
    {
      fs_kernel_attr r = {};
      std::snprintf(r.name, sizeof(r.name), "fs_rowmerge_kernel<%s>", dt ? "bf16" : "fp16");
      r.param = 0;
      r.block = NT;
      fill_attr(reinterpret_cast<const void*>(dt ? fs_rowmerge_kernel<1> : fs_rowmerge_kernel<0>), NT,
                static_cast<int>(merge_rows_per_cta(1024, 64) * merge_row_bytes(1024, 64)), &r);
      rows.push_back(r);
    }
    {
      fs_kernel_attr r = {};
      std::snprintf(r.name, sizeof(r.name), "fs_wide_hist_kernel<%s>", dt ? "bf16" : "fp16");
      r.param = 5;
      r.block = NT;
      fill_attr(reinterpret_cast<const void*>(dt ? fs_wide_hist_kernel<1, 5> : fs_wide_hist_kernel<0, 5>), NT, 0, &r);
      rows.push_back(r);
      std::snprintf(r.name, sizeof(r.name), "fs_wide_row_kernel<%s>", dt ? "bf16" : "fp16");
      r.param = 0;
      r.block = kRowThreads;
      fill_attr(reinterpret_cast<const void*>(dt ? fs_wide_row_kernel<1> : fs_wide_row_kernel<0>), kRowThreads,
                kWCacheKeys * 4, &r);
      rows.push_back(r);
    }
    {
      fs_kernel_attr r = {};
      std::snprintf(r.name, sizeof(r.name), "fs_tp_merge_kernel<%s>", dt ? "bf16" : "fp16");
      r.param = 0;
      r.block = NT;
      fill_attr(reinterpret_cast<const void*>(dt ? fs_tp_merge_kernel<1> : fs_tp_merge_kernel<0>), NT,
                static_cast<int>(shared_bytes(256)), &r);
      rows.push_back(r);
    }
    fs_kernel_attr r = {};
    std::snprintf(r.name, sizeof(r.name), "fs_merge_kernel<%s>", dt ? "bf16" : "fp16");
    r.param = 0;
    r.block = NT;
    fill_attr(reinterpret_cast<const void*>(dt ? fs_merge_kernel<1> : fs_merge_kernel<0>), NT,
              static_cast<int>(shared_bytes(256)), &r);
    rows.push_back(r);
  }
}

}  // namespace fsb

// ------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------

extern "C" fs_status fs_sample(const fs_sample_args* a, fs_stream_t stream) {
  fs_status st = fsb::check_common(a, true);
  if (st != FS_OK) return st;
  if ((st = fsb::check_top_p(a)) != FS_OK) return st;
  if (a->out_ids == nullptr) {
    fsb::set_error("out_ids is NULL");
    return FS_EINVAL;
  }
  fs_sample_args b = *a;
  b.stop_phase = 0;
  return fsb::run_cluster(&b, fsb::kModeSample, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" fs_status fs_topk(const fs_sample_args* a, fs_stream_t stream) {
  fs_status st = fsb::check_common(a, true);
  if (st != FS_OK) return st;
  if (a->topk_ids == nullptr) {
    fsb::set_error("topk_ids is NULL");
    return FS_EINVAL;
  }
  fs_sample_args b = *a;
  b.stop_phase = 0;
  b.top_p = 1.0f;
  b.top_p_rows = nullptr;
  return fsb::run_cluster(&b, fsb::kModeTopk, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" fs_status fs_probe_phase(const fs_sample_args* a, fs_stream_t stream) {
  fs_status st = fsb::check_common(a, true);
  if (st != FS_OK) return st;
  if ((st = fsb::check_top_p(a)) != FS_OK) return st;
  if (a->stop_phase < 1 || a->stop_phase > FS_NUM_PHASES) {
    fsb::set_error("phase must be in [1, %d]", FS_NUM_PHASES);
    return FS_EINVAL;
  }
  if (a->out_ids == nullptr) {
    fsb::set_error("out_ids is NULL");
    return FS_EINVAL;
  }
  fs_sample_args b = *a;
  b.topk_ids = nullptr;
  b.keep = nullptr;
  b.renormed = nullptr;
  if (b.stop_phase == FS_NUM_PHASES) b.stop_phase = 0;
  return fsb::run_cluster(&b, fsb::kModeSample, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" fs_status fs_shard_candidates(const fs_sample_args* a, uint64_t* cand_out,
                                         fs_stream_t stream) {
  fs_status st = fsb::check_common(a, true);
  if (st != FS_OK) return st;
  if (cand_out == nullptr) {
    fsb::set_error("cand_out is NULL");
    return FS_EINVAL;
  }
  if (a->top_k > a->vocab) {
    fsb::set_error("shard top_k (%lld) must not exceed the shard vocab (%lld)",
                   static_cast<long long>(a->top_k), static_cast<long long>(a->vocab));
    return FS_EINVAL;
  }
  fs_sample_args b = *a;
  b.stop_phase = 0;
  b.top_k_rows = nullptr;
  b.top_p_rows = nullptr;
  b.top_p = 1.0f;
  b.out_ids = nullptr;
  b.topk_ids = nullptr;
  b.keep = nullptr;
  b.renormed = nullptr;
  b.row_status = nullptr;
  return fsb::run_cluster(&b, fsb::kModeShard, cand_out, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" fs_status fs_merge_sample(const fs_sample_args* a, const uint64_t* cand, int32_t parts,
                                     fs_stream_t stream) {
  fs_status st = fsb::check_common(a, false);
  if (st != FS_OK) return st;
  if (cand == nullptr || parts < 1) {
    fsb::set_error("cand is NULL or parts < 1");
    return FS_EINVAL;
  }
  if (a->out_ids == nullptr && a->topk_ids == nullptr) {
    fsb::set_error("out_ids and topk_ids are both NULL");
    return FS_EINVAL;
  }
  if (a->out_ids != nullptr && (st = fsb::check_top_p(a)) != FS_OK) return st;
  return fsb::run_merge(a, cand, parts, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" fs_status fs_tp_merge_sample(const fs_sample_args* a, const uint64_t* local_cand,
                                        const fs_tp_peers* tp, fs_stream_t stream) {
  fs_status st = fsb::check_common(a, false);
  if (st != FS_OK) return st;
  if (local_cand == nullptr || tp == nullptr || tp->world < 1 || tp->world > 32 || tp->rank < 0 ||
      tp->rank >= tp->world || tp->recv == nullptr || tp->flags == nullptr || tp->peer_recv == nullptr ||
      tp->peer_flags == nullptr || (tp->epoch == 0u && tp->epoch_counter == nullptr) ||
      a->batch > tp->max_batch) {
    fsb::set_error("invalid tensor-parallel exchange arguments (world 1..32, rank < world, buffers set, "
                   "epoch >= 1 or an epoch counter, batch <= max_batch)");
    return FS_EINVAL;
  }
  if (a->out_ids == nullptr) {
    fsb::set_error("out_ids is NULL");
    return FS_EINVAL;
  }
  if ((st = fsb::check_top_p(a)) != FS_OK) return st;
  return fsb::run_tp_merge(a, local_cand, tp, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" fs_status fs_ipc_alloc(uint64_t bytes, void** dev_ptr_out) {
  if (bytes == 0 || dev_ptr_out == nullptr) {
    fsb::set_error("bytes is 0 or dev_ptr_out is NULL");
    return FS_EINVAL;
  }
  cudaError_t e = cudaMalloc(dev_ptr_out, bytes);
  if (e == cudaSuccess) e = cudaMemset(*dev_ptr_out, 0, bytes);
  if (e != cudaSuccess) {
    fsb::set_error("peer buffer of %llu bytes: %s", static_cast<unsigned long long>(bytes), cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

extern "C" fs_status fs_ipc_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return FS_OK;
  const cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) {
    fsb::set_error("cudaFree: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

extern "C" fs_status fs_ipc_handle(const void* dev_ptr, void* handle_out) {
  if (dev_ptr == nullptr || handle_out == nullptr) {
    fsb::set_error("dev_ptr or handle_out is NULL");
    return FS_EINVAL;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) {
    fsb::set_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  static_assert(sizeof(h) == FS_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return FS_OK;
}

extern "C" fs_status fs_ipc_open(const void* handle, void** dev_ptr_out) {
  if (handle == nullptr || dev_ptr_out == nullptr) {
    fsb::set_error("handle or dev_ptr_out is NULL");
    return FS_EINVAL;
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    fsb::set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

extern "C" fs_status fs_ipc_close(void* dev_ptr) {
  if (dev_ptr == nullptr) {
    fsb::set_error("dev_ptr is NULL");
    return FS_EINVAL;
  }
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) {
    fsb::set_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return FS_ELAUNCH;
  }
  return FS_OK;
}

extern "C" uint64_t fs_workspace_size(const fs_sample_args* a) { return fsb::workspace_size(a); }

extern "C" fs_status fs_plan(int64_t batch, int64_t vocab, int64_t top_k, int32_t splits,
                             fs_plan_info* out) {
  if (out == nullptr || batch < 1 || vocab < 1 || top_k < 1) {
    fsb::set_error("invalid fs_plan arguments");
    return FS_EINVAL;
  }
  fsb::PlanOut p;
  fs_status st = fsb::make_plan(batch, vocab, std::min(top_k, vocab), splits, FS_PATH_AUTO, &p);
  if (st != FS_OK) return st;
  out->splits = p.splits;
  out->chunks = p.chunks;
  out->threads = p.threads;
  out->capacity = p.capacity;
  out->maxima_per_thread = p.mpt;
  out->lanes_per_max = p.mgroup;
  out->smem_bytes = p.smem;
  out->path = p.wide ? FS_PATH_WIDE : p.stream ? FS_PATH_STREAM : FS_PATH_CLUSTER;
  out->workspace_bytes = p.workspace;
  return FS_OK;
}
