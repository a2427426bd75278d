// Device primitives of the B200 fused sampler: order keys, packed candidates, the seeded
// uniform, block scans/reductions and the shared-memory bitonic sort.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace fsb {

constexpr int kHistBins = 4096;   // 12-bit bins over the 16-bit order key (key >> 4)
constexpr int kMaxSplits = 16;    // CTAs per row = thread-block cluster size

// 16-bit order key of an FP16/BF16 bit pattern. Larger key <=> larger value; -0 is folded onto
// +0 first so that both zeros tie (the reference's stable FP32 sort treats them as equal,
// benchmarks/reference.py:53; the reference kernel's mono_key, csrc/fused_sampling.cuh:8-11,
// does not fold them). Negative values map below 0x8000, positive values at or above it.
__device__ __forceinline__ uint32_t order_key(uint32_t bits) {
  bits = (bits == 0x8000u) ? 0u : bits;
  return (bits & 0x8000u) ? (~bits & 0xFFFFu) : (bits | 0x8000u);
}

// Inverse of order_key on canonical keys (0x8000 decodes to +0).
__device__ __forceinline__ uint32_t key_to_bits(uint32_t key) {
  return (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
}

template <int DT>  // 1 = bf16, 0 = f16
__device__ __forceinline__ float bits_to_float(uint32_t bits) {
  if constexpr (DT == 1) {
    return __uint_as_float(bits << 16);
  } else {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
  }
}

template <int DT>
__device__ __forceinline__ float key_to_float(uint32_t key) {
  return bits_to_float<DT>(key_to_bits(key));
}

// Bit patterns of -inf and +inf, and the NaN test, per 16-bit format.
template <int DT>
struct Fmt {
  static constexpr uint32_t kNegInf = DT ? 0xFF80u : 0xFC00u;
  static constexpr uint32_t kPosInf = DT ? 0x7F80u : 0x7C00u;
  static constexpr uint32_t kNegInf2 = DT ? 0xFF80FF80u : 0xFC00FC00u;
  __device__ static __forceinline__ bool is_nan(uint32_t bits) { return (bits & 0x7FFFu) > kPosInf; }
};

// Packed candidate: key in the high word, (0xFFFFFFFF - id) in the low word, so that a larger
// packed value means a larger logit and, on equal logits, a lower id (the reference's pack,
// csrc/fused_sampling.cuh:13-23). 0 is below every real candidate and serves as padding.
__device__ __forceinline__ uint64_t pack(uint32_t key, uint32_t id) {
  return (static_cast<uint64_t>(key) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - id);
}
__device__ __forceinline__ uint32_t packed_key(uint64_t p) { return static_cast<uint32_t>(p >> 32); }
__device__ __forceinline__ uint32_t packed_id(uint64_t p) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(p & 0xFFFFFFFFull);
}

// Per-pair (two 16-bit lanes of one 32-bit word) max that propagates NaN, and >= test mask.
template <int DT>
__device__ __forceinline__ uint32_t pair_max_nan(uint32_t a, uint32_t b) {
  if constexpr (DT == 1) {
    __nv_bfloat162 r = __hmax2_nan(*reinterpret_cast<__nv_bfloat162*>(&a),
                                   *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  } else {
    __half2 r = __hmax2_nan(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
}

// 0xFFFF in each 16-bit lane where a >= b (IEEE: false on NaN, -0 == +0).
template <int DT>
__device__ __forceinline__ uint32_t pair_ge_mask(uint32_t a, uint32_t b) {
  if constexpr (DT == 1) {
    return __hge2_mask(*reinterpret_cast<__nv_bfloat162*>(&a),
                       *reinterpret_cast<__nv_bfloat162*>(&b));
  } else {
    return __hge2_mask(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  }
}

// Max of two 16-bit values given as bit patterns (NaN-propagating), via the pair op.
template <int DT>
__device__ __forceinline__ uint32_t half_max_nan(uint32_t a, uint32_t b) {
  return pair_max_nan<DT>(a, b) & 0xFFFFu;
}

// The reference's seeded uniform (csrc/fused_sampling.cuh:65-71): splitmix64 finaliser of
// seed + offset * 0x9E3779B97F4A7C15 + row * 0xD1B54A32D192ED03; top 24 bits / 2^24.
// Kept bit-identical so a (seed, offset) pair draws the same u as the reference kernel.
__device__ __forceinline__ float splitmix_uniform(uint64_t seed, uint64_t offset, uint64_t row) {
  uint64_t z = seed + offset * 0x9E3779B97F4A7C15ull + row * 0xD1B54A32D192ED03ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return static_cast<float>(static_cast<uint32_t>(z >> 40)) * (1.0f / 16777216.0f);
}

// ---- block-level helpers (every thread of the CTA must call them) --------------------------

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    T o = __shfl_up_sync(0xFFFFFFFFu, v, off);
    if (lane >= off) v += o;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  return v;
}

__device__ __forceinline__ int warp_min(int v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = min(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  return v;
}

// Inclusive scan over threads in thread order; `scratch` holds >= 33 elements of T.
// Returns the inclusive prefix; *total receives the block total.
template <typename T, int NT>
__device__ __forceinline__ T block_incl_scan(T v, T* scratch, T* total) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T inc = warp_incl_scan(v);
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    T w = lane < NW ? scratch[lane] : T(0);
    T wi = warp_incl_scan(w);
    if (lane < NW) scratch[lane] = wi - w;  // exclusive warp offsets
    if (lane == NW - 1) scratch[32] = wi;
  }
  __syncthreads();
  T res = inc + scratch[warp];
  *total = scratch[32];
  __syncthreads();
  return res;
}

template <typename T, int NT>
__device__ __forceinline__ T block_sum(T v, T* scratch) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = lane < NW ? scratch[lane] : T(0);
    w = warp_sum(w);
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  T r = scratch[32];
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ int block_min(int v, int* scratch) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_min(v);
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < NW ? scratch[lane] : 0x7FFFFFFF;
    w = warp_min(w);
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  int r = scratch[32];
  __syncthreads();
  return r;
}

// Descending bitonic sort of s[0..P) in shared memory, P a power of two.
template <int NT>
__device__ __forceinline__ void block_sort_desc(uint64_t* s, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (P >> 1); i += NT) {
        const int lo = ((i & ~(stride - 1)) << 1) | (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = s[lo], b = s[hi];
        if ((a < b) == desc) {
          s[lo] = b;
          s[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Descending bitonic sort of 32*R values held by one warp in blocked layout
// (lane l owns positions l*R .. l*R+R-1). Compile-time network.
template <int R>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&v)[R]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < R) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int pr = r ^ stride;
          if (pr > r) {
            const int idx = lane * R + r;
            const bool desc = (idx & size) == 0;
            const uint64_t a = v[r], b = v[pr];
            if ((a < b) == desc) {
              v[r] = b;
              v[pr] = a;
            }
          }
        }
      } else {
        const int lstride = stride / R;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, v[r], lstride);
          const int idx = lane * R + r;
          const bool lower = (idx & stride) == 0;
          const bool desc = (idx & size) == 0;
          const bool take_max = (lower == desc);
          v[r] = take_max ? (o > v[r] ? o : v[r]) : (o < v[r] ? o : v[r]);
        }
      }
    }
  }
}

}  // namespace fsb
