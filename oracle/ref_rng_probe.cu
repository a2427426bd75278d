// Golden-vector probe built against the reference's own device header
// (csrc/fused_sampling.cuh of sathviknookala/llm_sampling_kernel): evaluates its seeded uniform
// rng_uniform(seed, offset, row) (:65-71) and its order key mono_key (:8-11) on the GPU and
// prints them, so the CPU oracle's restatements can be pinned to the reference's own code.
// TEST INFRASTRUCTURE ONLY; built by oracle/Makefile into oracle/_ref/.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdio>
#include <cstdint>

#include "fused_sampling.cuh"

__global__ void rng_kernel(const uint64_t* seeds, const uint64_t* offs, const uint32_t* rows, float* out, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = fs::rng_uniform(seeds[i], offs[i], rows[i]);
}

__global__ void key_kernel(uint32_t* out) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536) out[i] = fs::mono_key(static_cast<uint16_t>(i));
}

int main() {
  const int n = 4096;
  uint64_t hs[n], ho[n];
  uint32_t hr[n];
  uint64_t x = 0x243F6A8885A308D3ull;  // fixed table of (seed, offset, row)
  for (int i = 0; i < n; ++i) {
    x ^= x << 13; x ^= x >> 7; x ^= x << 17;
    hs[i] = (i < 64) ? 0x5EEDull : x;
    ho[i] = (i < 64) ? static_cast<uint64_t>(i) : (x >> 17);
    hr[i] = (i < 64) ? 0u : static_cast<uint32_t>(i * 2654435761u);
  }
  hs[0] = 0; ho[0] = 1; hr[0] = 0;
  uint64_t *ds, *dof; uint32_t* dr; float* du; uint32_t* dk;
  cudaMalloc(&ds, sizeof(hs)); cudaMalloc(&dof, sizeof(ho)); cudaMalloc(&dr, sizeof(hr));
  cudaMalloc(&du, n * sizeof(float)); cudaMalloc(&dk, 65536 * sizeof(uint32_t));
  cudaMemcpy(ds, hs, sizeof(hs), cudaMemcpyHostToDevice);
  cudaMemcpy(dof, ho, sizeof(ho), cudaMemcpyHostToDevice);
  cudaMemcpy(dr, hr, sizeof(hr), cudaMemcpyHostToDevice);
  rng_kernel<<<(n + 255) / 256, 256>>>(ds, dof, dr, du, n);
  key_kernel<<<256, 256>>>(dk);
  static float hu[n];
  static uint32_t hk[65536];
  cudaMemcpy(hu, du, sizeof(hu), cudaMemcpyDeviceToHost);
  cudaMemcpy(hk, dk, sizeof(hk), cudaMemcpyDeviceToHost);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) { fprintf(stderr, "%s\n", cudaGetErrorString(e)); return 1; }
  printf("# rng_uniform seed offset row u_bits\n");
  for (int i = 0; i < n; ++i) {
    uint32_t b; memcpy(&b, &hu[i], 4);
    printf("u %llu %llu %u %08x\n", (unsigned long long)hs[i], (unsigned long long)ho[i], hr[i], b);
  }
  printf("# mono_key bits key\n");
  for (int i = 0; i < 65536; ++i) printf("k %u %u\n", i, hk[i]);
  return 0;
}
