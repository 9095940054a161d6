// Diagnostic: random 16-byte codebook-row gather throughput (the ceiling of the M = 1 VQ GEMV).
// Each thread walks a private xorshift sequence of row indices below `rows` and gathers the
// rows with the same load form as the GEMV (read-only path, L2 evict-last policy), 8 gathers
// in flight per thread; the XOR of all loaded words goes to `sink` so no load is dead.
#include "common.cuh"

namespace vq2 {

__device__ __forceinline__ uint32_t xorshift32(uint32_t x) {
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  return x;
}

__global__ void __launch_bounds__(256) gather_probe_kernel(const uint4* __restrict__ cb, uint32_t rows,
                                                           int64_t iters, uint32_t* sink) {
  const uint64_t pol = policy_evict_last();
  uint32_t s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = (blockIdx.x * 256u + threadIdx.x) * 7919u + j * 104729u + 1u;
  uint32_t acc = 0;
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j] = xorshift32(s[j]);
      const uint4 v = ld_cb_u4(cb + (s[j] % rows), pol);
      acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
  }
  if (acc == 0x9e3779b9u) sink[0] = acc;  // practically never taken; keeps the loads live
}

}  // namespace vq2

extern "C" int vq2_gather_probe(const void* cb, int64_t rows, int64_t blocks, int64_t iters, uint32_t* sink,
                                void* stream) {
  using namespace vq2;
  if (!cb || !sink) return VQ2_ERR_ARG;
  if (rows <= 0 || rows > UINT32_MAX || blocks <= 0 || blocks > INT32_MAX || iters <= 0) return VQ2_ERR_SHAPE;
  if (!aligned(cb, 16)) return VQ2_ERR_ALIGN;
  gather_probe_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(cb), (uint32_t)rows, iters, sink);
  return launch_status();
}
