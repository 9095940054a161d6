// Diagnostics: random 16-byte codebook-row gather throughput, the ceiling of the M = 1 VQ
// GEMV, through three memory paths:
//   mode 0: global memory, read-only path with an L2 evict-last policy (the GEMV's load form);
//           rows < 65536 restricts the rows touched (e.g. 4096 rows = 64 KB fits in L1);
//   mode 1: shared memory (each CTA stages the first 12,288 rows = 192 KB);
//   mode 2: distributed shared memory: an 8-CTA cluster holds the 1 MiB table (128 KB per CTA)
//           and every gather goes to the CTA owning the row.
// Each thread walks a private xorshift sequence of row indices with 8 gathers in flight; the
// XOR of all loaded words goes to `sink` so no load is dead.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace vq2 {

__device__ __forceinline__ uint32_t xorshift32(uint32_t x) {
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  return x;
}

constexpr int kSmemRows = 12288;
constexpr int kClusterCtas = 8;

template <int MODE>
__global__ void __launch_bounds__(256) gather_probe_kernel(const uint4* __restrict__ cb, uint32_t rows,
                                                           int64_t iters, uint32_t* sink) {
  extern __shared__ uint4 tab[];
  const uint64_t pol = policy_evict_last();
  if (MODE == 1) {
    for (int i = threadIdx.x; i < kSmemRows; i += blockDim.x) tab[i] = cb[i];
    __syncthreads();
  }
  uint4* peer[kClusterCtas];
  if (MODE == 2) {
    cg::cluster_group cl = cg::this_cluster();
    const int per = 65536 / kClusterCtas;
    for (int i = threadIdx.x; i < per; i += blockDim.x) tab[i] = cb[cl.block_rank() * per + i];
    cl.sync();
#pragma unroll
    for (int r = 0; r < kClusterCtas; ++r) peer[r] = cl.map_shared_rank(tab, r);
  }
  uint32_t s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = (blockIdx.x * 256u + threadIdx.x) * 7919u + j * 104729u + 1u;
  uint32_t acc = 0;
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j] = xorshift32(s[j]);
      uint4 v;
      if (MODE == 0) {
        v = ld_cb_u4(cb + (s[j] % rows), pol);
      } else if (MODE == 1) {
        v = tab[s[j] % kSmemRows];
      } else {
        const uint32_t c = s[j] & 0xffffu;
        v = peer[c >> 13][c & 8191u];
      }
      acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
  }
  if (MODE == 2) cg::this_cluster().sync();  // peers' tables stay alive until all reads finish
  if (acc == 0x9e3779b9u) sink[0] = acc;      // practically never taken; keeps the loads live
}

}  // namespace vq2

extern "C" int vq2_gather_probe(const void* cb, int64_t rows, int mode, int64_t blocks, int64_t iters,
                                uint32_t* sink, void* stream) {
  using namespace vq2;
  if (!cb || !sink) return VQ2_ERR_ARG;
  if (rows <= 0 || rows > 65536 || blocks <= 0 || blocks > INT32_MAX || iters <= 0) return VQ2_ERR_SHAPE;
  if (mode != 0 && rows < 65536) return VQ2_ERR_SHAPE;  // the smem modes stage fixed table sizes
  if (!aligned(cb, 16)) return VQ2_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint4* t = static_cast<const uint4*>(cb);
  if (mode == 0) {
    gather_probe_kernel<0><<<(unsigned)blocks, 256, 0, st>>>(t, (uint32_t)rows, iters, sink);
    return launch_status();
  }
  if (mode == 1) {
    const int smem = kSmemRows * 16;
    cudaError_t e = cudaFuncSetAttribute(gather_probe_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    gather_probe_kernel<1><<<(unsigned)blocks, 256, smem, st>>>(t, (uint32_t)rows, iters, sink);
    return launch_status();
  }
  if (mode == 2) {
    const int smem = 65536 / kClusterCtas * 16;
    cudaError_t e = cudaFuncSetAttribute(gather_probe_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((blocks + kClusterCtas - 1) / kClusterCtas * kClusterCtas));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kClusterCtas;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gather_probe_kernel<2>, t, (uint32_t)rows, iters, sink);
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    return launch_status();
  }
  return VQ2_ERR_ARG;
}
