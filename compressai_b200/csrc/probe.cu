// Diagnostics: random 16-byte codebook-row gather throughput, the ceiling of the M = 1 VQ
// GEMV, through three memory paths:
//   mode 0: global memory, read-only path with an L2 evict-last policy (the GEMV's load form);
//           rows < 65536 restricts the rows touched (e.g. 4096 rows = 64 KB fits in L1);
//   mode 1: shared memory (each CTA stages the first 12,288 rows = 192 KB);
//   mode 2: distributed shared memory: an 8-CTA cluster holds the 1 MiB table (128 KB per CTA)
//           and every gather goes to the CTA owning the row.
//   modes 3 / 4: the index-range-bucketed formulation of the M = 1 GEMV -- each CTA (1024
//           threads, one per SM) holds one 8192-row bucket of the codebook (128 KB) and the
//           activation row (2048 values, fp32 in mode 3, fp16 in mode 4) in shared memory, and
//           every entry (random group position, random row of the bucket) costs one codeword
//           read and one activation read from shared memory plus the 8-wide dot product.
// Each thread walks a private xorshift sequence of row indices with 8 gathers in flight; the
// XOR of all loaded words (or the sum of the dot products) goes to `sink` so no load is dead.
#include <cooperative_groups.h>

#include "gemv_dev.cuh"

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

constexpr int kBucketRows = 8192;

template <bool X16>
__global__ void __launch_bounds__(1024) bucket_probe_kernel(const uint4* __restrict__ cb, int64_t iters,
                                                            uint32_t* sink) {
  extern __shared__ uint4 tab[];                                   // [kBucketRows] codewords
  float* xs = reinterpret_cast<float*>(tab + kBucketRows);          // [2048] fp32 or [2048] fp16
  __half* xh = reinterpret_cast<__half*>(xs);
  for (int i = threadIdx.x; i < kBucketRows; i += blockDim.x) tab[i] = cb[i];
  for (int j = threadIdx.x; j < 2048; j += blockDim.x) {
    const float v = 1.f / (1.f + (float)j);
    if (X16) xh[j] = __float2half_rn(v);
    else xs[j] = v;
  }
  __syncthreads();
  uint32_t s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = (blockIdx.x * 1024u + threadIdx.x) * 7919u + j * 104729u + 1u;
  float acc = 0.f;
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j] = xorshift32(s[j]);
      const uint32_t pos = s[j] & 255u, code = (s[j] >> 8) & (kBucketRows - 1);
      float w[8], xv[8];
      decode8<__half>(tab[code], w);
      if (X16) {
        decode8<__half>(reinterpret_cast<const uint4*>(xh)[pos], xv);
      } else {
        const float4 a = reinterpret_cast<const float4*>(xs)[2 * pos], b = reinterpret_cast<const float4*>(xs)[2 * pos + 1];
        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w; xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) acc = fmaf(w[t], xv[t], acc);
    }
  }
  if (acc == 1234.5f) sink[0] = 1u;  // practically never taken; keeps the loads live
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
  if (mode == 3 || mode == 4) {
    const int smem = kBucketRows * 16 + 2048 * 4;
    auto kern = mode == 3 ? bucket_probe_kernel<false> : bucket_probe_kernel<true>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    kern<<<(unsigned)blocks, 1024, smem, st>>>(t, iters, sink);
    return launch_status();
  }
  return VQ2_ERR_ARG;
}
