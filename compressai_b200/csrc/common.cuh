// Shared device/host helpers for the VQ2 sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "vq2_b200.h"

namespace vq2 {

// Last CUDA runtime error seen by an entry point (for vq2_last_cuda_error()).
void set_last_cuda_error(cudaError_t e);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return VQ2_ERR_LAUNCH;
  }
  return VQ2_OK;
}

__host__ __device__ inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- value conversions ---------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Two packed 16-bit values (low half first) -> two floats.
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  // bf16 -> fp32 is a 16-bit left shift of the bit pattern.
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// ---- memory access with cache hints ----------------------------------------------------------
// L2 cache policies (createpolicy): streaming data is evicted first, the codebook last.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Streaming read of data used once (index tiles): read-only path, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint2 ld_stream_u2(const void* p, uint64_t pol) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(v.x), "=r"(v.y) : "l"(p), "l"(pol));
  return v;
}
// Codebook gather: read-only path, allocate in L1, keep in L2.
__device__ __forceinline__ uint4 ld_cb_u4(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::evict_last.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
  return v;
}

// ---- programmatic dependent launch (PDL) ------------------------------------------------------
// A kernel launched with programmatic stream serialization may start while the previous kernel
// in the stream is still running. It must call pdl_wait() before reading anything that kernel
// wrote (or writing anything it reads); work on constant inputs (weights) may come earlier.
// pdl_trigger() lets the next kernel in the stream start its own pre-wait portion.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether launches carry the PDL attribute (environment VQ2_PDL=0 disables it).
bool pdl_enabled();

// Launch `kern` on `st` with the PDL attribute when enabled; returns a VQ2 status.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return VQ2_ERR_LAUNCH;
  }
  return launch_status();
}

// Whether decode-sized MoE FFNs use the fused single-launch kernel (environment VQ2_MOE_FUSED=0
// selects the four-kernel path; both compute the same values).
bool moe_fused_enabled();

// Launch `kern` as clusters of `cluster_x` CTAs along x (plus the PDL attribute when enabled).
template <typename... KArgs, typename... Args>
int launch_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_x, cudaStream_t st,
                   Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = cluster_x;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return VQ2_ERR_LAUNCH;
  }
  return launch_status();
}

// ---- flags between GPUs over peer memory -----------------------------------------------------
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// The flag handshake of one CTA with every other rank, by ALL 32 lanes of one warp, after a CTA
// barrier that follows the CTA's stores into the peers' buffers. Each flag array lives at the
// base of a rank's buffer; this CTA's flag for sender s is word s * stride + b. Lane q (one per
// peer, in rounds of 32): a system-scope fence (it covers the CTA's earlier peer stores, ordered
// before it by the barrier), sequence number e into flag [rank][b] of peer q (release store), then
// a bounded wait (max_polls acquire loads, napping after the first tight_polls) until flag [q][b]
// of the local buffer has reached e. The peers are served in parallel, one per lane: serially,
// every release and every acquire is a system-scope round trip. Returns false on every lane when
// any wait gave up, after lane 0 raised *err to `timeout_code`; nothing traps. The caller's CTA
// barrier afterwards orders the acquires before the other threads' reads of the peers' data.
__device__ inline bool peer_flags_handshake(uint8_t* const* peers, int rank, int world, int stride, int b,
                                            uint32_t e, int max_polls, int tight_polls, int32_t* err,
                                            int timeout_code) {
  const int lane = threadIdx.x & 31;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(peers[rank]);
  bool ok = true;
  for (int q0 = 0; q0 < world; q0 += 32) {
    const int q = q0 + lane;
    if (q < world && q != rank) {
      fence_acq_rel_sys();
      st_release_sys(reinterpret_cast<uint32_t*>(peers[q]) + rank * stride + b, e);
      int it = 0;
      while ((int)(ld_acquire_sys(flags + q * stride + b) - e) < 0 && it < max_polls) {
        if (it >= tight_polls) __nanosleep(64);
        ++it;
      }
      if (it == max_polls) ok = false;
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0 && err) atomicMax(err, timeout_code);
  return ok;
}

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

}  // namespace vq2
