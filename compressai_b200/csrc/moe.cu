// MoE helper kernels: router (softmax top-k) and routing-weighted combine of expert outputs.
#include <cfloat>

#include "gemv.cuh"

namespace vq2 {

// Router, one warp per token: softmax over E logits, top-k, renormalised weights -- the math of
// transformers Qwen3_5MoeTopKRouter.forward (softmax fp32 -> topk -> /= sum). Selection runs on
// the logits (softmax is monotonic) with ties to the lower expert id; the renormalised weight
// of a selected expert is exp(l_i - l_max) / sum_selected exp(l_j - l_max) because the full
// softmax denominator cancels. Optionally the shared expert's weight sigmoid(h . g).
constexpr int kMaxRouteE = 1024;

__global__ void __launch_bounds__(256) moe_route_kernel(const float* __restrict__ logits, int64_t T, int E, int K,
                                                        int32_t* __restrict__ ids, float* __restrict__ w,
                                                        const void* h, int h_dtype, const float* __restrict__ g,
                                                        int64_t H, float* __restrict__ shared_w) {
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  if (t >= T) return;
  constexpr int PER = kMaxRouteE / 32;
  float v[PER];
  const float* lg = logits + t * E;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? lg[e] : -FLT_MAX;
  }
  uint32_t taken = 0;  // bit i: element i*32+lane selected
  float sel_v[32];
  int sel_e[32];
  for (int k = 0; k < K; ++k) {
    float bv = -FLT_MAX;
    int be = INT32_MAX;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && e < be))) { bv = v[i]; be = e; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    if (be != INT32_MAX && (be & 31) == lane) taken |= 1u << (be >> 5);
    sel_v[k] = bv;
    sel_e[k] = be;
  }
  if (lane == 0) {
    const float mx = sel_v[0];
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum += __expf(sel_v[k] - mx);
    for (int k = 0; k < K; ++k) {
      ids[t * K + k] = sel_e[k];
      w[t * K + k] = __expf(sel_v[k] - mx) / sum;
    }
  }
  if (g != nullptr) {
    float d = 0.f;
    for (int64_t i = lane; i < H; i += 32) {
      float hv;
      if (h_dtype == VQ2_F32) hv = static_cast<const float*>(h)[t * H + i];
      else if (h_dtype == VQ2_F16) hv = __half2float(static_cast<const __half*>(h)[t * H + i]);
      else hv = __bfloat162float(static_cast<const __nv_bfloat16*>(h)[t * H + i]);
      d = fmaf(hv, g[i], d);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    if (lane == 0) shared_w[t] = 1.f / (1.f + __expf(-d));
  }
}

// Combine: out[t] = sum_j w[t, j] * y[t*top_k + j] (+ add[t]) in fixed j order (fp32) --
// `(y_down * topk_w[:, None]).sum(0)` of reference PagedMoEExpert.forward
// (vq2/paged_runtime.py:510, :566) plus the shared-expert add of the installed transformers
// Qwen3_5MoeSparseMoeBlock.forward.

__global__ void __launch_bounds__(256) moe_combine_kernel(const float* __restrict__ y, const float* __restrict__ w,
                                                          int64_t T, int top_k, int64_t H,
                                                          const float* __restrict__ add, void* out, int out_dtype,
                                                          const int32_t* __restrict__ ids, int64_t num_experts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  if (i >= T * H) return;
  const int64_t t = i / H, h = i - t * H;
  float s = add ? add[i] : 0.f;
  for (int j = 0; j < top_k; ++j) {
    const int64_t p = t * top_k + j;
    if (ids && (ids[p] < 0 || ids[p] >= num_experts)) continue;  // problem not computed here
    s = fmaf(w[p], y[p * H + h], s);
  }
  if (out_dtype == VQ2_F16) static_cast<__half*>(out)[i] = __float2half_rn(s);
  else if (out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(s);
  else static_cast<float*>(out)[i] = s;
}

int run_combine(const float* y, const float* w, int64_t T, int top_k, int64_t H, const float* add, void* out,
                int out_dtype, cudaStream_t st, const int32_t* ids, int64_t num_experts) {
  const int64_t total = T * H;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  return launch_kernel(moe_combine_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, y, w, T, top_k,
                       H, add, out, out_dtype, ids, num_experts);
}

// Stable compaction with one CTA of 1024 threads: per 1024-problem chunk, a ballot gives each
// warp's count, a scan over the 32 warp counts gives offsets, and kept problems are written
// in their original order. The ids come from device memory, or (ids == nullptr, P <= 64) by
// value in the launch parameters, in which case they are also written to ids_copy for the
// kernels that follow.
__global__ void __launch_bounds__(1024) moe_compact_kernel(const int32_t* __restrict__ ids, IdsByValue iv, int64_t P,
                                                           int64_t num_experts, int32_t* __restrict__ out_ids,
                                                           int32_t* __restrict__ out_map, int32_t* __restrict__ count,
                                                           int32_t* __restrict__ ids_copy) {
  __shared__ int warp_tot[32];
  __shared__ int base;
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (int64_t c0 = 0; c0 < P; c0 += 1024) {
    const int64_t p = c0 + threadIdx.x;
    const int32_t id = p < P ? (ids ? ids[p] : iv.v[p < kIdsByValue ? p : 0]) : -1;
    if (ids_copy && p < P) ids_copy[p] = id;
    const bool keep = p < P && id >= 0 && id < num_experts;
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) warp_tot[warp] = __popc(m);
    __syncthreads();
    int off = base;
    for (int w = 0; w < warp; ++w) off += warp_tot[w];
    if (keep) {
      const int pos = off + __popc(m & ((1u << lane) - 1u));
      out_ids[pos] = id;
      out_map[pos] = static_cast<int32_t>(p);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += warp_tot[w];
      base += tot;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = base;
}

int run_compact(const int32_t* ids, int64_t P, int64_t num_experts, int32_t* out_ids, int32_t* out_map,
                int32_t* out_count, cudaStream_t st, const int32_t* host_ids, int32_t* ids_copy) {
  if (P <= 0 || P > 65536) return VQ2_ERR_SHAPE;
  IdsByValue iv{};
  if (host_ids) {
    if (P > kIdsByValue || !ids_copy) return VQ2_ERR_SHAPE;
    for (int64_t p = 0; p < P; ++p) iv.v[p] = host_ids[p];
    ids = nullptr;
  }
  return launch_kernel(moe_compact_kernel, dim3(1), dim3(1024), 0, st, ids, iv, P, num_experts, out_ids, out_map,
                       out_count, host_ids ? ids_copy : nullptr);
}

}  // namespace vq2

extern "C" int vq2_moe_combine(const float* y, const float* w, int64_t T, int64_t top_k, int64_t H,
                               const float* add, void* out, int out_dtype, void* stream) {
  using namespace vq2;
  if (!y || !w || !out) return VQ2_ERR_ARG;
  if (T <= 0 || top_k <= 0 || top_k > 64 || H <= 0) return VQ2_ERR_SHAPE;
  if (out_dtype != VQ2_F32 && out_dtype != VQ2_F16 && out_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  return run_combine(y, w, T, (int)top_k, H, add, out, out_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int vq2_moe_route(const float* logits, int64_t T, int64_t E, int64_t K, int32_t* ids, float* w,
                             const void* h, int h_dtype, const float* shared_gate, int64_t H, float* shared_w,
                             void* stream) {
  using namespace vq2;
  if (!logits || !ids || !w) return VQ2_ERR_ARG;
  if (T <= 0 || E <= 0 || E > kMaxRouteE || K <= 0 || K > 32 || K > E) return VQ2_ERR_SHAPE;
  if (shared_gate && (!h || !shared_w || H <= 0)) return VQ2_ERR_ARG;
  if (shared_gate && h_dtype != VQ2_F32 && h_dtype != VQ2_F16 && h_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  const int64_t blocks = (T * 32 + 255) / 256;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  return launch_kernel(moe_route_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), logits, T, (int)E, (int)K, ids, w, h, h_dtype,
                       shared_gate, H, shared_w);
}
