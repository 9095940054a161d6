// MoE helper kernels: routing-weighted combine of expert outputs.
// Semantics: `(y_down * topk_w[:, None]).sum(0)` of reference PagedMoEExpert.forward
// (vq2/paged_runtime.py:510, :566) plus the shared-expert add of the installed transformers
// Qwen3_5MoeSparseMoeBlock.forward; the sum runs in fixed expert order in fp32.
#include "common.cuh"

namespace vq2 {

__global__ void __launch_bounds__(256) moe_combine_kernel(const float* __restrict__ y, const float* __restrict__ w,
                                                          int64_t T, int top_k, int64_t H,
                                                          const float* __restrict__ add, void* out, int out_dtype) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T * H) return;
  const int64_t t = i / H, h = i - t * H;
  float s = add ? add[i] : 0.f;
  for (int j = 0; j < top_k; ++j) s = fmaf(w[t * top_k + j], y[(t * top_k + j) * H + h], s);
  if (out_dtype == VQ2_F16) static_cast<__half*>(out)[i] = __float2half_rn(s);
  else if (out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(s);
  else static_cast<float*>(out)[i] = s;
}

}  // namespace vq2

extern "C" int vq2_moe_combine(const float* y, const float* w, int64_t T, int64_t top_k, int64_t H,
                               const float* add, void* out, int out_dtype, void* stream) {
  using namespace vq2;
  if (!y || !w || !out) return VQ2_ERR_ARG;
  if (T <= 0 || top_k <= 0 || top_k > 64 || H <= 0) return VQ2_ERR_SHAPE;
  if (out_dtype != VQ2_F32 && out_dtype != VQ2_F16 && out_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  const int64_t total = T * H;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  moe_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      y, w, T, (int)top_k, H, add, out, out_dtype);
  return launch_status();
}
