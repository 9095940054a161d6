// Row decode of a VQ matrix: selected rows, dequantized in fp32, optionally brought back from the
// rotated space by the inverse randomized Hadamard transform -- the embedding lookup of a tied,
// VQ-compressed embedding (reference PackedEmbedding.forward, vq2/runtime.py:116-133) and the
// rotated-space row decode of PackedLinear.weight_rows (vq2/runtime.py:82-89).
//
// One CTA per requested row, n / 8 threads (n a multiple of 256, <= 8192): thread g gathers the codeword of index
// group g (plus the residual codeword at 3 bpw), scales it by the row scale and leaves the 8
// values in shared memory; with the inverse transform the CTA then runs blocked Sylvester
// Hadamard butterflies over each hb-element segment (3 stages in registers, a transpose through
// shared memory, 3 more in registers, the rest by warp shuffles), multiplies by hb^-1/2 and the
// sign, and scatters element j to position perm[j].
#include "gemv_dev.cuh"

namespace vq2 {

template <typename TV>
__global__ void __launch_bounds__(1024) embed_rows_kernel(const int64_t* __restrict__ ids, int64_t rows,
                                                          const int16_t* __restrict__ idx0,
                                                          const uint8_t* __restrict__ idx1, const void* cb0,
                                                          const void* cb1, const void* scale, int n, int hb,
                                                          const int32_t* __restrict__ perm,
                                                          const int8_t* __restrict__ sign, float inv_scale,
                                                          void* out, int out_dtype, int32_t* bad) {
  extern __shared__ float es[];  // [n] decoded row, then [segments][hb + hb/32] transpose scratch
  const int ng = n >> 3, g = threadIdx.x;
  const int64_t id = ids[blockIdx.x];
  if (id < 0 || id >= rows) {  // out-of-range token: zero row, flag it
    if (g == 0) atomicOr(bad, 1);
    for (int j = g; j < n; j += blockDim.x) {
      const int64_t o = (int64_t)blockIdx.x * n + j;
      if (out_dtype == VQ2_F16) static_cast<__half*>(out)[o] = __float2half_rn(0.f);
      else if (out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(0.f);
      else static_cast<float*>(out)[o] = 0.f;
    }
    return;
  }
  const float sc = to_f32<TV>(static_cast<const TV*>(scale)[id]);
  float v[8];
  {
    const uint32_t code = static_cast<uint16_t>(idx0[id * ng + g]);
    decode8<TV>(static_cast<const uint4*>(cb0)[code], v);
    if (idx1 != nullptr) {
      float r[8];
      decode8<TV>(static_cast<const uint4*>(cb1)[idx1[id * ng + g]], r);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] += r[i];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] *= sc;
  }
  if (perm == nullptr) {  // rotated-space row
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t o = (int64_t)blockIdx.x * n + 8 * g + i;
      if (out_dtype == VQ2_F16) static_cast<__half*>(out)[o] = __float2half_rn(v[i]);
      else if (out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(v[i]);
      else static_cast<float*>(out)[o] = v[i];
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) es[8 * g + i] = v[i];
  __syncthreads();
  // inverse transform, segment s of hb elements handled by T = hb / 8 threads
  const int T = hb >> 3, s = g / T, t = g % T;
  float* sc2 = es + n + s * (hb + (hb >> 5));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = es[s * hb + t + T * i];
  fwht8(v);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = t + T * i;
    sc2[e + (e >> 5)] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = 8 * t + i;
    v[i] = sc2[e + (e >> 5)];
  }
  fwht8(v);
  for (int td = 1; td <= (T >> 4); td <<= 1) {
    const bool upper = (t & td) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q = __shfl_xor_sync(0xffffffffu, v[i], td);
      v[i] = upper ? (q - v[i]) : (v[i] + q);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int j = s * hb + 8 * t + i;
    const float w = v[i] * inv_scale * static_cast<float>(sign[j]);
    const int64_t o = (int64_t)blockIdx.x * n + perm[j];
    if (out_dtype == VQ2_F16) static_cast<__half*>(out)[o] = __float2half_rn(w);
    else if (out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(w);
    else static_cast<float*>(out)[o] = w;
  }
}

}  // namespace vq2

extern "C" int vq2_embed_rows(const int64_t* ids, int64_t count, int64_t rows, const int16_t* idx0, const uint8_t* idx1,
                              const void* cb0, const void* cb1, const void* scale, int val_dtype, int64_t n,
                              const int32_t* perm, const int8_t* sign, int64_t hb, float inv_scale, void* out,
                              int out_dtype, int32_t* bad, void* stream) {
  using namespace vq2;
  if (!ids || !idx0 || !cb0 || !scale || !out || !bad) return VQ2_ERR_ARG;
  if ((idx1 == nullptr) != (cb1 == nullptr) || (perm == nullptr) != (sign == nullptr)) return VQ2_ERR_ARG;
  if (count <= 0 || count > INT32_MAX || rows <= 0 || n <= 0 || n % 256 != 0 || n > 8192) return VQ2_ERR_SHAPE;  // whole warps
  if (perm && (hb < 64 || hb > 2048 || (hb & (hb - 1)) != 0 || n % hb != 0)) return VQ2_ERR_SHAPE;
  if (out_dtype != VQ2_F32 && out_dtype != VQ2_F16 && out_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (!aligned(cb0, 16) || (cb1 && !aligned(cb1, 16))) return VQ2_ERR_ALIGN;
  const int threads = (int)(n / 8);
  const size_t smem = perm ? ((size_t)n + (size_t)(n / hb) * (hb + hb / 32)) * sizeof(float) : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) {  // up to 66.5 KB at n = 8192
    const cudaError_t e = val_dtype == VQ2_F16
        ? cudaFuncSetAttribute(embed_rows_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
        : cudaFuncSetAttribute(embed_rows_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return VQ2_ERR_LAUNCH;
    }
  }
  if (val_dtype == VQ2_F16)
    return launch_kernel(embed_rows_kernel<__half>, dim3((unsigned)count), dim3(threads), smem, st, ids, rows, idx0,
                         idx1, cb0, cb1, scale, (int)n, (int)hb, perm, sign, inv_scale, out, out_dtype, bad);
  if (val_dtype == VQ2_BF16)
    return launch_kernel(embed_rows_kernel<__nv_bfloat16>, dim3((unsigned)count), dim3(threads), smem, st, ids,
                         rows, idx0, idx1, cb0, cb1, scale, (int)n, (int)hb, perm, sign, inv_scale, out, out_dtype,
                         bad);
  return VQ2_ERR_DTYPE;
}

// ---- fixed-width index unpack ----------------------------------------------------------------
// Symbols of a fixed-width stream (vq2/export.py:39-70 layout: 16-bit little-endian words,
// bytes, 4-bit pairs low nibble first, 12-bit pairs in 3 bytes a | b << 12) -> 16-bit or 8-bit
// index elements; one thread per output pair.
namespace vq2 {
__global__ void __launch_bounds__(256) unpack_fixed_kernel(const uint8_t* __restrict__ src, int bits, int64_t n,
                                                           void* __restrict__ dst, int dst_bytes) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // symbol pair
  const int64_t i = 2 * p;
  if (i >= n) return;
  uint32_t a = 0, b = 0;
  if (bits == 16) {
    a = src[2 * i] | (src[2 * i + 1] << 8);
    if (i + 1 < n) b = src[2 * i + 2] | (src[2 * i + 3] << 8);
  } else if (bits == 8) {
    a = src[i];
    if (i + 1 < n) b = src[i + 1];
  } else if (bits == 4) {
    const uint32_t v = src[p];
    a = v & 15u;
    b = v >> 4;
  } else {  // 12
    const uint32_t w = src[3 * p] | (src[3 * p + 1] << 8) | (src[3 * p + 2] << 16);
    a = w & 4095u;
    b = w >> 12;
  }
  if (dst_bytes == 2) {
    static_cast<uint16_t*>(dst)[i] = static_cast<uint16_t>(a);
    if (i + 1 < n) static_cast<uint16_t*>(dst)[i + 1] = static_cast<uint16_t>(b);
  } else {
    static_cast<uint8_t*>(dst)[i] = static_cast<uint8_t>(a);
    if (i + 1 < n) static_cast<uint8_t*>(dst)[i + 1] = static_cast<uint8_t>(b);
  }
}
}  // namespace vq2

extern "C" int64_t vq2_fixed_stream_bytes(int bits, int64_t n) {
  if (n < 0) return -1;
  if (bits == 16) return 2 * n;
  if (bits == 8) return n;
  if (bits == 4) return (n + 1) / 2;
  if (bits == 12) return 3 * ((n + 1) / 2);
  return -1;
}

extern "C" int vq2_unpack_fixed(const uint8_t* src, int64_t src_bytes, int bits, int64_t n, void* dst,
                                int dst_bytes, void* stream) {
  using namespace vq2;
  if (!src || !dst) return VQ2_ERR_ARG;
  if (n <= 0 || (bits != 4 && bits != 8 && bits != 12 && bits != 16)) return VQ2_ERR_SHAPE;
  if (dst_bytes != 1 && dst_bytes != 2) return VQ2_ERR_DTYPE;
  if (bits > 8 && dst_bytes == 1) return VQ2_ERR_DTYPE;  // 12/16-bit symbols need 16-bit elements
  if (src_bytes < vq2_fixed_stream_bytes(bits, n)) return VQ2_ERR_SHAPE;
  const int64_t pairs = (n + 1) / 2, blocks = (pairs + 255) / 256;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  return launch_kernel(unpack_fixed_kernel, dim3((unsigned)blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       src, bits, n, dst, dst_bytes);
}
