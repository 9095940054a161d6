// Device helpers of the VQ GEMV kernels shared by vq_gemv.cu and the fused MoE layer kernel
// (moe_fused.cu): the padded activation tile layout, codebook row decode and the activation
// staging with the fused randomized Hadamard transform.
#pragma once
#include "gemv.cuh"

namespace vq2 {

// Where a GEMV's activations come from and how they are transformed while staged.
struct ActSrc {
  const void* x;          // activations (mode SWIGLU_RHT: fp32 [gate | up] rows of 2n)
  int x_dtype, x_mode, n, hb;
  int64_t x_row_stride;
  const int32_t* perm;
  const int8_t* sign;
  float rot_scale;
};

__device__ __forceinline__ ActSrc act_src(const GemvArgs& a) {
  ActSrc s;
  s.x = a.x; s.x_dtype = a.x_dtype; s.x_mode = a.x_mode; s.n = a.n; s.hb = a.hb;
  s.x_row_stride = a.x_row_stride; s.perm = a.perm; s.sign = a.sign; s.rot_scale = a.rot_scale;
  return s;
}

// Padded position of activation element (group g, lane t) in shared memory.
__device__ __forceinline__ int xs_pos(int g, int t) { return g * 8 + (g >> 3) * 4 + t; }
__host__ __device__ constexpr int xs_len(int n) { return n + n / 16; }

template <typename TV>
__device__ __forceinline__ void decode8(const uint4 w, float f[8]) {
  float2 a = unpack2<TV>(w.x), b = unpack2<TV>(w.y), c = unpack2<TV>(w.z), d = unpack2<TV>(w.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

constexpr int kScratchFloats = 2048 + 64;  // one RHT transpose round: SEG x (hb + hb/32) floats

__device__ __forceinline__ float load_act(const void* x, int dt, int64_t off) {
  if (dt == VQ2_F32) return static_cast<const float*>(x)[off];
  if (dt == VQ2_F16) return __half2float(static_cast<const __half*>(x)[off]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[off]);
}

__device__ __forceinline__ void fwht8(float v[8]) {
#pragma unroll
  for (int d = 1; d < 8; d <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if ((i & d) == 0) {
        const float a = v[i], b = v[i + d];
        v[i] = a + b;
        v[i + d] = a - b;
      }
    }
  }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

// Stage MT activation rows (starting at element offset xoff) into the padded fp32 tile xs.
// Mode ROTATED copies; modes RHT / SWIGLU_RHT apply the forward randomized Hadamard transform
// (perm gather, sign, blocked Sylvester Hadamard, rot_scale) with the whole CTA: a segment of
// hb elements belongs to T = hb/8 threads (8 values each): 3 butterfly stages in registers,
// one transpose through `scratch`, 3 more in registers, the rest with warp shuffles (the same
// scheme as the standalone vq2_rht kernel). Must be called by all 256 threads.
template <int MT>
__device__ void stage_activations(const ActSrc& a, int64_t xoff, int mcount, float* xs, int xl, float* scratch) {
  const int n = a.n;
  if (a.x_mode == VQ2_ACT_ROTATED) {
    for (int i = threadIdx.x; i < MT * n; i += blockDim.x) {
      const int mi = i / n, j = i - mi * n;
      const float v = mi < mcount ? load_act(a.x, a.x_dtype, xoff + (int64_t)mi * a.x_row_stride + j) : 0.f;
      xs[mi * xl + xs_pos(j >> 3, j & 7)] = v;
    }
    return;
  }
  const int hb = a.hb, T = hb >> 3, SEG = 256 / T, nb = n / hb;
  const int s = threadIdx.x / T, t = threadIdx.x % T;
  const int segs = MT * nb;
  const bool swiglu = (a.x_mode == VQ2_ACT_SWIGLU_RHT);
  float* sc = scratch + s * (hb + (hb >> 5));
  for (int s0 = 0; s0 < segs; s0 += SEG) {
    const int gs = s0 + s;
    const int mi = gs / nb, b = gs - mi * nb;
    const bool active = gs < segs && mi < mcount;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float val = 0.f;
      if (active) {
        const int j = b * hb + t + T * i;
        const int64_t row = xoff + (int64_t)mi * a.x_row_stride;
        const int p = a.perm[j];
        if (swiglu) {  // plain loads: L1 lines are reused by the permuted reads of one row; rows
                       // written by other CTAs of the same launch are read only after an acquire
          const float* g = static_cast<const float*>(a.x) + row;
          val = silu_f(g[p]) * g[n + p];
        } else {
          val = load_act(a.x, a.x_dtype, row + p);
        }
        val *= static_cast<float>(a.sign[j]);
      }
      v[i] = val;
    }
    fwht8(v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = t + T * i;
      sc[e + (e >> 5)] = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = 8 * t + i;
      v[i] = sc[e + (e >> 5)];
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
    if (gs < segs) {
      const int g = (b * hb >> 3) + t;  // 8-element group index within the row
      float* o = xs + mi * xl + xs_pos(g, 0);
      const float r = a.rot_scale;
      *reinterpret_cast<float4*>(o) = make_float4(v[0] * r, v[1] * r, v[2] * r, v[3] * r);
      *reinterpret_cast<float4*>(o + 4) = make_float4(v[4] * r, v[5] * r, v[6] * r, v[7] * r);
    }
    __syncthreads();
  }
}


}  // namespace vq2
