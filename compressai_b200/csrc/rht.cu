// Randomized Hadamard transform (RHT), forward and inverse, fp32 result; plus the SwiGLU
// activation fused in front of the forward transform.
//
// One hb-point block of one row is a "segment", owned by T = hb/8 threads holding 8 values
// each. The Walsh-Hadamard butterflies (one per bit of the in-block index; their order is
// free) run in three register-resident phases:
//   1. thread t holds elements t + T*i (i = 0..7): bits of value hb/8, hb/4, hb/2;
//   2. after one shared-memory transpose thread t holds 8t .. 8t+7: bits 1, 2, 4;
//   3. the remaining bits 8 .. hb/16 are thread-index bits 1 .. T/16, exchanged with warp
//      shuffles (T/16 <= 16, so partners are always in the same warp).
// Forward: gather x[perm[j]] * sign[j] on load, contiguous store. Inverse: contiguous load,
// multiply by sign[j] and scatter to perm[j] on store.
// Forward results are fp32, or (for the tensor-core GEMV's A/B operand) split into a 16-bit
// high half and the 16-bit rounding of the remainder, as that GEMV's split_hilo kernel does.
// Semantics: Rot.fwd / Rot.inv in reference vq2/vq.py:66-87 (perm gather, sign, blocked
// Sylvester Hadamard, hb^-0.5), FastRot in vq2/runtime.py:57-63 (out_scale = 1), and the
// SwiGLU + rot_512.fwd of PagedMoEExpert.forward, vq2/paged_runtime.py:501-504.
#include <type_traits>

#include "gemv.cuh"

namespace vq2 {

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

enum RhtMode { kForward = 0, kInverse = 1, kSwiGLU = 2 };

template <typename TX>
__device__ __forceinline__ float ldx(const void* x, int64_t i) {
  return to_f32<TX>(static_cast<const TX*>(x)[i]);
}

// silu(g) = g * sigmoid(g). Fast division (reciprocal + multiply): the IEEE-exact divide is a
// multi-instruction sequence, and the staging of a SwiGLU row evaluates thousands of these.
// 1 + exp(-g) beyond 2^126 (g < -87) gives 0, the limit of g * sigmoid(g).
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.f + __expf(-g)); }

// TO = float: fp32 result in xr. TO = __half / __nv_bfloat16 (forward modes only): the result w
// stored as hi = TO(w) in xr and lo = TO(w - float(hi)) in xl, both [M, n] with row stride
// xr_row_stride; with xl null only the hi half is written.
template <int LOG_HB, int MODE, typename TX, typename TO = float>
__global__ void __launch_bounds__(256) rht_kernel(const void* __restrict__ x, int64_t x_row_stride, int64_t M,
                                                  int64_t n, const int32_t* __restrict__ perm,
                                                  const int8_t* __restrict__ sign, float out_scale,
                                                  void* __restrict__ xr_, int64_t xr_row_stride,
                                                  void* __restrict__ xl_ = nullptr) {
  constexpr int HBK = 1 << LOG_HB;
  constexpr int T = HBK / 8;    // threads per segment
  constexpr int SEG = 256 / T;  // segments per CTA
  __shared__ float sm[SEG][HBK + HBK / 32];  // one pad float every 32 spreads the banks

  const int s = threadIdx.x / T;
  const int t = threadIdx.x % T;
  const int64_t nb = n / HBK;
  const int64_t gs = static_cast<int64_t>(blockIdx.x) * SEG + s;
  const bool active = gs < M * nb;
  const int64_t m = active ? gs / nb : 0;
  const int64_t base = active ? (gs % nb) * HBK : 0;
  const int64_t xrow = m * x_row_stride;
  pdl_wait();  // x may be the previous kernel's output (the tables are constant but few)

  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float val = 0.f;
    if (active) {
      const int64_t j = base + t + T * i;
      if (MODE == kInverse) {
        val = ldx<TX>(x, xrow + j);
      } else if (MODE == kForward) {
        val = ldx<TX>(x, xrow + perm[j]) * static_cast<float>(sign[j]);
      } else {  // kSwiGLU: x is fp32 [M, 2n] = [gate | up]
        const int64_t p = perm[j];
        const float g = ldx<float>(x, xrow + p), u = ldx<float>(x, xrow + n + p);
        val = silu_f(g) * u * static_cast<float>(sign[j]);
      }
    }
    v[i] = val;
  }
  fwht8(v);  // bits hb/8, hb/4, hb/2 (value index i <-> element t + T*i)
  auto sidx = [](int e) { return e + (e >> 5); };
#pragma unroll
  for (int i = 0; i < 8; ++i) sm[s][sidx(t + T * i)] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = sm[s][sidx(8 * t + i)];
  fwht8(v);  // bits 1, 2, 4
#pragma unroll
  for (int td = 1; td <= T / 16; td <<= 1) {
    const bool upper = (t & td) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float p = __shfl_xor_sync(0xffffffffu, v[i], td);
      v[i] = upper ? (p - v[i]) : (v[i] + p);
    }
  }
  if (!active) return;
  const int64_t j0 = base + 8 * t;
  if constexpr (!std::is_same<TO, float>::value) {  // hi / lo split for the tensor-core GEMV
    TO hi[8], lo[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float w = v[i] * out_scale;
      hi[i] = from_f32<TO>(w);
      lo[i] = from_f32<TO>(w - to_f32<TO>(hi[i]));
    }
    TO* oh = static_cast<TO*>(xr_) + m * xr_row_stride + j0;
    TO* ol = xl_ ? static_cast<TO*>(xl_) + m * xr_row_stride + j0 : nullptr;  // null: hi only
    if (aligned(oh, 16) && (!ol || aligned(ol, 16))) {
      *reinterpret_cast<uint4*>(oh) = *reinterpret_cast<const uint4*>(hi);
      if (ol) *reinterpret_cast<uint4*>(ol) = *reinterpret_cast<const uint4*>(lo);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        oh[i] = hi[i];
        if (ol) ol[i] = lo[i];
      }
    }
    return;
  }
  float* o = static_cast<float*>(xr_) + m * xr_row_stride;
  if (MODE == kInverse) {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[perm[j0 + i]] = v[i] * out_scale * static_cast<float>(sign[j0 + i]);
  } else if (aligned(o + j0, 16)) {
    reinterpret_cast<float4*>(o + j0)[0] =
        make_float4(v[0] * out_scale, v[1] * out_scale, v[2] * out_scale, v[3] * out_scale);
    reinterpret_cast<float4*>(o + j0)[1] =
        make_float4(v[4] * out_scale, v[5] * out_scale, v[6] * out_scale, v[7] * out_scale);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[j0 + i] = v[i] * out_scale;
  }
}

template <int MODE, typename TX, typename TO = float>
static int launch_rht(const void* x, int64_t xs, int64_t M, int64_t n, int log_hb, const int32_t* perm,
                      const int8_t* sign, float scale, void* xr, int64_t xrs, cudaStream_t st, void* xl = nullptr) {
  const int T = (1 << log_hb) / 8;
  const int seg = 256 / T;
  const int64_t segs = M * (n >> log_hb);
  const int64_t blocks = (segs + seg - 1) / seg;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  const dim3 grid(static_cast<unsigned>(blocks));
  switch (log_hb) {
#define VQ2_RHT_CASE(L) \
  case L: return launch_kernel(rht_kernel<L, MODE, TX, TO>, grid, dim3(256), 0, st, x, xs, M, n, perm, sign, scale, xr, xrs, xl);
    VQ2_RHT_CASE(6) VQ2_RHT_CASE(7) VQ2_RHT_CASE(8) VQ2_RHT_CASE(9) VQ2_RHT_CASE(10) VQ2_RHT_CASE(11)
#undef VQ2_RHT_CASE
    default: return VQ2_ERR_SHAPE;
  }
}

static int log2_hb(int64_t n, int64_t hb) {
  if (n <= 0 || hb < 64 || hb > 2048 || (hb & (hb - 1)) != 0 || n % hb != 0) return -1;
  int l = 0;
  while ((int64_t(1) << l) < hb) ++l;
  return l;
}

// Forward RHT (x_mode RHT: x in x_dtype) or SwiGLU + RHT (x_mode SWIGLU_RHT: fp32 [gate | up])
// of M rows, written as the hi / lo operand halves of the tensor-core GEMV (xh, xl: [M, n] in
// val_dtype). One launch instead of a transform followed by the split.
int rht_split(const void* x, int x_dtype, int x_mode, int64_t x_row_stride, int64_t M, int64_t n, int64_t hb,
              const int32_t* perm, const int8_t* sign, float scale, void* xh, void* xl, int val_dtype,
              cudaStream_t st) {
  const int l = log2_hb(n, hb);
  if (l < 0 || M <= 0) return VQ2_ERR_SHAPE;
  if (x_mode == VQ2_ACT_SWIGLU_RHT) {
    if (x_dtype != VQ2_F32) return VQ2_ERR_DTYPE;
    return val_dtype == VQ2_F16 ? launch_rht<kSwiGLU, float, __half>(x, x_row_stride, M, n, l, perm, sign, scale, xh, n, st, xl)
                                : launch_rht<kSwiGLU, float, __nv_bfloat16>(x, x_row_stride, M, n, l, perm, sign, scale, xh, n, st, xl);
  }
  if (x_mode != VQ2_ACT_RHT) return VQ2_ERR_ARG;
#define VQ2_RHT_SPLIT(TXT)                                                                                     \
  return val_dtype == VQ2_F16                                                                                  \
             ? launch_rht<kForward, TXT, __half>(x, x_row_stride, M, n, l, perm, sign, scale, xh, n, st, xl)   \
             : launch_rht<kForward, TXT, __nv_bfloat16>(x, x_row_stride, M, n, l, perm, sign, scale, xh, n, st, xl);
  switch (x_dtype) {
    case VQ2_F32: VQ2_RHT_SPLIT(float)
    case VQ2_F16: VQ2_RHT_SPLIT(__half)
    case VQ2_BF16: VQ2_RHT_SPLIT(__nv_bfloat16)
    default: return VQ2_ERR_DTYPE;
  }
#undef VQ2_RHT_SPLIT
}

}  // namespace vq2

extern "C" int vq2_rht(const void* x, int x_dtype, int64_t x_row_stride, int64_t M, int64_t n, int64_t hb,
                       const int32_t* perm, const int8_t* sign, float out_scale, int inverse, float* xr,
                       int64_t xr_row_stride, void* stream) {
  using namespace vq2;
  if (!x || !perm || !sign || !xr) return VQ2_ERR_ARG;
  const int l = log2_hb(n, hb);
  if (M <= 0 || l < 0 || x_row_stride < n || xr_row_stride < n) return VQ2_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VQ2_RHT_DT(MODE)                                                                              \
  switch (x_dtype) {                                                                                  \
    case VQ2_F32: return launch_rht<MODE, float>(x, x_row_stride, M, n, l, perm, sign, out_scale, xr, xr_row_stride, st); \
    case VQ2_F16: return launch_rht<MODE, __half>(x, x_row_stride, M, n, l, perm, sign, out_scale, xr, xr_row_stride, st); \
    case VQ2_BF16: return launch_rht<MODE, __nv_bfloat16>(x, x_row_stride, M, n, l, perm, sign, out_scale, xr, xr_row_stride, st); \
    default: return VQ2_ERR_DTYPE;                                                                    \
  }
  if (inverse) { VQ2_RHT_DT(kInverse) } else { VQ2_RHT_DT(kForward) }
#undef VQ2_RHT_DT
}

extern "C" int vq2_swiglu_rht(const float* gu, int64_t gu_row_stride, int64_t M, int64_t n, int64_t hb,
                              const int32_t* perm, const int8_t* sign, float out_scale, float* xr,
                              int64_t xr_row_stride, void* stream) {
  using namespace vq2;
  if (!gu || !perm || !sign || !xr) return VQ2_ERR_ARG;
  const int l = log2_hb(n, hb);
  if (M <= 0 || l < 0 || gu_row_stride < 2 * n || xr_row_stride < n) return VQ2_ERR_SHAPE;
  return launch_rht<kSwiGLU, float>(gu, gu_row_stride, M, n, l, perm, sign, out_scale, xr, xr_row_stride,
                                    static_cast<cudaStream_t>(stream));
}
