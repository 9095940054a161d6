// Codebook-decode GEMV on CUDA cores (fp32 accumulation), dense and expert-indexed.
//
//   y[m, r] = rs * scale[r] * sum_g dot(cb0[idx0[r, g]] (+ cb1[idx1[r, g]]), xr[m, 8g:8g+8])
//
// Work split: a warp owns RW x RPL rows; LPR lanes cover one row (RPL = 32 / LPR rows per
// warp-load), each lane loading 8 consecutive int16 indices (16 B) of its row per chunk with
// one streaming 128-bit load. Each index is decoded by a 16-byte gather of the fp16/bf16
// codebook row (read-only path, L1-allocating, L2 evict-last) and dotted with the 8 matching
// activations held in shared memory as fp32. The residual codebook (3 bpw) is staged in
// shared memory. Lane partial sums are reduced with warp shuffles; lane 0 of each row writes
// the scaled result in the value dtype.
//
// The activation tile in shared memory is padded by 4 floats every 8 groups so that the 8
// lanes of one 128-bit access phase, which read groups 8 apart, hit distinct bank groups.
//
// Semantics: reference vq2/kernels.py:32-78 (_vq_gemv_16_8/_vq_gemv_16, M = 1) and
// :117-176 (_parallel_moe_*: expert-indexed, shared or per-expert activation).
#include <atomic>

#include "common.cuh"

namespace vq2 {

struct GemvArgs {
  const void* x;          // activations, x_dtype
  int x_dtype;
  int64_t x_row_stride;   // elements between activation rows m
  int64_t x_k_stride;     // elements between activation groups of problems (0 = shared)
  int64_t x_k_div;        // problem k reads activation group k / x_k_div
  int M;                  // activation rows
  const int16_t* idx0;    // [E, out, ng]
  const uint8_t* idx1;    // [E, out, ng] or null
  const void* cb0;        // [65536, 8] val
  const void* cb1;        // [256, 8] val or null
  const void* scale;      // [E, out] val
  void* y;                // y_dtype
  int y_dtype;
  int64_t y_row_stride;   // elements between output rows m
  int64_t y_k_stride;     // elements between problems k
  const int32_t* e_ids;   // [K] or null (problem k uses expert 0)
  int64_t num_experts;
  int64_t idx_e_stride;   // out * ng
  int64_t scale_e_stride; // out
  int out;
  int n;
  float rs;
};

// Padded position of activation element (group g, lane t) in shared memory.
__device__ __forceinline__ int xs_pos(int g, int t) { return g * 8 + (g >> 3) * 4 + t; }
__host__ __device__ constexpr int xs_len(int n) { return n + n / 16; }

template <typename TV>
__device__ __forceinline__ void decode8(const uint4 w, float f[8]) {
  float2 a = unpack2<TV>(w.x), b = unpack2<TV>(w.y), c = unpack2<TV>(w.z), d = unpack2<TV>(w.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

template <int LPR, int RW, int MT, bool RES, typename TV>
__global__ void __launch_bounds__(256) vq_gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int n = a.n;
  const int xl = xs_len(n);
  float* xs = smem;                                            // [MT][xl]
  uint4* cb1s = reinterpret_cast<uint4*>(smem + MT * xl);      // [256] when RES

  const int k = blockIdx.y;
  const int m0 = blockIdx.z * MT;
  const int mt = min(MT, a.M - m0);
  int64_t e = 0;
  bool valid = true;
  if (a.e_ids) {
    e = a.e_ids[k];
    valid = (e >= 0 && e < a.num_experts);
    if (!valid) e = 0;
  }

  // ---- activations -> fp32, padded layout ----
  for (int i = threadIdx.x; i < MT * n; i += blockDim.x) {
    const int mi = i / n, j = i - mi * n;
    float v = 0.f;
    if (mi < mt) {
      const int64_t off = (int64_t)(m0 + mi) * a.x_row_stride + (int64_t)(k / a.x_k_div) * a.x_k_stride + j;
      if (a.x_dtype == VQ2_F32) v = static_cast<const float*>(a.x)[off];
      else if (a.x_dtype == VQ2_F16) v = __half2float(static_cast<const __half*>(a.x)[off]);
      else v = __bfloat162float(static_cast<const __nv_bfloat16*>(a.x)[off]);
    }
    xs[mi * xl + xs_pos(j >> 3, j & 7)] = v;
  }
  if (RES) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) cb1s[i] = static_cast<const uint4*>(a.cb1)[i];
  }
  __syncthreads();

  constexpr int RPL = 32 / LPR;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LPR, li = lane % LPR;
  const int row0 = blockIdx.x * (8 * RW * RPL) + warp * (RW * RPL) + sub;
  const int ng = n >> 3;
  const int chunks = ng / (8 * LPR);
  const int16_t* idx0 = a.idx0 + e * a.idx_e_stride;
  const uint8_t* idx1 = RES ? a.idx1 + e * a.idx_e_stride : nullptr;
  const uint4* cb0 = static_cast<const uint4*>(a.cb0);
  const uint64_t pol_s = policy_evict_first();
  const uint64_t pol_c = policy_evict_last();

  float acc[RW][MT];
#pragma unroll
  for (int rw = 0; rw < RW; ++rw)
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) acc[rw][mi] = 0.f;

  for (int c = 0; c < chunks; ++c) {
    const int gl = c * LPR + li;   // this lane's 8-group block index
    const int g0 = gl * 8;
    uint4 iv[RW];
    uint2 jv[RW];
#pragma unroll
    for (int rw = 0; rw < RW; ++rw) {
      const int r = row0 + rw * RPL;
      if (valid && r < a.out) {
        iv[rw] = ld_stream_u4(idx0 + (int64_t)r * ng + g0, pol_s);
        if (RES) jv[rw] = ld_stream_u2(idx1 + (int64_t)r * ng + g0, pol_s);
      } else {
        iv[rw] = make_uint4(0, 0, 0, 0);
        if (RES) jv[rw] = make_uint2(0, 0);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float xv[MT][8];
      const int p = xs_pos(g0 + j, 0);
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const float4 lo = *reinterpret_cast<const float4*>(xs + mi * xl + p);
        const float4 hi = *reinterpret_cast<const float4*>(xs + mi * xl + p + 4);
        xv[mi][0] = lo.x; xv[mi][1] = lo.y; xv[mi][2] = lo.z; xv[mi][3] = lo.w;
        xv[mi][4] = hi.x; xv[mi][5] = hi.y; xv[mi][6] = hi.z; xv[mi][7] = hi.w;
      }
#pragma unroll
      for (int rw = 0; rw < RW; ++rw) {
        const uint32_t w32 = (&iv[rw].x)[j >> 1];
        const uint32_t code = (j & 1) ? (w32 >> 16) : (w32 & 0xffffu);
        float wv[8];
        decode8<TV>(ld_cb_u4(cb0 + code, pol_c), wv);
        if (RES) {
          const uint32_t b = ((&jv[rw].x)[j >> 2] >> ((j & 3) * 8)) & 0xffu;
          float rv[8];
          decode8<TV>(cb1s[b], rv);
#pragma unroll
          for (int t = 0; t < 8; ++t) wv[t] += rv[t];
        }
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
          float s = acc[rw][mi];
#pragma unroll
          for (int t = 0; t < 8; ++t) s = fmaf(wv[t], xv[mi][t], s);
          acc[rw][mi] = s;
        }
      }
    }
  }

#pragma unroll
  for (int rw = 0; rw < RW; ++rw)
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) acc[rw][mi] += __shfl_xor_sync(0xffffffffu, acc[rw][mi], off);

  if (li == 0) {
    const TV* sc = static_cast<const TV*>(a.scale) + e * a.scale_e_stride;
    const int64_t ybase = (int64_t)k * a.y_k_stride;
#pragma unroll
    for (int rw = 0; rw < RW; ++rw) {
      const int r = row0 + rw * RPL;
      if (r < a.out) {
        const float s = valid ? to_f32<TV>(sc[r]) * a.rs : 0.f;
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
          if (mi < mt) {
            const int64_t o = ybase + (int64_t)(m0 + mi) * a.y_row_stride + r;
            const float v = acc[rw][mi] * s;
            if (a.y_dtype == VQ2_F16) static_cast<__half*>(a.y)[o] = __float2half_rn(v);
            else if (a.y_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(v);
            else static_cast<float*>(a.y)[o] = v;
          }
        }
      }
    }
  }
}

// ---- host dispatch ------------------------------------------------------------------------
constexpr int kRW = 2;
constexpr int kMaxXsBytes = 80 * 1024;  // activation tile cap; the rest of the SM's 256 KB stays L1

template <int LPR, int MT, bool RES, typename TV>
static int launch4(const GemvArgs& a, int K, cudaStream_t st) {
  constexpr int rows_per_cta = 8 * kRW * (32 / LPR);
  const int mtiles = (a.M + MT - 1) / MT;
  if (K > 65535 || mtiles > 65535) return VQ2_ERR_SHAPE;  // grid.y / grid.z limits
  const dim3 grid((a.out + rows_per_cta - 1) / rows_per_cta, K, mtiles);
  const size_t smem = (size_t)MT * xs_len(a.n) * sizeof(float) + (RES ? 256 * sizeof(uint4) : 0);
  auto kern = vq_gemv_kernel<LPR, kRW, MT, RES, TV>;
  if (smem > 48 * 1024) {
    // Opt in to the largest dynamic shared memory this kernel can use, once per device.
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(done.load() & bit)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxXsBytes + 4096);
      if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
      done.fetch_or(bit);
    }
  }
  kern<<<grid, 256, smem, st>>>(a);
  return launch_status();
}

template <int LPR, bool RES, typename TV>
static int launch3(const GemvArgs& a, int mt, int K, cudaStream_t st) {
  switch (mt) {
    case 1: return launch4<LPR, 1, RES, TV>(a, K, st);
    case 2: return launch4<LPR, 2, RES, TV>(a, K, st);
    case 4: return launch4<LPR, 4, RES, TV>(a, K, st);
    default: return launch4<LPR, 8, RES, TV>(a, K, st);
  }
}

template <bool RES, typename TV>
static int launch2(const GemvArgs& a, int lpr, int mt, int K, cudaStream_t st) {
  switch (lpr) {
    case 4: return launch3<4, RES, TV>(a, mt, K, st);
    case 8: return launch3<8, RES, TV>(a, mt, K, st);
    case 16: return launch3<16, RES, TV>(a, mt, K, st);
    default: return launch3<32, RES, TV>(a, mt, K, st);
  }
}

// Largest M tile (1, 2, 4, 8) whose fp32 activation tile fits kMaxXsBytes of shared memory,
// leaving the rest of the SM's 256 KB to L1 for codebook rows.
static int pick_mt(int64_t M, int64_t n) {
  int mt = M >= 8 ? 8 : M >= 4 ? 4 : M >= 2 ? 2 : 1;
  while (mt > 1 && (int64_t)mt * xs_len((int)n) * 4 > kMaxXsBytes) mt >>= 1;
  return mt;
}

static int pick_lpr(int64_t ng) {
  const int64_t v = ng / 8;  // 16-byte vectors per row
  if (v % 32 == 0) return 32;
  if (v % 16 == 0) return 16;
  if (v % 8 == 0) return 8;
  if (v % 4 == 0) return 4;
  return 0;
}

int run_gemv(const GemvArgs& a, int K, bool res, int val_dtype, cudaStream_t st) {
  const int lpr = pick_lpr(a.n / 8);
  if (lpr == 0) return VQ2_ERR_SHAPE;
  if ((int64_t)xs_len(a.n) * 4 > kMaxXsBytes) return VQ2_ERR_SHAPE;  // n <= 19264
  const int mt = pick_mt(a.M, a.n);
  if (val_dtype == VQ2_F16)
    return res ? launch2<true, __half>(a, lpr, mt, K, st) : launch2<false, __half>(a, lpr, mt, K, st);
  if (val_dtype == VQ2_BF16)
    return res ? launch2<true, __nv_bfloat16>(a, lpr, mt, K, st) : launch2<false, __nv_bfloat16>(a, lpr, mt, K, st);
  return VQ2_ERR_DTYPE;
}

}  // namespace vq2

static bool dtype_ok(int d) { return d == VQ2_F32 || d == VQ2_F16 || d == VQ2_BF16; }

extern "C" int vq2_gemv(const void* xr, int x_dtype, int64_t M, int64_t x_row_stride, const int16_t* idx0,
                        const uint8_t* idx1, const void* cb0, const void* cb1, const void* scale, int val_dtype,
                        void* y, int y_dtype, int64_t y_row_stride, int64_t out, int64_t n, float rs,
                        void* stream) {
  using namespace vq2;
  if (!xr || !idx0 || !cb0 || !scale || !y) return VQ2_ERR_ARG;
  if ((idx1 == nullptr) != (cb1 == nullptr)) return VQ2_ERR_ARG;
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return VQ2_ERR_DTYPE;
  if (M <= 0 || out <= 0 || n <= 0 || n % 64 != 0 || out > INT32_MAX || n > INT32_MAX || M > INT32_MAX)
    return VQ2_ERR_SHAPE;
  if (x_row_stride < n || y_row_stride < out) return VQ2_ERR_SHAPE;
  if (!aligned(idx0, 16) || !aligned(cb0, 16) || (cb1 && !aligned(cb1, 16)) || (idx1 && !aligned(idx1, 8)))
    return VQ2_ERR_ALIGN;
  GemvArgs a{};
  a.x = xr; a.x_dtype = x_dtype; a.x_row_stride = x_row_stride; a.x_k_stride = 0; a.x_k_div = 1;
  a.M = (int)M;
  a.idx0 = idx0; a.idx1 = idx1; a.cb0 = cb0; a.cb1 = cb1; a.scale = scale;
  a.y = y; a.y_dtype = y_dtype; a.y_row_stride = y_row_stride; a.y_k_stride = 0;
  a.e_ids = nullptr; a.num_experts = 1; a.idx_e_stride = 0; a.scale_e_stride = 0;
  a.out = (int)out; a.n = (int)n; a.rs = rs;
  return run_gemv(a, 1, idx1 != nullptr, val_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int vq2_moe_gemv(const void* x, int x_dtype, int64_t x_k_stride, int64_t x_k_div,
                            const int32_t* e_ids, int64_t K, int64_t num_experts, const int16_t* idx,
                            const void* cb0, const void* scale, int val_dtype, void* y, int y_dtype,
                            int64_t out, int64_t ng, float rs, void* stream) {
  using namespace vq2;
  if (!x || !e_ids || !idx || !cb0 || !scale || !y) return VQ2_ERR_ARG;
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return VQ2_ERR_DTYPE;
  if (K <= 0 || num_experts <= 0 || out <= 0 || ng <= 0 || ng % 8 != 0 || out > INT32_MAX || ng * 8 > INT32_MAX)
    return VQ2_ERR_SHAPE;
  if (x_k_stride < 0 || x_k_div <= 0) return VQ2_ERR_SHAPE;
  if (!aligned(idx, 16) || !aligned(cb0, 16)) return VQ2_ERR_ALIGN;
  GemvArgs a{};
  a.x = x; a.x_dtype = x_dtype; a.x_row_stride = 0; a.x_k_stride = x_k_stride; a.x_k_div = x_k_div; a.M = 1;
  a.idx0 = idx; a.idx1 = nullptr; a.cb0 = cb0; a.cb1 = nullptr; a.scale = scale;
  a.y = y; a.y_dtype = y_dtype; a.y_row_stride = 0; a.y_k_stride = out;
  a.e_ids = e_ids; a.num_experts = num_experts; a.idx_e_stride = out * ng; a.scale_e_stride = out;
  a.out = (int)out; a.n = (int)(ng * 8); a.rs = rs;
  return run_gemv(a, (int)K, false, val_dtype, static_cast<cudaStream_t>(stream));
}
