// Batched VQ GEMV (M >= 8 activation rows) on the tensor cores.
//
//   y[m, r] = rs * scale[r] * sum_k W[r, k] * xr[m, k],  W[r, 8g + t] = cb0[idx0[r, g]][t] (+ cb1[idx1[r, g]][t])
//
// At M >= 16 the CUDA-core kernel runs out of FMA and shared-memory bandwidth (8*M FMAs per
// gathered codeword); here the decoded weights feed mma.sync.m16n8k16 (fp32 accumulation)
// straight from the gather, with no shared-memory staging of W:
//   * a warp owns 16 weight rows of an item (a CTA: 8 warps, 128 rows) and all M-tile tokens;
//   * per K chunk of 128 (16 groups) each lane loads one 16-byte vector of its row's indices
//     (prefetched one chunk ahead); the index a lane needs for an MMA step comes from the
//     owning lane by one shuffle per row pair;
//   * the A fragment of one m16n8k16 step is four 4-byte pieces of four codebook rows (row gid
//     and gid+8, groups g and g+1, halves 2*tig..2*tig+1): one codeword is read by the four
//     lanes of a quad, so a warp touches 8 codewords = 8 cache lines per gather instruction,
//     the same L1TEX cost per codeword as the CUDA-core kernel;
//   * the activations are split once per call into 16-bit hi + lo halves (x = hi + lo to
//     ~2^-22 relative, split_hilo_kernel) so two MMAs per step keep the product within fp32
//     accuracy of the oracle; each chunk (M tile x 128 x {hi, lo}) is streamed into a double
//     buffer in shared memory with 16-byte cp.async copies while the previous chunk computes;
//   * 3 bpw adds the residual codebook (shared memory) as a second A operand with its own MMAs,
//     so the two codebooks are never summed in 16-bit;
//   * split-K for matrices with too few 128-row items to fill the GPU: each item is a thread-block
//     cluster of S CTAs (S <= 8), CTA rank r computing K chunks [r * chunks / S, (r+1) * chunks / S);
//     the partial accumulators meet in distributed shared memory and rank 0 adds them in rank
//     order (deterministic) before the epilogue.
// Semantics: the batched form of reference vq2/kernels.py:32-78 (which serves M = 1 only;
// vq2/runtime.py:105-110 dequantizes and calls F.linear for M > 1).
#include <cooperative_groups.h>

#include <atomic>

#include "gemv.cuh"

namespace cg = cooperative_groups;

namespace vq2 {

constexpr int kTcKC = 128;          // K elements per chunk (16 groups)
constexpr int kTcXPad = kTcKC + 8;  // padded activation row (halves): 272 B -> conflict-free B loads

template <typename TV> struct Mma;
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ __half cvt(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float back(__half v) { return __half2float(v); }
};
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ __nv_bfloat16 cvt(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float back(__nv_bfloat16 v) { return __bfloat162float(v); }
};

__device__ __forceinline__ uint32_t ld_cb_u32(const void* p, uint64_t pol) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::evict_last.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int nbytes = valid ? 16 : 0;  // 0: fill the 16 bytes with zeros, read nothing
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(nbytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// x = hi + lo in the 16-bit type TV, hi = round(x), lo = round(x - hi): the operand split of the
// tensor-core path, written once per call for all CTAs (xh [M, n] then xl [M, n]; xl null: hi
// only).
template <typename TV>
__global__ void __launch_bounds__(256) split_hilo_kernel(const void* __restrict__ x, int x_dtype, int64_t M, int64_t n,
                                                         int64_t x_row_stride, TV* __restrict__ xh,
                                                         TV* __restrict__ xl) {
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * n) return;
  const int64_t m = i / n, k = i - m * n;
  const int64_t off = m * x_row_stride + k;
  float v;
  if (x_dtype == VQ2_F32) v = static_cast<const float*>(x)[off];
  else if (x_dtype == VQ2_F16) v = __half2float(static_cast<const __half*>(x)[off]);
  else v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[off]);
  const TV hi = Mma<TV>::cvt(v);
  xh[i] = hi;
  if (xl) xl[i] = Mma<TV>::cvt(v - Mma<TV>::back(hi));
}

// NT: 8-token tiles per M tile (M tile = 8 * NT tokens); RES: 3 bpw. a.x = the hi halves
// [M, n]; the lo halves follow at a.x + M * n (see run_gemm_tc).
template <int NT, bool RES, typename TV>
__global__ void __launch_bounds__(256, 2) vq_gemm_tc_kernel(const GemvArgs a) {
  constexpr int MT = 8 * NT;
  constexpr int XB = MT * kTcXPad;  // halves per operand per buffer
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TV* xs = reinterpret_cast<TV*>(smem_raw);             // [2 buffers][hi, lo][MT][kTcXPad]
  uint4* cb1s = reinterpret_cast<uint4*>(xs + 4 * XB);  // [256] residual codebook (RES)

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int n = a.n, ng = n >> 3, chunks = n / kTcKC;
  const int64_t items = (int64_t)a.row_blocks * a.mtiles;
  const uint64_t pol_s = policy_evict_first();
  const uint64_t pol_c = policy_evict_last();
  const unsigned char* cb0 = static_cast<const unsigned char*>(a.cb0);
  const TV* gxh = static_cast<const TV*>(a.x);
  const TV* gxl = gxh + (int64_t)a.M * n;

  pdl_wait();
  if (RES) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) cb1s[i] = static_cast<const uint4*>(a.cb1)[i];
  }
  pdl_trigger();

  // copy activation chunk c of the M tile at m0 into buffer b (hi and lo), 16 bytes per cp.async
  auto stage = [&](int b, int m0, int mcount, int c) {
    TV* dh = xs + (2 * b) * XB;
    TV* dl = dh + XB;
    for (int q = threadIdx.x; q < MT * (kTcKC / 8); q += blockDim.x) {
      const int m = q / (kTcKC / 8), v = q - m * (kTcKC / 8);
      const bool ok = m < mcount;
      const int64_t so = ok ? (int64_t)(m0 + m) * n + (int64_t)c * kTcKC + v * 8 : 0;
      cp_async16(dh + m * kTcXPad + v * 8, gxh + so, ok);
      cp_async16(dl + m * kTcXPad + v * 8, gxl + so, ok);
    }
    cp_async_commit();
  };

  // Split-K launches (cluster of S CTAs per item) or persistent contiguous item ranges (S = 1).
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  int64_t i0, i1;
  if (S > 1) {
    i0 = (int64_t)blockIdx.x / S;
    i1 = min(items, i0 + 1);
  } else {
    const int64_t per = (items + gridDim.x - 1) / gridDim.x;
    i0 = (int64_t)blockIdx.x * per;
    i1 = min(items, i0 + per);
  }
  const int c0 = (int)((int64_t)rank * chunks / S), c1 = (int)((int64_t)(rank + 1) * chunks / S);
  for (int64_t it = i0; it < i1; ++it) {
    const int mt = (int)(it / a.row_blocks);
    const int rbg = (int)(it - (int64_t)mt * a.row_blocks);
    int p = 0;
#pragma unroll 1
    while (p + 1 < a.nprob && rbg >= a.p_rb0[p + 1]) ++p;
    const int rb = rbg - a.p_rb0[p];
    const int out = a.p_out[p];
    const int16_t* idx0 = a.p_idx0[p];
    const uint8_t* idx1 = a.p_idx1[p];
    const int row_w = rb * 128 + warp * 16;  // first row of this warp
    const int m0 = mt * MT;
    const int mcount = min(MT, a.M - m0);

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

    // this lane's index vector per chunk: row (lane >> 1), groups 8 * (lane & 1) .. +7
    const int lrow = row_w + (lane >> 1);
    const bool lrow_ok = lrow < out;
    auto load_iv = [&](int c, uint4& iv, uint2& jv) {
      iv = make_uint4(0, 0, 0, 0);
      jv = make_uint2(0, 0);
      if (lrow_ok && c < c1) {
        const int gbase = c * 16 + 8 * (lane & 1);
        iv = ld_stream_u4(idx0 + (int64_t)lrow * ng + gbase, pol_s);
        if (RES) jv = ld_stream_u2(idx1 + (int64_t)lrow * ng + gbase, pol_s);
      }
    };
    uint4 iv, niv;
    uint2 jv, njv;
    __syncthreads();  // readers of both buffers (previous item) are done
    stage(0, m0, mcount, c0);
    load_iv(c0, iv, jv);
    for (int c = c0; c < c1; ++c) {
      const int buf = (c - c0) & 1;
      if (c + 1 < c1) stage(buf ^ 1, m0, mcount, c + 1);
      else cp_async_commit();  // keep one group per iteration so wait_group<1> covers chunk c
      load_iv(c + 1, niv, njv);
      cp_async_wait<1>();      // chunk c has landed
      __syncthreads();
      const TV* xh = xs + (2 * buf) * XB;
      const TV* xl = xh + XB;
#pragma unroll
      for (int s = 0; s < 8; ++s) {  // 16 K per step: groups 2s and 2s+1 of the chunk
        // indices of (row gid, groups 2s, 2s+1) and (row gid+8, ...): lanes 2*row + (2s >= 8)
        const int word = s & 3;
        const uint32_t wlo = __shfl_sync(0xffffffffu, (&iv.x)[word], 2 * gid + (s >> 2));
        const uint32_t whi = __shfl_sync(0xffffffffu, (&iv.x)[word], 2 * (gid + 8) + (s >> 2));
        const uint32_t a0 = ld_cb_u32(cb0 + (size_t)(wlo & 0xffffu) * 16 + tig * 4, pol_c);
        const uint32_t a1 = ld_cb_u32(cb0 + (size_t)(whi & 0xffffu) * 16 + tig * 4, pol_c);
        const uint32_t a2 = ld_cb_u32(cb0 + (size_t)(wlo >> 16) * 16 + tig * 4, pol_c);
        const uint32_t a3 = ld_cb_u32(cb0 + (size_t)(whi >> 16) * 16 + tig * 4, pol_c);
        uint32_t r0 = 0, r1 = 0, r2 = 0, r3 = 0;
        if (RES) {
          const uint32_t bl = __shfl_sync(0xffffffffu, (&jv.x)[(s >> 1) & 1], 2 * gid + (s >> 2));
          const uint32_t bh = __shfl_sync(0xffffffffu, (&jv.x)[(s >> 1) & 1], 2 * (gid + 8) + (s >> 2));
          const int sh = (s & 1) * 16;  // byte pair (2s, 2s+1) within the 32-bit word
          const uint32_t* c1 = reinterpret_cast<const uint32_t*>(cb1s);
          r0 = c1[((bl >> sh) & 0xffu) * 4 + tig];
          r1 = c1[((bh >> sh) & 0xffu) * 4 + tig];
          r2 = c1[((bl >> (sh + 8)) & 0xffu) * 4 + tig];
          r3 = c1[((bh >> (sh + 8)) & 0xffu) * 4 + tig];
        }
        const int kk = s * 16 + tig * 2;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int xo = (j * 8 + gid) * kTcXPad + kk;
          const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(xh + xo);
          const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(xh + xo + 8);
          const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(xl + xo);
          const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(xl + xo + 8);
          Mma<TV>::run(acc[j], a0, a1, a2, a3, bh0, bh1);
          Mma<TV>::run(acc[j], a0, a1, a2, a3, bl0, bl1);
          if (RES) {
            Mma<TV>::run(acc[j], r0, r1, r2, r3, bh0, bh1);
            Mma<TV>::run(acc[j], r0, r1, r2, r3, bl0, bl1);
          }
        }
      }
      __syncthreads();  // this buffer is free for chunk c + 2
      iv = niv;
      jv = njv;
    }
    cp_async_wait<0>();

    if (S > 1) {  // split-K: partial sums through distributed shared memory, added in rank order
      float* part = reinterpret_cast<float*>(smem_raw);  // the activation buffers are free now
      __syncthreads();
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) part[(j * 4 + q) * 256 + threadIdx.x] = acc[j][q];
      cluster.sync();
      if (rank == 0) {
        for (int r = 1; r < S; ++r) {
          const float* rp = cluster.map_shared_rank(part, r);
#pragma unroll
          for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[j][q] += rp[(j * 4 + q) * 256 + threadIdx.x];
        }
      }
      cluster.sync();  // the other ranks keep their shared memory until rank 0 has read it
      if (rank != 0) continue;
    }

    // epilogue: acc[j] = D[rows gid, gid+8][tokens 8j + 2tig, +1]
    const TV* sc = static_cast<const TV*>(a.p_scale[p]);
    void* y = a.p_y[p];
    const int ra = row_w + gid, rb2 = row_w + gid + 8;
    const float sa = ra < out ? Mma<TV>::back(sc[ra]) * a.rs : 0.f;
    const float sb = rb2 < out ? Mma<TV>::back(sc[rb2]) * a.rs : 0.f;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = q < 2 ? ra : rb2;
        const int m = j * 8 + tig * 2 + (q & 1);
        if (row < out && m < mcount) {
          const float v = acc[j][q] * (q < 2 ? sa : sb);
          const int64_t o = (int64_t)(m0 + m) * a.y_row_stride + row;
          if (a.y_dtype == VQ2_F16) static_cast<__half*>(y)[o] = __float2half_rn(v);
          else if (a.y_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(v);
          else static_cast<float*>(y)[o] = v;
        }
      }
    }
  }
}

template <int NT, bool RES, typename TV>
static int launch_tc(GemvArgs a, cudaStream_t st) {
  constexpr int MT = 8 * NT;
  a.mtiles = (a.M + MT - 1) / MT;
  int rb = 0;
  for (int p = 0; p < a.nprob; ++p) {
    a.p_rb0[p] = rb;
    rb += (a.p_out[p] + 127) / 128;
  }
  a.p_rb0[a.nprob] = rb;
  a.row_blocks = rb;
  const int64_t items = (int64_t)rb * a.mtiles;
  const size_t smem = (size_t)4 * MT * kTcXPad * sizeof(TV) + (RES ? 256 * sizeof(uint4) : 0);
  auto kern = vq_gemm_tc_kernel<NT, RES, TV>;
  static std::atomic<uint64_t> done{0};
  static std::atomic<int> blocks_per_sm{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    int nb = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, 256, smem);
    blocks_per_sm.store(nb > 0 ? nb : 1);
    done.fetch_or(bit);
  }
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm.load();
  if (items <= 0) return VQ2_OK;
  // Split-K when the items fill less than half the GPU: the largest power of two S <= 8 with
  // items * S <= cap and at least two K chunks per CTA.
  const int chunks = a.n / kTcKC;
  int S = 1;
  while (S < 8 && items * (2 * S) <= cap && chunks >= 2 * (2 * S)) S *= 2;
  if (S == 1) {
    const int64_t grid = items < cap ? items : cap;
    return launch_kernel(kern, dim3((unsigned)grid), dim3(256), smem, st, a);
  }
  return launch_cluster(kern, dim3((unsigned)(items * S)), dim3(256), smem, S, st, a);
}

template <bool RES, typename TV>
static int launch_tc_nt(const GemvArgs& a, cudaStream_t st) {
  if (a.M <= 8) return launch_tc<1, RES, TV>(a, st);
  if (a.M <= 16) return launch_tc<2, RES, TV>(a, st);
  if (a.M <= 32) return launch_tc<4, RES, TV>(a, st);
  return launch_tc<8, RES, TV>(a, st);
}

template <typename TV>
static int run_split(const GemvArgs& a, void* ws, cudaStream_t st) {
  TV* xh = static_cast<TV*>(ws);
  const int64_t total = (int64_t)a.M * a.n;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  return launch_kernel(split_hilo_kernel<TV>, dim3((unsigned)blocks), dim3(256), 0, st, a.x, a.x_dtype,
                       (int64_t)a.M, (int64_t)a.n, a.x_row_stride, xh, xh + total);
}

int64_t gemm_tc_workspace(int64_t M, int64_t n) { return 2 * M * n * 2; }

int tc_operands(const GemvArgs& a, void* xh, void* xl, int val_dtype, cudaStream_t st) {
  if (!aligned(xh, 16) || (xl && !aligned(xl, 16))) return VQ2_ERR_ALIGN;
  if (a.x_mode != VQ2_ACT_ROTATED)
    return rht_split(a.x, a.x_dtype, a.x_mode, a.x_row_stride, a.M, a.n, a.hb, a.perm, a.sign, a.rot_scale, xh, xl,
                     val_dtype, st);
  const int64_t total = (int64_t)a.M * a.n;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  if (val_dtype == VQ2_F16)
    return launch_kernel(split_hilo_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, st, a.x, a.x_dtype,
                         (int64_t)a.M, (int64_t)a.n, a.x_row_stride, static_cast<__half*>(xh),
                         static_cast<__half*>(xl));
  if (val_dtype == VQ2_BF16)
    return launch_kernel(split_hilo_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, st, a.x,
                         a.x_dtype, (int64_t)a.M, (int64_t)a.n, a.x_row_stride, static_cast<__nv_bfloat16*>(xh),
                         static_cast<__nv_bfloat16*>(xl));
  return VQ2_ERR_DTYPE;
}

// Tensor-core path for multi-matrix problems with n % 128 == 0; `ws` holds
// gemm_tc_workspace(M, n) bytes for the split operand. Pre-rotated activations are split by
// split_hilo_kernel; modes RHT / SWIGLU_RHT are transformed and split in one launch
// (rht_split). Returns -1 when the problem is not eligible (the caller then uses the CUDA-core
// kernel).
int run_gemm_tc(const GemvArgs& a0, bool res, int val_dtype, void* ws, cudaStream_t st) {
  if (a0.nprob <= 0 || a0.n % kTcKC != 0 || ws == nullptr) return -1;
  if (!aligned(ws, 16)) return VQ2_ERR_ALIGN;
  GemvArgs a = a0;
  a.x = ws;
  a.x_row_stride = a.n;
  a.x_mode = VQ2_ACT_ROTATED;
  int s;
  if (a0.x_mode != VQ2_ACT_ROTATED) {
    const int64_t total = (int64_t)a0.M * a0.n;
    void* xl = static_cast<char*>(ws) + total * 2;
    if ((s = rht_split(a0.x, a0.x_dtype, a0.x_mode, a0.x_row_stride, a0.M, a0.n, a0.hb, a0.perm, a0.sign,
                       a0.rot_scale, ws, xl, val_dtype, st)) != VQ2_OK)
      return s;
    if (val_dtype == VQ2_F16) return res ? launch_tc_nt<true, __half>(a, st) : launch_tc_nt<false, __half>(a, st);
    if (val_dtype == VQ2_BF16)
      return res ? launch_tc_nt<true, __nv_bfloat16>(a, st) : launch_tc_nt<false, __nv_bfloat16>(a, st);
    return VQ2_ERR_DTYPE;
  }
  if (val_dtype == VQ2_F16) {
    if ((s = run_split<__half>(a0, ws, st)) != VQ2_OK) return s;
    return res ? launch_tc_nt<true, __half>(a, st) : launch_tc_nt<false, __half>(a, st);
  }
  if (val_dtype == VQ2_BF16) {
    if ((s = run_split<__nv_bfloat16>(a0, ws, st)) != VQ2_OK) return s;
    return res ? launch_tc_nt<true, __nv_bfloat16>(a, st) : launch_tc_nt<false, __nv_bfloat16>(a, st);
  }
  return VQ2_ERR_DTYPE;
}

}  // namespace vq2
