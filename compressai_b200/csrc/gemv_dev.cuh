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

// silu(g) = g * sigmoid(g). Fast division (reciprocal + multiply): the IEEE-exact divide is a
// multi-instruction sequence, and the staging of a SwiGLU row evaluates thousands of these.
// 1 + exp(-g) beyond 2^126 (g < -87) gives 0, the limit of g * sigmoid(g).
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.f + __expf(-g)); }

// Shared-memory ("fast") staging, used by the GEMV kernels: the rotation table is loaded into
// shared memory before the dependency wait (it is constant), the activation rows are read after
// it with independent coalesced loads (one memory round trip) into `raw`, and the permuted reads
// of the transform come from shared memory. When the transform is one pass (MT * n <= 2048:
// every raw value is read before the pass writes the tile) `raw` aliases the tile; otherwise it
// is a separate buffer of fast_raw_rows rows (all MT while MT + 1 rows fit kFastStageFloats,
// else one row per round). The old form (every permuted element read from global memory)
// remains for the shapes whose buffers do not fit and for the fused MoE kernel.
constexpr int kFastStageFloats = 12288;
// Dynamic shared memory of a GEMV CTA at most (the kernels' MaxDynamicSharedMemorySize): an
// activation tile of up to 80 KB, the transform scratch, the residual codebook and the fast
// staging buffers. Two CTAs of that size still share one SM.
constexpr int kGemvSmemCap = 112 * 1024;
__host__ __device__ constexpr bool stage_in_place(int mt, int n) { return mt * n <= 2048; }
__host__ __device__ constexpr int fast_raw_rows(int mt, int n) {
  return stage_in_place(mt, n) || (mt + 1) * n <= kFastStageFloats ? mt : 1;
}
__host__ __device__ constexpr int fast_extra_floats(int mt, int n) {
  return (stage_in_place(mt, n) ? 0 : fast_raw_rows(mt, n) * n) + (n + 1) / 2;  // raw rows + table
}
__host__ __device__ constexpr bool fast_stage(int mt, int n) {
  return n <= 32768 && (mt * xs_len(n) + kScratchFloats + 1024 + fast_extra_floats(mt, n)) * 4 <= kGemvSmemCap;
}
// Extra shared-memory floats of fast staging in mode `mode` (ROTATED needs none: it copies
// straight into the tile; the table has 16-bit entries).
__host__ __device__ constexpr int fast_stage_floats(int mt, int n, int mode) {
  return mode != VQ2_ACT_ROTATED && fast_stage(mt, n) ? fast_extra_floats(mt, n) : 0;
}

// Rotation table for fast staging: perm (< 2^15) with the sign in bit 15. All threads of the CTA
// call it; a barrier must follow before the table is read.
__device__ __forceinline__ void stage_perm(const ActSrc& a, uint16_t* ps) {
  if (a.x_mode == VQ2_ACT_ROTATED) return;
  const int n = a.n, nt = blockDim.x;
  if ((reinterpret_cast<uintptr_t>(a.perm) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.sign) & 3) == 0 &&
      n <= 8 * 4 * nt) {  // all loads issued before any store: one round trip
    const int4* p4 = reinterpret_cast<const int4*>(a.perm);
    const uint32_t* s4 = reinterpret_cast<const uint32_t*>(a.sign);
    int4 pv[8];
    uint32_t sv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int v = k * nt + threadIdx.x;
      if (4 * v < n) {
        pv[k] = p4[v];
        sv[k] = s4[v];
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int v = k * nt + threadIdx.x;
      if (4 * v < n) {
        const int4 q = pv[k];
        const uint32_t sg = sv[k];  // four int8 signs; bit 7 of a byte is set when negative
        const uint32_t lo = (q.x | (sg & 0x80u) << 8) | (q.y | (sg & 0x8000u)) << 16;
        const uint32_t hi = (q.z | (sg & 0x800000u) >> 8) | (q.w | (sg & 0x80000000u) >> 16) << 16;
        *reinterpret_cast<uint2*>(ps + 4 * v) = make_uint2(lo, hi);
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < n; i += nt) ps[i] = static_cast<uint16_t>(a.perm[i] | (a.sign[i] < 0 ? 0x8000 : 0));
}

constexpr int kLoadsInFlight = 2;  // 16-byte loads per thread per round (x2 for SwiGLU rows)

__device__ __forceinline__ int stage_pos(int j, bool padded) { return padded ? xs_pos(j >> 3, j & 7) : j; }

// Coalesced loads of `cnt` consecutive activations from element `off` of x into dst (padded
// tile positions or linear): value x[off + j], or silu(x[off + j]) * x[off + n + j] for SwiGLU
// rows (fp32 [gate | up]). All loads of a round are issued before its stores.
__device__ __forceinline__ void load_row(const ActSrc& a, int64_t off, int cnt, bool swiglu, float* dst,
                                         bool padded) {
  const int nt = blockDim.x;
  const bool f32 = swiglu || a.x_dtype == VQ2_F32;
  const uintptr_t addr = f32 ? reinterpret_cast<uintptr_t>(static_cast<const float*>(a.x) + off)
                             : reinterpret_cast<uintptr_t>(static_cast<const __half*>(a.x) + off);
  const bool vec = (addr & 15) == 0 && (!swiglu || (a.n & 3) == 0);
  if (vec && f32) {
    const float4* g = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + off);
    const int nv = cnt >> 2;
    for (int v0 = 0; v0 < nv; v0 += nt * kLoadsInFlight) {
      float4 gv[kLoadsInFlight], uv[kLoadsInFlight];
#pragma unroll
      for (int k = 0; k < kLoadsInFlight; ++k) {
        const int v = v0 + k * nt + threadIdx.x;
        if (v < nv) {
          gv[k] = g[v];
          if (swiglu) uv[k] = g[v + (a.n >> 2)];
        }
      }
#pragma unroll
      for (int k = 0; k < kLoadsInFlight; ++k) {
        const int v = v0 + k * nt + threadIdx.x;
        if (v < nv) {
          float4 r = gv[k];
          if (swiglu) {
            r.x = silu_f(r.x) * uv[k].x; r.y = silu_f(r.y) * uv[k].y;
            r.z = silu_f(r.z) * uv[k].z; r.w = silu_f(r.w) * uv[k].w;
          }
          *reinterpret_cast<float4*>(dst + stage_pos(4 * v, padded)) = r;
        }
      }
    }
    return;
  }
  if (vec) {  // 16-bit: 8 values per 16-byte load
    const uint4* g = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.x) + off);
    const int nv = cnt >> 3;
    for (int v0 = 0; v0 < nv; v0 += nt * kLoadsInFlight) {
      uint4 w[kLoadsInFlight];
#pragma unroll
      for (int k = 0; k < kLoadsInFlight; ++k) {
        const int v = v0 + k * nt + threadIdx.x;
        if (v < nv) w[k] = g[v];
      }
#pragma unroll
      for (int k = 0; k < kLoadsInFlight; ++k) {
        const int v = v0 + k * nt + threadIdx.x;
        if (v < nv) {
          float f[8];
          if (a.x_dtype == VQ2_F16) decode8<__half>(w[k], f);
          else decode8<__nv_bfloat16>(w[k], f);
          float* d = dst + stage_pos(8 * v, padded);
          *reinterpret_cast<float4*>(d) = make_float4(f[0], f[1], f[2], f[3]);
          *reinterpret_cast<float4*>(d + 4) = make_float4(f[4], f[5], f[6], f[7]);
        }
      }
    }
    return;
  }
  for (int j0 = 0; j0 < cnt; j0 += nt * 8) {  // unaligned rows: scalar loads, 8 in flight
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = j0 + k * nt + threadIdx.x;
      v[k] = 0.f;
      if (j < cnt) {
        if (swiglu) {
          const float* g = static_cast<const float*>(a.x) + off;
          v[k] = silu_f(g[j]) * g[a.n + j];
        } else {
          v[k] = load_act(a.x, a.x_dtype, off + j);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = j0 + k * nt + threadIdx.x;
      if (j < cnt) dst[stage_pos(j, padded)] = v[k];
    }
  }
}

// Stage MT activation rows (starting at element offset xoff) into the padded fp32 tile xs.
// Mode ROTATED copies; modes RHT / SWIGLU_RHT apply the forward randomized Hadamard transform
// (perm gather, sign, blocked Sylvester Hadamard, rot_scale) with the whole CTA: a segment of
// hb elements belongs to T = hb/8 threads (8 values each): 3 butterfly stages in registers,
// one transpose through `scratch`, 3 more in registers, the rest with warp shuffles (the same
// scheme as the standalone vq2_rht kernel). With `raw` the rows are staged the fast way
// (fast_stage above; `ps` is the table from stage_perm). Must be called by all 256 threads.
template <int MT>
__device__ __forceinline__ void stage_activations(const ActSrc& a, int64_t xoff, int mcount, float* xs, int xl,
                                                  float* scratch, float* raw = nullptr,
                                                  const uint16_t* ps = nullptr) {
  const int n = a.n;
  const bool swiglu = (a.x_mode == VQ2_ACT_SWIGLU_RHT), rotated = (a.x_mode == VQ2_ACT_ROTATED);
  if constexpr (MT > 1) {  // one raw row per round: stage each row as its own one-row tile
    if (raw != nullptr && !rotated && fast_raw_rows(MT, n) == 1) {
#pragma unroll 1
      for (int mi = 0; mi < MT; ++mi)
        stage_activations<1>(a, xoff + (int64_t)mi * a.x_row_stride, mi < mcount ? 1 : 0, xs + mi * xl, xl,
                             scratch, raw, ps);
      return;
    }
  }
  if (raw != nullptr) {
#pragma unroll 1
    for (int mi = 0; mi < MT; ++mi) {
      if (mi < mcount) {
        load_row(a, xoff + (int64_t)mi * a.x_row_stride, n, swiglu, rotated ? xs + mi * xl : raw + mi * n, rotated);
      } else if (rotated) {  // the transform reads no rows past mcount
        for (int j = threadIdx.x; j < n; j += blockDim.x) xs[mi * xl + stage_pos(j, true)] = 0.f;
      }
    }
    if (rotated) return;
    __syncthreads();
  } else if (rotated) {
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
  float* sc = scratch + s * (hb + (hb >> 5));
  for (int s0 = 0; s0 < segs; s0 += SEG) {
    const int gs = s0 + s;
    const int mi = gs / nb, b = gs - mi * nb;
    const bool active = gs < segs && mi < mcount;
    float v[8];
    if (raw != nullptr) {  // uniform branch, outside the unrolled loads
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t q = ps[b * hb + t + T * i];
        const float r = active ? raw[mi * n + (q & 0x7fffu)] : 0.f;
        v[i] = (q & 0x8000u) ? -r : r;
      }
    } else {
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
