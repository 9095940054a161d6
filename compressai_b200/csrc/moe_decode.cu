// A batch-1 MoE layer (one token: the decode step) in two launches instead of the router kernel
// + gate_up GEMV + down GEMV of the general path.
//
//   1. moe_t1_gate_up_kernel: EVERY CTA routes the token itself -- top-k of the E <= 256 logits
//      (per-warp ranks by shuffles, then one rank pass over the 8 x k candidates), the local pool
//      rows, the compacted problem list -- stages the forward RHT of the hidden row, and computes
//      its contiguous share of the P x 1024 gate_up rows (fp32, into the workspace).
//   2. moe_t1_down_kernel: routes again, BEFORE its dependency wait (the logits and the hidden
//      row are at least two kernels old when it starts: the gate_up kernel between lets it start
//      only after its own wait), computes the routing weights and the shared expert's sigmoid
//      gate, loads its rows' index vectors; after the wait it stages SwiGLU + RHT 512 of every
//      problem's gate_up row, and each warp computes one output row over ALL problems and sums
//      them with the routing weights in problem order -- the combine needs no second pass and no
//      cross-CTA counters. The output is the layer's hidden row, or (expert parallelism) this
//      rank's fp32 partial, which the peer combine kernel sums over the ranks.
//
// Why: a single token's routing on one 1024-thread CTA (the general router) costs ~6 us of
// serial work on one SM while the other 147 wait (rank counting ~2.3 us, the RHT of the hidden
// row on a quarter of the CTA ~2 us), and its results then cost the GEMVs another dependent
// load chain. Recomputing the routing per CTA is ~0.3 us, in parallel.
//
// The arithmetic is that of the general path (router kernel: key order, weights, shared gate;
// GEMV: staging, FMA order, shuffle order, scale; fused combine: fmaf chain in problem order),
// so outputs are bit-identical to it (VQ2_MOE_T1=0 selects the general path).
//
// Reference: PagedMoEExpert.forward (vq2/paged_runtime.py:439-511) with the router of the
// installed transformers Qwen3_5MoeTopKRouter (softmax -> top-k -> renormalise; the weights here
// are exp(l - l_max) / sum over the selected, which equals it) and the shared expert of
// Qwen3_5MoeSparseMoeBlock; kernels vq2/kernels.py:117-176 (_parallel_moe_gate_up / _down).
//
// Shapes: hidden 2048 (RHT block 2048), expert intermediate 512 (RHT block 512), top-k <= 8,
// E <= 256, 2 bpw, fp16/bf16 codebook; run_moe_t1 returns -1 for anything else.
#include <cfloat>
#include <cstdlib>
#include <cstring>

#include "gemv_dev.cuh"

namespace vq2 {

constexpr int kT1H = 2048;            // hidden size
constexpr int kT1I = 512;             // expert intermediate size
constexpr int kT1GuRows = 2 * kT1I;   // gate | up rows of an expert
constexpr int kT1MaxK = 8;
constexpr int kT1MaxP = kT1MaxK + 1;  // + the shared expert
constexpr int kT1MaxE = 256;

struct MoeT1Args {
  const void* h;            // [H] the token's hidden row
  int h_dtype;
  const float* logits;      // [E]
  int E, K;
  const float* gate;        // shared-expert gate [H] fp32, or null (no shared expert)
  int lo, hi, rank, world, shared_row;
  const uint8_t* pool;      // expert records [pool_rows, rec]
  int64_t pool_rows, rec, off_gu_idx, off_gu_scale, off_dn_idx, off_dn_scale;
  const void* cb0;
  const int32_t* perm_in;   // RHT 2048
  const int8_t* sign_in;
  float scale_in;
  const int32_t* perm_mid;  // RHT 512
  const int8_t* sign_mid;
  float scale_mid;
  float* gu;                // [K + 1, 1024] fp32 gate_up rows by original problem index
  void* out;                // [H] out_dtype
  int out_dtype;
  // paged mode (ids_in != null): the token's experts, weights and pool slots come from the device
  // LRU step, and a record missed in this step is read from the pinned host image by the kernels
  // that use it, which write it into its slot on the way (gate_up rows by launch 1, down rows by
  // launch 2: together the whole record)
  const int32_t* ids_in;    // [K] expert ids of the layer (image offsets)
  const int32_t* slots;     // [K] pool slots, -1: skipped
  const int32_t* miss;      // LRU miss list {count, expert[K], slot[K]}
  const float* w_in;        // [K] routing weights
  const uint8_t* image;     // device address of the page-locked image
  const int64_t* rec_off;   // [num_experts] record offsets in the image
  int64_t num_experts;
};

// The routing of one token as every CTA computes it.
struct T1Route {
  unsigned long long cand[8 * kT1MaxK];  // each warp's top-k keys
  float lg[kT1MaxE];
  int sel_e[kT1MaxK];
  float sel_v[kT1MaxK];
  int pid[kT1MaxP];   // pool row of compacted problem c
  int pmap[kT1MaxP];  // its original problem index (0..K-1 routed, K shared)
  const uint8_t* src[kT1MaxP];  // record to read: the pool row, or (paged miss) the image's copy
  uint8_t* dst[kT1MaxP];        // paged miss: the pool slot the record is written to; else null
  int P;
};

// Top-k, local pool rows and the compacted problem list of the token (router kernel semantics:
// ids in rank order; routed expert e -> pool row e - lo when lo <= e < hi; the shared expert's
// problem on rank 0 of the group, as the token index is 0). All 256 threads; ends with a barrier.
__device__ __forceinline__ void t1_route(const MoeT1Args& a, T1Route& s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float v = tid < a.E ? __ldcg(a.logits + tid) : 0.f;
  const unsigned long long key = tid < a.E ? route_key(v, tid) : 0ull;
  if (tid < a.E) s.lg[tid] = v;
  if (lane < a.K) s.cand[warp * a.K + lane] = 0ull;
  int cnt = 0;
#pragma unroll
  for (int m = 0; m < 32; ++m) cnt += __shfl_sync(0xffffffffu, key, m) > key ? 1 : 0;
  __syncwarp();
  if (cnt < a.K) s.cand[warp * a.K + cnt] = key;  // lanes past E share one zero key's slot
  __syncthreads();
  const int nc = 8 * a.K;
  if (tid < nc) {
    const unsigned long long k = s.cand[tid];
    int r = 0;
    for (int d = 0; d < nc; ++d) r += s.cand[d] > k ? 1 : 0;
    if (r < a.K && k != 0ull) {
      const int e = static_cast<int>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffull));
      s.sel_e[r] = e;
      s.sel_v[r] = s.lg[e];
    }
  }
  __syncthreads();
  if (tid == 0) {
    int P = 0;
    const int ks = a.K + (a.gate ? 1 : 0);
    for (int j = 0; j < ks; ++j) {
      int id;
      if (j < a.K) {
        const int e = s.sel_e[j];
        id = (e >= a.lo && e < a.hi) ? e - a.lo : -1;
      } else {
        id = (a.rank == 0) ? a.shared_row : -1;  // token 0 % world
      }
      if (id >= 0 && id < a.pool_rows) {
        s.pid[P] = id;
        s.pmap[P] = j;
        s.src[P] = a.pool + id * a.rec;
        s.dst[P] = nullptr;
        ++P;
      }
    }
    s.P = P;
  }
  __syncthreads();
}

// Paged mode: the problem list from the LRU step's slots (in k order, skipping -1), the record
// of a slot on the step's miss list read from the image. All 256 threads; ends with a barrier.
__device__ __forceinline__ void t1_problems_paged(const MoeT1Args& a, T1Route& s) {
  if (threadIdx.x == 0) {
    const int nm = min(max(__ldcg(a.miss), 0), a.K);
    int P = 0;
    for (int j = 0; j < a.K; ++j) {
      const int sl = __ldcg(a.slots + j), e = __ldcg(a.ids_in + j);
      if (sl < 0 || sl >= a.pool_rows || e < 0 || e >= a.num_experts) continue;
      bool missed = false;
      for (int m = 0; m < nm; ++m) missed |= __ldcg(a.miss + 1 + a.K + m) == sl;
      uint8_t* slot = const_cast<uint8_t*>(a.pool) + sl * a.rec;
      s.pid[P] = sl;
      s.pmap[P] = j;
      s.src[P] = missed ? a.image + __ldcg(a.rec_off + e) : slot;
      s.dst[P] = missed ? slot : nullptr;
      ++P;
    }
    s.P = P;
  }
  __syncthreads();
}

// 16 bytes of a record: from the pool (streaming load), or from the host image (plain load),
// then written into the slot.
__device__ __forceinline__ uint4 t1_rec_u4(const uint8_t* src, uint8_t* dst, int64_t off, uint64_t pol) {
  if (dst == nullptr) return ld_stream_u4(src + off, pol);
  const uint4 v = *reinterpret_cast<const uint4*>(src + off);
  *reinterpret_cast<uint4*>(dst + off) = v;
  return v;
}
template <typename TV>
__device__ __forceinline__ float t1_rec_scale(const uint8_t* src, uint8_t* dst, int64_t off, bool store) {
  const TV v = *reinterpret_cast<const TV*>(src + off);
  if (dst != nullptr && store) *reinterpret_cast<TV*>(dst + off) = v;
  return to_f32<TV>(v);
}

// Forward RHT (blocks of HB = the row length) of `rows` rows of the tile in place: raw values at
// linear positions of row mi (stride xl) in, transformed values at the padded positions out. The
// transform of stage_activations: HB / 8 threads per row, 8 values each, 3 butterfly stages in
// registers, a transpose through the scratch, 3 more, then shuffle stages; 256 / (HB / 8) rows
// per round. A row's raw values are all read before the round's first barrier and its outputs
// written after it. All 256 threads; ends with a barrier.
template <int HB>
__device__ __forceinline__ void t1_rht_rows(float* xs, int xl, int rows, const uint16_t* ps, float* scratch,
                                            float rot_scale) {
  constexpr int TT = HB / 8, SEGR = 256 / TT;
  const int s = threadIdx.x / TT, t = threadIdx.x % TT;
  float* scs = scratch + s * (HB + (HB >> 5));
  for (int s0 = 0; s0 < rows; s0 += SEGR) {
    const int mi = s0 + s;
    const bool active = mi < rows;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t q = ps[t + TT * i];
      const float x = active ? xs[mi * xl + (q & 0x7fffu)] : 0.f;
      v[i] = (q & 0x8000u) ? -x : x;
    }
    fwht8(v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = t + TT * i;
      scs[e + (e >> 5)] = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = 8 * t + i;
      v[i] = scs[e + (e >> 5)];
    }
    fwht8(v);
    for (int td = 1; td <= (TT >> 4); td <<= 1) {
      const bool upper = (t & td) != 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float o = __shfl_xor_sync(0xffffffffu, v[i], td);
        v[i] = upper ? (o - v[i]) : (v[i] + o);
      }
    }
    if (active) {
      float* o = xs + mi * xl + xs_pos(t, 0);
      *reinterpret_cast<float4*>(o) = make_float4(v[0] * rot_scale, v[1] * rot_scale, v[2] * rot_scale,
                                                  v[3] * rot_scale);
      *reinterpret_cast<float4*>(o + 4) = make_float4(v[4] * rot_scale, v[5] * rot_scale, v[6] * rot_scale,
                                                      v[7] * rot_scale);
    }
    __syncthreads();
  }
}

// 8 activations from 16 (fp16 / bf16) or 32 (fp32) bytes.
__device__ __forceinline__ void t1_load8(const void* p, int dtype, int64_t off, float (&f)[8]) {
  if (dtype == VQ2_F32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else if (dtype == VQ2_F16) {
    decode8<__half>(*reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + off), f);
  } else {
    decode8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + off), f);
  }
}

constexpr int kT1GuSmemFloats = 2176 + kScratchFloats + kT1H / 2;  // tile, scratch, 16-bit table
constexpr int kT1DnXl = 544;                                          // xs_len(512)
constexpr int kT1DnSmemFloats = kT1MaxP * kT1DnXl + kScratchFloats + kT1I / 2;

// ---- launch 1: routing + gate_up rows ------------------------------------------------------
template <typename TV>
__global__ void __launch_bounds__(256, 2) moe_t1_gate_up_kernel(const MoeT1Args a) {
  extern __shared__ __align__(16) float smem[];
  constexpr int xl = xs_len(kT1H);
  static_assert(xl == 2176, "tile layout");
  float* xs = smem;
  float* scratch = smem + xl;
  uint16_t* ps = reinterpret_cast<uint16_t*>(scratch + kScratchFloats);
  __shared__ T1Route rt;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint64_t pol_s = policy_evict_first();
  const uint64_t pol_c = policy_evict_last();
  {  // rotation table (constant)
    ActSrc src{};
    src.x_mode = VQ2_ACT_RHT; src.n = kT1H; src.hb = kT1H; src.perm = a.perm_in; src.sign = a.sign_in;
    stage_perm(src, ps);
  }
  pdl_wait();
  pdl_trigger();
  float hv[8];
  t1_load8(a.h, a.h_dtype, 8 * tid, hv);  // in flight with the logits of the routing
  if (a.ids_in) t1_problems_paged(a, rt);
  else t1_route(a, rt);
  const int P = rt.P;
  const int64_t R = (int64_t)P * kT1GuRows;
  const int64_t lo = blockIdx.x * R / gridDim.x, hi = (blockIdx.x + 1) * R / gridDim.x;
  const int npairs = (int)((hi - lo + 1) / 2);
  // index vectors of one pair of rows (rows past hi read nothing)
  auto load_pair = [&](int q, uint4 (&iv)[2], float (&sv)[2]) {
#pragma unroll
    for (int rw = 0; rw < 2; ++rw) {
      const int64_t g = lo + 2 * q + rw;
      iv[rw] = make_uint4(0, 0, 0, 0);
      sv[rw] = 0.f;
      if (q < npairs && g < hi) {
        const int c = (int)(g / kT1GuRows), r = (int)(g % kT1GuRows);
        iv[rw] = t1_rec_u4(rt.src[c], rt.dst[c], a.off_gu_idx + ((int64_t)r * (kT1H / 8) + lane * 8) * 2, pol_s);
        if (lane == 0) sv[rw] = t1_rec_scale<TV>(rt.src[c], rt.dst[c], a.off_gu_scale + 2 * r, true);
      }
    }
  };
  uint4 iv[2];
  float sv[2];
  int q = warp;
  load_pair(q, iv, sv);  // HBM round trip under the transform
#pragma unroll
  for (int k = 0; k < 8; ++k) xs[8 * tid + k] = hv[k];
  __syncthreads();
  t1_rht_rows<kT1H>(xs, xl, 1, ps, scratch, a.scale_in);
  float xreg[64];
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // this lane's 8 groups (conflict-free: lanes 68 floats apart)
    const float4 l4 = *reinterpret_cast<const float4*>(xs + xs_pos(lane * 8 + j, 0));
    const float4 h4 = *reinterpret_cast<const float4*>(xs + xs_pos(lane * 8 + j, 4));
    xreg[j * 8 + 0] = l4.x; xreg[j * 8 + 1] = l4.y; xreg[j * 8 + 2] = l4.z; xreg[j * 8 + 3] = l4.w;
    xreg[j * 8 + 4] = h4.x; xreg[j * 8 + 5] = h4.y; xreg[j * 8 + 6] = h4.z; xreg[j * 8 + 7] = h4.w;
  }
  const uint4* cb0 = static_cast<const uint4*>(a.cb0);
  for (; q < npairs; q += 8) {
    uint4 nv[2];
    float nsv[2];
    load_pair(q + 8, nv, nsv);
    float acc[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int rw = 0; rw < 2; ++rw) {
        const uint32_t w32 = (&iv[rw].x)[j >> 1];
        const uint32_t code = (j & 1) ? (w32 >> 16) : (w32 & 0xffffu);
        float wv[8];
        decode8<TV>(ld_cb_u4(cb0 + code, pol_c), wv);
        float s = acc[rw];
#pragma unroll
        for (int t = 0; t < 8; ++t) s = fmaf(wv[t], xreg[j * 8 + t], s);
        acc[rw] = s;
      }
    }
#pragma unroll
    for (int rw = 0; rw < 2; ++rw)
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[rw] += __shfl_xor_sync(0xffffffffu, acc[rw], off);
    if (lane == 0) {
#pragma unroll
      for (int rw = 0; rw < 2; ++rw) {
        const int64_t g = lo + 2 * q + rw;
        if (g < hi) {
          const int c = (int)(g / kT1GuRows), r = (int)(g % kT1GuRows);
          a.gu[(int64_t)rt.pmap[c] * kT1GuRows + r] = acc[rw] * sv[rw];
        }
      }
    }
#pragma unroll
    for (int rw = 0; rw < 2; ++rw) {
      iv[rw] = nv[rw];
      sv[rw] = nsv[rw];
    }
  }
}

// ---- launch 2: routing weights + down rows over all problems + combine -----------------------
template <typename TV>
__global__ void __launch_bounds__(256, 2) moe_t1_down_kernel(const MoeT1Args a) {
  extern __shared__ __align__(16) float smem[];
  constexpr int xl = kT1DnXl;
  static_assert(xl == xs_len(kT1I), "tile layout");
  float* xs = smem;                                  // [P][544]: raw SwiGLU rows, then transformed
  float* scratch = smem + kT1MaxP * xl;
  uint16_t* ps = reinterpret_cast<uint16_t*>(scratch + kScratchFloats);
  __shared__ T1Route rt;
  __shared__ float s_wj[kT1MaxP];        // weight of original problem j
  __shared__ float s_w[kT1MaxP];         // weight of compacted problem c
  __shared__ float s_red[32];
  __shared__ float s_y[8][kT1MaxP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int li = lane & 7, sub = lane >> 3;
  const uint64_t pol_s = policy_evict_first();
  const uint64_t pol_c = policy_evict_last();
  // ---- before the dependency wait: everything that depends only on the layer's inputs
  {
    ActSrc src{};
    src.x_mode = VQ2_ACT_SWIGLU_RHT; src.n = kT1I; src.hb = kT1I; src.perm = a.perm_mid; src.sign = a.sign_mid;
    stage_perm(src, ps);
  }
  float d = 0.f;  // shared-expert gate: this thread's 8 terms, summed as the router kernel does
  if (a.gate) {
    float hv[8], gv[8];
    t1_load8(a.h, a.h_dtype, 8 * tid, hv);
    t1_load8(a.gate, VQ2_F32, 8 * tid, gv);
#pragma unroll
    for (int k = 0; k < 8; ++k) d = fmaf(hv[k], gv[k], d);
  }
  if (a.ids_in) t1_problems_paged(a, rt);
  else t1_route(a, rt);
  const int P = rt.P;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
  if (lane == 0) s_red[warp] = d;
  if (a.ids_in) {
    if (tid < a.K) s_wj[tid] = __ldcg(a.w_in + tid);
  } else if (tid < a.K) {
    const float mx = rt.sel_v[0];
    float sum = 0.f;
    for (int k = 0; k < a.K; ++k) sum += expf(rt.sel_v[k] - mx);
    s_wj[tid] = expf(rt.sel_v[tid] - mx) / sum;
  }
  __syncthreads();
  if (a.gate && warp == 1) {  // the 32 warp sums (8 warps of data, zeros for the rest)
    float dd = lane < 8 ? s_red[lane] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, off);
    if (lane == 0) s_wj[a.K] = 1.f / (1.f + expf(-dd));
  }
  __syncthreads();
  if (tid < P) s_w[tid] = s_wj[rt.pmap[tid]];
  // this CTA's rows, one per warp; lanes (sub, li): problem slots sub + 4q, groups li*8 .. +7
  const int r0 = (int)((int64_t)blockIdx.x * kT1H / gridDim.x), r1 = (int)((int64_t)(blockIdx.x + 1) * kT1H / gridDim.x);
  const int r = r0 + warp;
  const bool row_ok = r < r1;
  uint4 iv[3];
  float sc[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int p = sub + 4 * q;
    iv[q] = make_uint4(0, 0, 0, 0);
    sc[q] = 0.f;
    if (row_ok && p < P) {
      iv[q] = t1_rec_u4(rt.src[p], rt.dst[p], a.off_dn_idx + ((int64_t)r * (kT1I / 8) + li * 8) * 2, pol_s);
      sc[q] = t1_rec_scale<TV>(rt.src[p], rt.dst[p], a.off_dn_scale + 2 * r, li == 0);
    }
  }
  pdl_wait();
  pdl_trigger();
  // ---- SwiGLU of every problem's gate_up row (one round of loads) into the tile rows, linear
  {
    constexpr int nv = kT1I / 4;
    float4 gv[5], uv[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const int v = k * 256 + tid, p = v / nv, c = v % nv;
      if (p < P) {
        const float4* g = reinterpret_cast<const float4*>(a.gu + (int64_t)rt.pmap[p] * kT1GuRows);
        gv[k] = g[c];
        uv[k] = g[c + nv];
      }
    }
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const int v = k * 256 + tid, p = v / nv, c = v % nv;
      if (p < P) {
        float4 o = gv[k];
        o.x = silu_f(o.x) * uv[k].x; o.y = silu_f(o.y) * uv[k].y;
        o.z = silu_f(o.z) * uv[k].z; o.w = silu_f(o.w) * uv[k].w;
        *reinterpret_cast<float4*>(xs + p * xl + 4 * c) = o;
      }
    }
  }
  __syncthreads();
  t1_rht_rows<kT1I>(xs, xl, P, ps, scratch, a.scale_mid);
  // ---- this warp's row over the problems: 8 gathers per lane per slot, then the dot products
  const uint4* cb0 = static_cast<const uint4*>(a.cb0);
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int p = sub + 4 * q;
    float acc = 0.f;
    if (row_ok && p < P) {
      const float* xrow = xs + p * xl;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t w32 = (&iv[q].x)[j >> 1];
        const uint32_t code = (j & 1) ? (w32 >> 16) : (w32 & 0xffffu);
        float wv[8];
        decode8<TV>(ld_cb_u4(cb0 + code, pol_c), wv);
        const int pos = xs_pos(li * 8 + j, 0);
        const float4 l4 = *reinterpret_cast<const float4*>(xrow + pos);
        const float4 h4 = *reinterpret_cast<const float4*>(xrow + pos + 4);
        const float xv[8] = {l4.x, l4.y, l4.z, l4.w, h4.x, h4.y, h4.z, h4.w};
#pragma unroll
        for (int t = 0; t < 8; ++t) acc = fmaf(wv[t], xv[t], acc);
      }
    }
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (li == 0 && p < P) s_y[warp][p] = acc * sc[q];
  }
  __syncwarp();
  if (lane == 0 && row_ok) {  // routing-weighted sum in problem order
    float s = 0.f;
    for (int c = 0; c < P; ++c) s = fmaf(s_w[c], s_y[warp][c], s);
    if (a.out_dtype == VQ2_F16) static_cast<__half*>(a.out)[r] = __float2half_rn(s);
    else if (a.out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(a.out)[r] = __float2bfloat16_rn(s);
    else static_cast<float*>(a.out)[r] = s;
  }
}

bool moe_t1_enabled() {
  const char* v = std::getenv("VQ2_MOE_T1");  // A/B switch, read per call
  return !(v && std::strcmp(v, "0") == 0);
}

template <typename TV>
static int launch_t1(const MoeT1Args& a, cudaStream_t st) {
  auto k1 = moe_t1_gate_up_kernel<TV>;
  auto k2 = moe_t1_down_kernel<TV>;
  const int s1 = kT1GuSmemFloats * 4, s2 = kT1DnSmemFloats * 4;
  static int done[64] = {};  // per device: carveouts that leave most of the SM's memory as L1
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev & 63]) {
    const int pct1 = (2 * (s1 + 4096) * 100 + 228 * 1024 - 1) / (228 * 1024);
    const int pct2 = (2 * (s2 + 4096) * 100 + 228 * 1024 - 1) / (228 * 1024);
    cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributePreferredSharedMemoryCarveout, pct1);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k2, cudaFuncAttributePreferredSharedMemoryCarveout, pct2);
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    done[dev & 63] = 1;
  }
  const dim3 grid((unsigned)(2 * sm_count()));
  int s = launch_kernel(k1, grid, dim3(256), (size_t)s1, st, a);
  if (s != VQ2_OK) return s;
  return launch_kernel(k2, grid, dim3(256), (size_t)s2, st, a);
}

// Shape checks shared by both modes: -1 when the layer is not the specialisation's.
static int t1_shapes_ok(int64_t K, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, int64_t hb_in,
                        int64_t hb_mid, int val_dtype) {
  if (K <= 0 || K > kT1MaxK) return -1;
  if (gu_cols * 8 != kT1H || gu_rows != kT1GuRows || dn_rows != kT1H || dn_cols * 8 != kT1I) return -1;
  if (hb_in != kT1H || hb_mid != kT1I) return -1;
  if (val_dtype != VQ2_F16 && val_dtype != VQ2_BF16) return -1;
  return 0;
}

int run_moe_t1(const void* h, int h_dtype, const float* logits, int64_t E, int64_t K, const float* shared_gate,
               int64_t lo, int64_t hi, int rank, int world, const void* pool, int64_t pool_rows, int64_t gu_rows,
               int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
               const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in, const int32_t* perm_mid,
               const int8_t* sign_mid, int64_t hb_mid, float scale_mid, int64_t rec, int64_t off_gu_idx,
               int64_t off_gu_scale, int64_t off_dn_idx, int64_t off_dn_scale, float* gu, void* out, int out_dtype,
               cudaStream_t st) {
  if (!moe_t1_enabled()) return -1;
  if (E <= 0 || E > kT1MaxE || K > E) return -1;
  if (t1_shapes_ok(K, gu_rows, gu_cols, dn_rows, dn_cols, hb_in, hb_mid, val_dtype) != 0) return -1;
  if (!aligned(h, 16) || !aligned(gu, 16) || (shared_gate && !aligned(shared_gate, 16)) || !aligned(perm_in, 16) ||
      !aligned(sign_in, 4) || !aligned(perm_mid, 16) || !aligned(sign_mid, 4))
    return -1;
  MoeT1Args a{};
  a.h = h; a.h_dtype = h_dtype; a.logits = logits; a.E = (int)E; a.K = (int)K; a.gate = shared_gate;
  a.lo = (int)lo; a.hi = (int)hi; a.rank = rank; a.world = world; a.shared_row = (int)(hi - lo);
  a.pool = static_cast<const uint8_t*>(pool); a.pool_rows = pool_rows; a.rec = rec;
  a.off_gu_idx = off_gu_idx; a.off_gu_scale = off_gu_scale; a.off_dn_idx = off_dn_idx; a.off_dn_scale = off_dn_scale;
  a.cb0 = cb0; a.perm_in = perm_in; a.sign_in = sign_in; a.scale_in = scale_in;
  a.perm_mid = perm_mid; a.sign_mid = sign_mid; a.scale_mid = scale_mid;
  a.gu = gu; a.out = out; a.out_dtype = out_dtype;
  return val_dtype == VQ2_F16 ? launch_t1<__half>(a, st) : launch_t1<__nv_bfloat16>(a, st);
}

// Paged mode (vq2_paged_moe_t1): the same two launches on the LRU step's slots.
int run_moe_t1_paged(const void* h, int h_dtype, int64_t K, const int32_t* ids, const int32_t* slots,
                     const int32_t* miss, const float* w, const void* pool, int64_t capacity, int64_t gu_rows,
                     int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
                     const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in,
                     const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid, float scale_mid,
                     const void* image, const int64_t* rec_off, int64_t num_experts, float* gu, void* out,
                     int out_dtype, cudaStream_t st) {
  if (t1_shapes_ok(K, gu_rows, gu_cols, dn_rows, dn_cols, hb_in, hb_mid, val_dtype) != 0) return VQ2_ERR_SHAPE;
  if (!aligned(h, 16) || !aligned(gu, 16) || !aligned(pool, 16) || !aligned(image, 16) || !aligned(cb0, 16) ||
      !aligned(perm_in, 16) || !aligned(sign_in, 4) || !aligned(perm_mid, 16) || !aligned(sign_mid, 4))
    return VQ2_ERR_ALIGN;
  MoeT1Args a{};
  a.h = h; a.h_dtype = h_dtype; a.K = (int)K; a.E = 0; a.gate = nullptr;
  a.pool = static_cast<const uint8_t*>(pool); a.pool_rows = capacity;
  a.rec = 2 * gu_rows * gu_cols + 2 * gu_rows + 2 * dn_rows * dn_cols + 2 * dn_rows;
  a.off_gu_idx = 0; a.off_gu_scale = 2 * gu_rows * gu_cols; a.off_dn_idx = a.off_gu_scale + 2 * gu_rows;
  a.off_dn_scale = a.off_dn_idx + 2 * dn_rows * dn_cols;
  a.cb0 = cb0; a.perm_in = perm_in; a.sign_in = sign_in; a.scale_in = scale_in;
  a.perm_mid = perm_mid; a.sign_mid = sign_mid; a.scale_mid = scale_mid;
  a.gu = gu; a.out = out; a.out_dtype = out_dtype;
  a.ids_in = ids; a.slots = slots; a.miss = miss; a.w_in = w; a.image = static_cast<const uint8_t*>(image);
  a.rec_off = rec_off; a.num_experts = num_experts;
  return val_dtype == VQ2_F16 ? launch_t1<__half>(a, st) : launch_t1<__nv_bfloat16>(a, st);
}

}  // namespace vq2

extern "C" int vq2_paged_moe_t1(const void* h, int h_dtype, int64_t top_k, const int32_t* ids,
                                const int32_t* slots, const int32_t* miss, const float* w, const void* pool,
                                int64_t capacity, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows,
                                int64_t dn_cols, const void* cb0, int val_dtype, const int32_t* perm_in,
                                const int8_t* sign_in, int64_t hb_in, float scale_in, const int32_t* perm_mid,
                                const int8_t* sign_mid, int64_t hb_mid, float scale_mid, const void* image_dev,
                                const int64_t* rec_off, int64_t num_experts, void* workspace, int64_t workspace_bytes,
                                void* out, int out_dtype, void* stream) {
  using namespace vq2;
  if (!h || !ids || !slots || !miss || !w || !pool || !cb0 || !perm_in || !sign_in || !perm_mid || !sign_mid ||
      !image_dev || !rec_off || !workspace || !out)
    return VQ2_ERR_ARG;
  if (h_dtype != VQ2_F32 && h_dtype != VQ2_F16 && h_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (out_dtype != VQ2_F32 && out_dtype != VQ2_F16 && out_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (capacity <= 0 || num_experts <= 0) return VQ2_ERR_SHAPE;
  if (workspace_bytes < vq2_paged_moe_t1_workspace(top_k)) return VQ2_ERR_ARG;
  return run_moe_t1_paged(h, h_dtype, top_k, ids, slots, miss, w, pool, capacity, gu_rows, gu_cols, dn_rows,
                          dn_cols, cb0, val_dtype, perm_in, sign_in, hb_in, scale_in, perm_mid, sign_mid, hb_mid,
                          scale_mid, image_dev, rec_off, num_experts, static_cast<float*>(workspace), out, out_dtype,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int64_t vq2_paged_moe_t1_workspace(int64_t top_k) {
  if (top_k <= 0 || top_k > vq2::kT1MaxK) return -1;
  return top_k * vq2::kT1GuRows * 4;
}
