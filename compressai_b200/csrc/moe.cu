// MoE helper kernels: router (softmax top-k) and routing-weighted combine of expert outputs.
#include <cfloat>

#include "gemv_dev.cuh"

namespace vq2 {

// Router of one MoE layer, ONE CTA of 1024 threads for all T tokens (decode sizes): the math of
// transformers Qwen3_5MoeTopKRouter.forward (softmax fp32 -> topk -> /= sum of the selected) and
// of the shared expert's sigmoid(h . shared_gate) in Qwen3_5MoeSparseMoeBlock.forward.
//   * Selection by rank counting: each of the TPT threads of a token holds one logit and counts
//     the logits that beat it (greater, or equal with a lower expert id); ranks < K are the
//     top-k in descending order with ties to the lower id, as the reference's argmax order.
//     Softmax is monotonic, so this selects on the logits themselves.
//   * Weights: exp(l_k - l_max) / sum over the selected of exp(l_j - l_max), summed in rank
//     order by every selected thread alike (deterministic). The full softmax denominator
//     cancels, so this is the reference's renormalised softmax up to fp32 rounding (~1e-7).
//   * Layer mode (RouteArgs.xrot set): the expert ids are mapped to rows of this rank's pool
//     (lo <= e < hi -> e - lo, else -1), the shared expert becomes problem column K (pool row
//     shared_row, computed on rank t % world), the input RHT of every token's hidden state is
//     written once for all CTAs of the gate_up GEMV, and the problems are compacted in order
//     (ids, map, count, per-token start and count) for the GEMVs that follow.
constexpr int kRouteThreads = 1024;

template <int TPT>
__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const RouteArgs r) {
  constexpr int TPR = kRouteThreads / TPT;  // tokens per round
  __shared__ float sl[TPR][TPT];
  __shared__ int sel_e[TPR][32];
  __shared__ float sel_v[TPR][32];
  __shared__ float red[kRouteThreads / 32];
  __shared__ float rht_sc[8 * (kRouteThreads + kRouteThreads / 32)];  // (1024 / (hb / 8)) x (hb + hb / 32)
  __shared__ int warp_tot[32];
  __shared__ int base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slot = tid / TPT, i = tid % TPT;
  pdl_trigger();  // the GEMV that follows may start its own preamble
  pdl_wait();      // logits, hidden state and the workspace belong to earlier kernels until here
  for (int64_t z = tid; r.zero && z < r.zero_n; z += kRouteThreads) r.zero[z] = 0;

  for (int t0 = 0; t0 < r.T; t0 += TPR) {
    const int t = t0 + slot;
    const bool tok = t < r.T;
    // ---- logits, shared-gate partial dot product (loads of both issued before use)
    const float l = (tok && i < r.E) ? r.logits[(int64_t)t * r.E + i] : -FLT_MAX;
    float d = 0.f;
    if (r.gate != nullptr && tok) {
      for (int k = i; k < r.H; k += TPT) {
        const int64_t o = (int64_t)t * r.H + k;
        const float hv = r.h_dtype == VQ2_F32 ? static_cast<const float*>(r.h)[o]
                         : r.h_dtype == VQ2_F16 ? __half2float(static_cast<const __half*>(r.h)[o])
                                                : __bfloat162float(static_cast<const __nv_bfloat16*>(r.h)[o]);
        d = fmaf(hv, r.gate[k], d);
      }
    }
    sl[slot][i] = l;
    if (r.gate != nullptr) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      if (lane == 0) red[warp] = d;
    }
    __syncthreads();
    // ---- rank of this logit among its token's E logits
    if (tok && i < r.E) {
      int rank = 0;
      const float* row = sl[slot];
#pragma unroll 8
      for (int j = 0; j < r.E; ++j) {
        const float o = row[j];
        rank += (o > l || (o == l && j < i)) ? 1 : 0;
      }
      if (rank < r.K) {
        sel_e[slot][rank] = i;
        sel_v[slot][rank] = l;
      }
    }
    __syncthreads();
    if (tok && i < r.K) {
      const float mx = sel_v[slot][0];
      float sum = 0.f;
      for (int k = 0; k < r.K; ++k) sum += expf(sel_v[slot][k] - mx);
      const int e = sel_e[slot][i];
      const int64_t o = (int64_t)t * r.ks + i;
      r.ids[o] = r.layer ? ((e >= r.lo && e < r.hi) ? e - r.lo : -1) : e;
      r.w[o] = expf(sel_v[slot][i] - mx) / sum;
    }
    if (r.gate != nullptr && tok && i == 0) {
      float dd = 0.f;
      for (int wv = 0; wv < TPT / 32; ++wv) dd += red[slot * (TPT / 32) + wv];
      const float sw = 1.f / (1.f + expf(-dd));
      if (r.layer) {
        r.ids[(int64_t)t * r.ks + r.K] = (t % r.world == r.rank) ? r.shared_row : -1;
        r.w[(int64_t)t * r.ks + r.K] = sw;
      } else if (r.shared_w) {
        r.shared_w[t] = sw;
      }
    }
    __syncthreads();
  }
  if (!r.layer) return;

  // ---- forward RHT of every token's hidden state, fp32 [T, H]: segments of hb elements, each
  // handled by hb / 8 threads (8 values each): 3 butterfly stages in registers, a transpose
  // through shared memory, 3 more in registers, the rest by warp shuffles
  {
    const int TS = r.hb >> 3, SPR = kRouteThreads / TS, nb = r.H / r.hb;
    const int sg = tid / TS, ts = tid % TS;
    float* sc = rht_sc + sg * (r.hb + (r.hb >> 5));
    for (int s0 = 0; s0 < r.T * nb; s0 += SPR) {
      const int gs = s0 + sg;
      const bool act = sg < SPR && gs < r.T * nb;
      const int t = act ? gs / nb : 0, b = act ? gs % nb : 0;
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float val = 0.f;
        if (act) {
          const int j = b * r.hb + ts + TS * q;
          const int64_t o = (int64_t)t * r.H + r.perm[j];
          const float hv = r.h_dtype == VQ2_F32 ? static_cast<const float*>(r.h)[o]
                           : r.h_dtype == VQ2_F16 ? __half2float(static_cast<const __half*>(r.h)[o])
                                                  : __bfloat162float(static_cast<const __nv_bfloat16*>(r.h)[o]);
          val = hv * static_cast<float>(r.sign[j]);
        }
        v[q] = val;
      }
      fwht8(v);
      if (act) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int e = ts + TS * q;
          sc[e + (e >> 5)] = v[q];
        }
      }
      __syncthreads();
      if (act) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int e = 8 * ts + q;
          v[q] = sc[e + (e >> 5)];
        }
      }
      fwht8(v);
      for (int td = 1; td <= (TS >> 4); td <<= 1) {
        const bool upper = (ts & td) != 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float o = __shfl_xor_sync(0xffffffffu, v[q], td);
          v[q] = upper ? (o - v[q]) : (v[q] + o);
        }
      }
      if (act) {
        float* o = r.xrot + (int64_t)t * r.H + b * r.hb + 8 * ts;
        reinterpret_cast<float4*>(o)[0] = make_float4(v[0] * r.rot_scale, v[1] * r.rot_scale, v[2] * r.rot_scale,
                                                      v[3] * r.rot_scale);
        reinterpret_cast<float4*>(o)[1] = make_float4(v[4] * r.rot_scale, v[5] * r.rot_scale, v[6] * r.rot_scale,
                                                      v[7] * r.rot_scale);
      }
      __syncthreads();
    }
  }

  // ---- stable compaction of the T * ks problems (pool row >= 0) and per-token ranges
  const int P = r.T * r.ks;
  if (tid == 0) base = 0;
  __syncthreads();
  for (int c0 = 0; c0 < P; c0 += kRouteThreads) {
    const int p = c0 + tid;
    const int32_t id = p < P ? r.ids[p] : -1;
    const bool keep = id >= 0;
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) warp_tot[warp] = __popc(m);
    __syncthreads();
    int off = base;
    for (int wv = 0; wv < warp; ++wv) off += warp_tot[wv];
    if (keep) {
      const int pos = off + __popc(m & ((1u << lane) - 1u));
      r.c_ids[pos] = id;
      r.c_map[pos] = p;
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int wv = 0; wv < 32; ++wv) tot += warp_tot[wv];
      base += tot;
    }
    __syncthreads();
  }
  if (tid == 0) *r.c_cnt = base;
  // per-token ranges: count of kept problems before token t and within it
  for (int t = tid; t < r.T; t += kRouteThreads) {
    int before = 0, mine = 0;
    for (int p = 0; p < t * r.ks; ++p) before += r.ids[p] >= 0 ? 1 : 0;
    for (int k = 0; k < r.ks; ++k) mine += r.ids[t * r.ks + k] >= 0 ? 1 : 0;
    r.tstart[t] = before;
    r.tcnt[t] = mine;
    if (mine == 0 && r.out != nullptr) {  // nothing of this token is computed here: its output is zero
      for (int k = 0; k < r.H; ++k) {
        const int64_t o = (int64_t)t * r.H + k;
        if (r.out_dtype == VQ2_F16) static_cast<__half*>(r.out)[o] = __float2half_rn(0.f);
        else if (r.out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(r.out)[o] = __float2bfloat16_rn(0.f);
        else static_cast<float*>(r.out)[o] = 0.f;
      }
    }
  }
}

// Router, one CTA of 1024 threads per token (layer mode). Used when every problem of the layer
// is local to this GPU (the problem list is then the identity: nothing to compact) or when a
// persistent arrival counter is given (expert parallelism: the last CTA to finish compacts the
// layer's problems and resets the counter). All global loads a token needs -- its logits, its
// hidden row (16-byte vectors), the shared gate -- are issued together after the dependency
// wait; the rotation table is staged in shared memory before it (constant). Each of the TPT
// logit slots has PARTS = 1024 / TPT threads that split the rank count.
constexpr int kRouteMaxH = 4096;

template <int TPT>
__global__ void __launch_bounds__(1024) moe_route_token_kernel(const RouteArgs r) {
  constexpr int PARTS = 1024 / TPT;
  __shared__ float sl[TPT];
  __shared__ int sel_e[32];
  __shared__ float sel_v[32];
  __shared__ float red[32];
  __shared__ __align__(16) float hs[kRouteMaxH];
  __shared__ uint16_t ps[kRouteMaxH];
  __shared__ float sc[kRouteMaxH + kRouteMaxH / 32];  // segments x (hb + hb / 32) floats
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = blockIdx.x;
  const int H = r.H, nv = H >> 3;
  // rotation table (constant): perm with the sign in bit 15
  for (int j = tid; j < H; j += 1024) ps[j] = static_cast<uint16_t>(r.perm[j] | (r.sign[j] < 0 ? 0x8000 : 0));
  pdl_trigger();
  pdl_wait();
  // ---- all loads of this token at once: logit slot, hidden row (8 values per thread), gate
  const int i = tid / PARTS, part = tid % PARTS;
  float l = -FLT_MAX;
  if (part == 0 && i < r.E) l = r.logits[(int64_t)t * r.E + i];
  float hv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float gv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (tid < nv) {
    const int64_t off = (int64_t)t * H + 8 * tid;
    if (r.h_dtype == VQ2_F32) {
      const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(r.h) + off);
      const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(r.h) + off + 4);
      hv[0] = a.x; hv[1] = a.y; hv[2] = a.z; hv[3] = a.w; hv[4] = b.x; hv[5] = b.y; hv[6] = b.z; hv[7] = b.w;
    } else if (r.h_dtype == VQ2_F16) {
      decode8<__half>(*reinterpret_cast<const uint4*>(static_cast<const __half*>(r.h) + off), hv);
    } else {
      decode8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(r.h) + off), hv);
    }
    if (r.gate) {
      const float4 a = *reinterpret_cast<const float4*>(r.gate + 8 * tid);
      const float4 b = *reinterpret_cast<const float4*>(r.gate + 8 * tid + 4);
      gv[0] = a.x; gv[1] = a.y; gv[2] = a.z; gv[3] = a.w; gv[4] = b.x; gv[5] = b.y; gv[6] = b.z; gv[7] = b.w;
    }
  }
  if (part == 0 && i < TPT) sl[i] = l;
  float d = 0.f;
  if (tid < nv) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      hs[8 * tid + k] = hv[k];
      d = fmaf(hv[k], gv[k], d);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
  if (lane == 0) red[warp] = d;
  for (int64_t z = tid; r.zero && z < r.zero_n / r.T; z += 1024) r.zero[(int64_t)t * (r.zero_n / r.T) + z] = 0;
  __syncthreads();
  // ---- rank of each logit
  if (TPT <= 256 && r.K <= 8) {
    // top-k by route_key (the rank rule below): each of the first 8 warps ranks its 32 keys by
    // shuffles and keeps its top k; one pass ranks the 8 x k candidates
    __shared__ unsigned long long cand[64];
    if (tid < 256) {
      const float v = tid < r.E ? sl[tid] : 0.f;
      const unsigned long long key = tid < r.E ? route_key(v, tid) : 0ull;
      if (lane < r.K) cand[warp * r.K + lane] = 0ull;
      int cnt = 0;
#pragma unroll
      for (int m = 0; m < 32; ++m) cnt += __shfl_sync(0xffffffffu, key, m) > key ? 1 : 0;
      __syncwarp();
      if (cnt < r.K) cand[warp * r.K + cnt] = key;  // lanes past E share one zero key's slot
    }
    __syncthreads();
    if (tid < 8 * r.K) {
      const unsigned long long k = cand[tid];
      int rank = 0;
      for (int d = 0; d < 8 * r.K; ++d) rank += cand[d] > k ? 1 : 0;
      if (rank < r.K && k != 0ull) {
        const int e = static_cast<int>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffull));
        sel_e[rank] = e;
        sel_v[rank] = sl[e];
      }
    }
  } else {  // PARTS threads count interleaved slices of the others
    const float li = i < r.E ? sl[i] : -FLT_MAX;
    int rank = 0;
#pragma unroll 8
    for (int j = part; j < r.E; j += PARTS) {
      const float o = sl[j];
      rank += (o > li || (o == li && j < i)) ? 1 : 0;
    }
#pragma unroll
    for (int off = 1; off < PARTS; off <<= 1) rank += __shfl_xor_sync(0xffffffffu, rank, off);
    if (part == 0 && i < r.E && rank < r.K) {
      sel_e[rank] = i;
      sel_v[rank] = li;
    }
  }
  __syncthreads();
  const int64_t row = (int64_t)t * r.ks;
  if (tid < r.K) {
    const float mx = sel_v[0];
    float sum = 0.f;
    for (int k = 0; k < r.K; ++k) sum += expf(sel_v[k] - mx);
    const int e = sel_e[tid];
    r.ids[row + tid] = (e >= r.lo && e < r.hi) ? e - r.lo : -1;
    r.w[row + tid] = expf(sel_v[tid] - mx) / sum;
  }
  if (r.gate && warp == 1) {  // the 32 warp sums of the shared-gate dot product, by shuffles
    float dd = red[lane];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, off);
    if (lane == 0) {
      r.ids[row + r.K] = (t % r.world == r.rank) ? r.shared_row : -1;
      r.w[row + r.K] = 1.f / (1.f + expf(-dd));
    }
  }
  // ---- forward RHT of the hidden row from shared memory into xrot
  {
    const int TS = r.hb >> 3, nb = H / r.hb;
    const int sg = tid / TS, ts = tid % TS;
    const bool act = sg < nb;
    float* scr = sc + (act ? sg : 0) * (r.hb + (r.hb >> 5));
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float val = 0.f;
      if (act) {
        const uint32_t pq = ps[sg * r.hb + ts + TS * q];
        const float x = hs[pq & 0x7fffu];
        val = (pq & 0x8000u) ? -x : x;
      }
      v[q] = val;
    }
    fwht8(v);
    if (act) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int e = ts + TS * q;
        scr[e + (e >> 5)] = v[q];
      }
    }
    __syncthreads();
    if (act) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int e = 8 * ts + q;
        v[q] = scr[e + (e >> 5)];
      }
    }
    fwht8(v);
    for (int td = 1; td <= (TS >> 4); td <<= 1) {
      const bool upper = (ts & td) != 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float o = __shfl_xor_sync(0xffffffffu, v[q], td);
        v[q] = upper ? (o - v[q]) : (v[q] + o);
      }
    }
    if (act) {
      float* o = r.xrot + (int64_t)t * H + sg * r.hb + 8 * ts;
      reinterpret_cast<float4*>(o)[0] = make_float4(v[0] * r.rot_scale, v[1] * r.rot_scale, v[2] * r.rot_scale,
                                                    v[3] * r.rot_scale);
      reinterpret_cast<float4*>(o)[1] = make_float4(v[4] * r.rot_scale, v[5] * r.rot_scale, v[6] * r.rot_scale,
                                                    v[7] * r.rot_scale);
    }
  }
  // ---- the problem list
  if (r.arrive == nullptr) {  // every problem is local: the identity list
    if (tid < r.ks) {
      r.c_ids[row + tid] = r.ids[row + tid];
      r.c_map[row + tid] = static_cast<int32_t>(row + tid);
    }
    if (tid == 0) {
      r.tstart[t] = static_cast<int32_t>(row);
      r.tcnt[t] = r.ks;
      if (t == 0) *r.c_cnt = r.T * r.ks;
    }
    return;
  }
  // expert parallel: the last CTA compacts all tokens' problems in order and resets the counter
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(r.arrive, 1) == r.T - 1) ? 1 : 0;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __shared__ int warp_tot[32];
  __shared__ int base;
  const int P = r.T * r.ks;
  if (tid == 0) base = 0;
  __syncthreads();
  for (int c0 = 0; c0 < P; c0 += 1024) {
    const int p = c0 + tid;
    const int32_t id = p < P ? __ldcg(r.ids + p) : -1;
    const bool keep = id >= 0;
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) warp_tot[warp] = __popc(m);
    __syncthreads();
    int off = base;
    for (int wv = 0; wv < warp; ++wv) off += warp_tot[wv];
    if (keep) {
      const int pos = off + __popc(m & ((1u << lane) - 1u));
      r.c_ids[pos] = id;
      r.c_map[pos] = p;
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int wv = 0; wv < 32; ++wv) tot += warp_tot[wv];
      base += tot;
    }
    __syncthreads();
  }
  if (tid == 0) {
    *r.c_cnt = base;
    *r.arrive = 0;
  }
  // per-token counts in parallel, then their exclusive prefix (the transform scratch is free now;
  // T <= kRouteMaxH fits it)
  int* cnt = reinterpret_cast<int*>(sc);
  for (int tt = tid; tt < r.T; tt += 1024) {
    int mine = 0;
    for (int k = 0; k < r.ks; ++k) mine += __ldcg(r.ids + tt * r.ks + k) >= 0 ? 1 : 0;
    cnt[tt] = mine;
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int tt = 0; tt < r.T; ++tt) {
      const int c = cnt[tt];
      cnt[tt] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int tt = tid; tt < r.T; tt += 1024) {
    const int start = cnt[tt];
    r.tstart[tt] = start;
    r.tcnt[tt] = (tt + 1 < r.T ? cnt[tt + 1] : base) - start;
  }
}

int run_route(const RouteArgs& r, cudaStream_t st) {
  if (r.T <= 0 || r.E <= 0 || r.E > kRouteThreads || r.K <= 0 || r.K > 32 || r.K > r.E) return VQ2_ERR_SHAPE;
  if (r.layer) {
    if (!r.xrot || !r.perm || !r.sign || !r.c_ids || !r.c_map || !r.c_cnt || !r.tstart || !r.tcnt) return VQ2_ERR_ARG;
    if (r.hb < 64 || r.hb > 2048 || (r.hb & (r.hb - 1)) != 0 || r.H % r.hb != 0) return VQ2_ERR_SHAPE;
    if (!aligned(r.xrot, 16) || r.world <= 0 || r.rank < 0 || r.rank >= r.world) return VQ2_ERR_ARG;
  }
  const int tpt = r.E <= 32 ? 32 : r.E <= 64 ? 64 : r.E <= 128 ? 128 : r.E <= 256 ? 256 : r.E <= 512 ? 512 : 1024;
  const bool all_local = r.lo == 0 && r.hi == r.E && r.world == 1;
  if (r.layer && (all_local || r.arrive) && r.H <= kRouteMaxH && r.H % 256 == 0 && r.out == nullptr) {
    // one CTA per token (the per-token work in parallel)
    const dim3 g((unsigned)r.T);
    switch (tpt) {
      case 32: return launch_kernel(moe_route_token_kernel<32>, g, dim3(1024), 0, st, r);
      case 64: return launch_kernel(moe_route_token_kernel<64>, g, dim3(1024), 0, st, r);
      case 128: return launch_kernel(moe_route_token_kernel<128>, g, dim3(1024), 0, st, r);
      case 256: return launch_kernel(moe_route_token_kernel<256>, g, dim3(1024), 0, st, r);
      case 512: return launch_kernel(moe_route_token_kernel<512>, g, dim3(1024), 0, st, r);
      default: return launch_kernel(moe_route_token_kernel<1024>, g, dim3(1024), 0, st, r);
    }
  }
  switch (tpt) {
    case 32: return launch_kernel(moe_route_kernel<32>, dim3(1), dim3(kRouteThreads), 0, st, r);
    case 64: return launch_kernel(moe_route_kernel<64>, dim3(1), dim3(kRouteThreads), 0, st, r);
    case 128: return launch_kernel(moe_route_kernel<128>, dim3(1), dim3(kRouteThreads), 0, st, r);
    case 256: return launch_kernel(moe_route_kernel<256>, dim3(1), dim3(kRouteThreads), 0, st, r);
    case 512: return launch_kernel(moe_route_kernel<512>, dim3(1), dim3(kRouteThreads), 0, st, r);
    default: return launch_kernel(moe_route_kernel<1024>, dim3(1), dim3(kRouteThreads), 0, st, r);
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
  for (int j0 = 0; j0 < top_k; j0 += 8) {  // 8 problems' loads in flight, summed in problem order
    bool ok[8];
    float wp[8], yv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t p = t * top_k + j0 + k;
      ok[k] = j0 + k < top_k && (!ids || (ids[p] >= 0 && ids[p] < num_experts));  // else not computed here
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t p = t * top_k + j0 + k;
      wp[k] = ok[k] ? w[p] : 0.f;
      yv[k] = ok[k] ? y[p * H + h] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (ok[k]) s = fmaf(wp[k], yv[k], s);
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
  if (T <= 0 || T > (1 << 20) || E <= 0 || E > kRouteThreads || K <= 0 || K > 32 || K > E) return VQ2_ERR_SHAPE;
  if (shared_gate && (!h || !shared_w || H <= 0 || H > (1 << 24))) return VQ2_ERR_ARG;
  if (shared_gate && h_dtype != VQ2_F32 && h_dtype != VQ2_F16 && h_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  RouteArgs r{};
  r.logits = logits; r.T = (int)T; r.E = (int)E; r.K = (int)K;
  r.h = h; r.h_dtype = h_dtype; r.H = (int)H; r.gate = shared_gate;
  r.ids = ids; r.w = w; r.ks = (int)K; r.shared_w = shared_w; r.layer = false;
  return run_route(r, static_cast<cudaStream_t>(stream));
}

// ---- router logits ------------------------------------------------------------------------
// logits[t, e] = sum_i h[t, i] * W[e, i] with the dense router weight W [E, H] (bf16 or fp16, as
// the reference keeps it unquantized), fp32 accumulation: one warp per expert, 16-byte loads of
// the weight row (L1-resident across tokens) and of each token's hidden row, a shuffle reduction.
// Replaces the F.linear of Qwen3_5MoeTopKRouter.forward (modeling_qwen3_5_moe.py:762-764).
namespace vq2 {
__device__ __forceinline__ void load8(const void* p, int dtype, int64_t off, float (&f)[8]) {
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

__global__ void __launch_bounds__(256) router_logits_kernel(const void* __restrict__ h, int h_dtype,
                                                            const void* __restrict__ W, int w_dtype, int T, int E,
                                                            int H, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_wait();
  if (e >= E) return;
  const int nc = H >> 3;
  for (int t = 0; t < T; ++t) {
    float acc = 0.f;
    for (int c = lane; c < nc; c += 32) {
      float w[8], x[8];
      load8(W, w_dtype, (int64_t)e * H + 8 * c, w);
      load8(h, h_dtype, (int64_t)t * H + 8 * c, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = fmaf(w[i], x[i], acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) out[(int64_t)t * E + e] = acc;
  }
}
}  // namespace vq2

extern "C" int vq2_router_logits(const void* h, int h_dtype, int64_t T, const void* W, int w_dtype, int64_t E,
                                 int64_t H, float* logits, void* stream) {
  using namespace vq2;
  if (!h || !W || !logits) return VQ2_ERR_ARG;
  if (T <= 0 || T > (1 << 20) || E <= 0 || E > (1 << 20) || H <= 0 || H % 8 != 0 || H > (1 << 24)) return VQ2_ERR_SHAPE;
  if (h_dtype != VQ2_F32 && h_dtype != VQ2_F16 && h_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (w_dtype != VQ2_F16 && w_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (!aligned(h, 16) || !aligned(W, 16)) return VQ2_ERR_ALIGN;
  return launch_kernel(router_logits_kernel, dim3((unsigned)((E + 7) / 8)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), h, h_dtype, W, w_dtype, (int)T, (int)E, (int)H, logits);
}
