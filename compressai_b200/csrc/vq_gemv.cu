// Codebook-decode GEMV on CUDA cores (fp32 accumulation), dense and expert-indexed.
//
//   y[m, r] = rs * scale[r] * sum_g dot(cb0[idx0[r, g]] (+ cb1[idx1[r, g]]), xr[m, 8g:8g+8])
//
// Bound: every 2-byte index costs one random 16-byte codebook gather. On B200 the codebook
// (1 MiB fp16) lives in L2 and random 16-byte L2 gathers sustain ~1.1 per clock per SM, so the
// kernel is gather-throughput bound well below HBM bandwidth; the design keeps that pipe busy:
//
// * Work items are (problem k, M tile, block of rows); a persistent grid walks them with a
//   grid stride. A warp owns RW x RPL rows of an item; LPR lanes cover one row, each lane
//   loading 8 consecutive int16 indices (16 B) per chunk with one streaming 128-bit load.
// * The next task's index vectors are prefetched into registers while the current task's
//   gathers and FMAs run, so HBM latency overlaps the gather pipe.
// * Codebook rows are gathered with 128-bit read-only loads (L2 evict-last policy); index
//   streams use no-L1-allocate loads with an L2 evict-first policy so they do not push
//   codebook lines out.
// * For n = 2048 at M = 1 each lane's 64 activations stay in registers for the whole kernel;
//   otherwise the fp32 activation tile sits in shared memory, padded by 4 floats every 8 groups
//   so the 8 lanes of one 128-bit access phase (groups 8 apart) hit distinct bank groups.
// * The residual codebook (3 bpw, 4 KB) is staged in shared memory.
// * Programmatic dependent launch: weights are prefetched before griddepcontrol.wait, so a
//   GEMV's first index loads overlap the tail of the kernel that produces its input.
//
// Semantics: reference vq2/kernels.py:32-78 (_vq_gemv_16_8/_vq_gemv_16, M = 1) and
// :117-176 (_parallel_moe_*: expert-indexed, shared or per-expert activation).
#include <atomic>

#include "gemv_dev.cuh"

namespace vq2 {

// Order-preserving 64-bit key of (value, row) for a greedy argmax by atomicMax: the float's bits
// flipped so that unsigned order is numeric order, then the row complemented so that ties go to
// the smaller row (torch.argmax's choice). NaN-free inputs assumed; 0 means "none".
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xffffffffu - static_cast<uint32_t>(row));
}

// Activation staging. For M tile 1 it is a real call: it runs once per activation tile, and
// keeping its code out of the main loop leaves that loop's register allocation (gathers in
// flight) to itself. Larger M tiles inline it (as a call, its callee-saved registers made the
// permuted global loads of the old staging form spill and serialise).
template <int MT>
__device__ __noinline__ void stage_tile_call(const ActSrc a, int64_t xoff, int mcount, float* xs, int xl,
                                             float* scratch, float* raw, const uint16_t* ps) {
  stage_activations<MT>(a, xoff, mcount, xs, xl, scratch, raw, ps);
}
template <int MT>
__device__ __forceinline__ void stage_tile(const ActSrc& a, int64_t xoff, int mcount, float* xs, int xl,
                                           float* scratch, float* raw, const uint16_t* ps) {
  if constexpr (MT == 1) stage_tile_call<1>(a, xoff, mcount, xs, xl, scratch, raw, ps);
  else stage_activations<MT>(a, xoff, mcount, xs, xl, scratch, raw, ps);
}

// Fused combine (the kEpiComb kernel variants only) after an item of expert-indexed problem o, row
// block rb (RPC rows) is written:
// arrival count per (token, row block); the CTA that brings it to the token's problem count sums
// the token's problems over the block's rows in problem order (the fmaf chain of
// moe_combine_kernel, so the result is bit-identical) and writes comb_out. Called by all
// threads of the CTA at the same point of the item sequence.
__device__ __forceinline__ void combine_tail(const float* __restrict__ comb_w, const int32_t* __restrict__ tstart,
                                         const int32_t* __restrict__ tcnt, int32_t* ctr,
                                         const int32_t* __restrict__ prob_map, const float* y, int64_t y_k_stride,
                                         void* comb_out, int comb_dtype, int comb_ks, int row_blocks, int out, int o,
                                         int rb, int rpc, bool wrote) {
  __shared__ int s_last;
  if (wrote) __threadfence();  // this thread's output rows are visible GPU-wide before the arrival
  __syncthreads();
  const int t = o / comb_ks;
  if (threadIdx.x == 0) {
    const int old = atomicAdd(ctr + (int64_t)t * row_blocks + rb, 1);
    s_last = (old == tcnt[t] - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int r = rb * rpc + (int)threadIdx.x;
  if ((int)threadIdx.x < rpc && r < out) {
    const int c0 = tstart[t], cn = tcnt[t];
    float s = 0.f;
    int c = c0;
    for (; c < c0 + cn; c += 8) {  // 8 problems' loads in flight, summed in problem order
      int oo[8];
      float wv[8], yv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) oo[k] = (c + k < c0 + cn) ? (prob_map ? prob_map[c + k] : c + k) : -1;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        wv[k] = oo[k] >= 0 ? comb_w[oo[k]] : 0.f;
        yv[k] = oo[k] >= 0 ? __ldcg(y + (int64_t)oo[k] * y_k_stride + r) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (oo[k] >= 0) s = fmaf(wv[k], yv[k], s);
    }
    const int64_t i = (int64_t)t * out + r;
    if (comb_dtype == VQ2_F16) static_cast<__half*>(comb_out)[i] = __float2half_rn(s);
    else if (comb_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(comb_out)[i] = __float2bfloat16_rn(s);
    else static_cast<float*>(comb_out)[i] = s;
  }
}

// Epilogue of a kernel variant: plain stores, + the fused MoE combine, or the greedy argmax.
constexpr int kEpiPlain = 0, kEpiComb = 1, kEpiArgmax = 2;

// Variants that stage the fast way: all but the 3 bpw two-row register variant, whose
// registers are taken by its two rows of residual indices.
template <int RW, bool RES, bool XREG>
constexpr bool variant_fast_stage() { return !(RES && XREG && RW == 2); }

template <int LPR, int RW, int MT, bool RES, bool XREG, typename TV, int EPI = kEpiPlain>
__global__ void __launch_bounds__(256, 2) vq_gemv_kernel(const GemvArgs a) {
  static_assert(!XREG || (LPR == 32 && MT == 1), "register activations need one 256-group chunk, M tile 1");
  constexpr int RPL = 32 / LPR;   // rows per warp-load
  constexpr int RPW = RW * RPL;   // rows per warp per item
  constexpr int RPC = 8 * RPW;    // rows per CTA per item
  extern __shared__ __align__(16) float smem[];
  const int n = a.n, ng = n >> 3, xl = xs_len(n);
  float* xs = smem;                                            // [MT][xl] activation tile
  float* scratch = smem + MT * xl;                             // RHT transpose scratch (2112 floats)
  uint4* cb1s = reinterpret_cast<uint4*>(scratch + kScratchFloats);  // [256] when RES
  // Fast staging (gemv_dev.cuh): raw activation rows (or the tile itself) and the rotation
  // table after the residual codebook; recomputed where used, so no registers stay tied up
  // across the main loop.
  auto fast_raw = [&]() -> float* {
    if (!variant_fast_stage<RW, RES, XREG>() || !fast_stage(MT, a.n)) return nullptr;
    if (a.x_mode == VQ2_ACT_ROTATED || stage_in_place(MT, a.n)) return smem;
    return smem + MT * xs_len(a.n) + kScratchFloats + (RES ? 4 * 256 : 0);
  };
  auto fast_ps = [&]() -> uint16_t* {
    return reinterpret_cast<uint16_t*>(smem + MT * xs_len(a.n) + kScratchFloats + (RES ? 4 * 256 : 0) +
                                       (stage_in_place(MT, a.n) ? 0 : fast_raw_rows(MT, a.n) * a.n));
  };

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LPR, li = lane % LPR;
  const int chunks = ng / (8 * LPR);
  const bool multi = a.nprob > 0;
  const uint4* cb0 = static_cast<const uint4*>(a.cb0);
  const uint64_t pol_s = policy_evict_first();
  const uint64_t pol_c = policy_evict_last();
  const bool weights_known = (a.e_ids == nullptr);  // expert ids may come from the previous kernel

  // One work item = RPC rows of one problem for one M tile. Each CTA owns a contiguous range
  // of items, so consecutive items mostly share their problem and activation tile.
  struct Item { int rb, mt, k, o, out; int64_t e; const int16_t* i0; const uint8_t* i1; bool valid; };
  auto decode = [&](int64_t it) -> Item {
    Item w;
    if (multi) {
      w.mt = (int)(it / a.row_blocks);
      const int rbg = (int)(it - (int64_t)w.mt * a.row_blocks);
      int p = 0;
#pragma unroll 1
      while (p + 1 < a.nprob && rbg >= a.p_rb0[p + 1]) ++p;
      w.k = p;
      w.o = p;
      w.rb = rbg - a.p_rb0[p];
      w.out = a.p_out[p];
      w.e = 0;
      w.i0 = a.p_idx0[p];
      w.i1 = a.p_idx1[p];
      w.valid = true;
    } else {
      w.rb = (int)(it % a.row_blocks);
      const int64_t q = it / a.row_blocks;
      w.mt = (int)(q % a.mtiles);
      w.k = (int)(q / a.mtiles);
      w.o = a.prob_map ? a.prob_map[w.k] : w.k;
      w.out = a.out;
      int64_t e = 0;
      w.valid = true;
      if (a.e_ids) {
        e = a.e_ids[w.k];
        w.valid = (e >= 0 && e < a.num_experts);
        if (!w.valid) e = 0;
      }
      w.e = e;
      w.i0 = a.idx0 + e * a.idx_e_stride;
      w.i1 = RES ? a.idx1 + e * a.idx1_e_stride : nullptr;
    }
    return w;
  };
  // Index vectors of chunk c of item w; with the last chunk, the rows' scales too (lane li == 0
  // only), so the epilogue waits on no memory round trip of its own.
  auto load_idx = [&](const Item& w, int c, uint4 (&iv)[RW], uint2 (&jv)[RW], float (&sv)[RW]) {
    const int g0 = (c * LPR + li) * 8;
    const TV* sc = multi ? static_cast<const TV*>(a.p_scale[w.k])
                         : static_cast<const TV*>(a.scale) + w.e * a.scale_e_stride;
#pragma unroll
    for (int rw = 0; rw < RW; ++rw) {
      const int r = w.rb * RPC + warp * RPW + rw * RPL + sub;
      sv[rw] = 0.f;
      if (w.valid && r < w.out) {
        iv[rw] = ld_stream_u4(w.i0 + (int64_t)r * ng + g0, pol_s);
        if (RES) jv[rw] = ld_stream_u2(w.i1 + (int64_t)r * ng + g0, pol_s);
        if (li == 0 && c == chunks - 1) sv[rw] = to_f32<TV>(sc[r]) * a.rs;
      } else {
        iv[rw] = make_uint4(0, 0, 0, 0);
        if (RES) jv[rw] = make_uint2(0, 0);
      }
    }
  };

  // This CTA's contiguous item range. With two CTAs per SM (the grid is the SMs x 2), CTAs b and
  // b + G/2 split one SM-sized share of the items between them, so per-SM totals differ by at
  // most one item (a CTA-level floor/ceil split alone can still give some SMs two large ranges);
  // otherwise a plain floor/ceil split.
  auto cta_items = [&](int64_t items, int64_t& lo, int64_t& hi) {
    const int64_t G = gridDim.x, b = blockIdx.x;
    if (G % 2 == 0) {
      const int64_t half = G / 2, pr = b % half;
      const int64_t p0 = pr * items / half, p1 = (pr + 1) * items / half, mid = p0 + (p1 - p0 + 1) / 2;
      lo = b < half ? p0 : mid;
      hi = b < half ? mid : p1;
    } else {
      lo = b * items / G;
      hi = (b + 1) * items / G;
    }
  };

  // Items are known before the dependency wait unless the problem count lives on the device.
  const int64_t items_max = multi ? (int64_t)a.row_blocks * a.mtiles : (int64_t)a.row_blocks * a.K * a.mtiles;
  int64_t item, item_end;
  cta_items(items_max, item, item_end);
  int chunk = 0;
  uint4 iv[RW];
  uint2 jv[RW];
  float sv[RW];
  Item cur;
  if (weights_known && item < item_end) {  // constant weights: safe before the dependency wait
    cur = decode(item);
    load_idx(cur, 0, iv, jv, sv);
  }
  if (variant_fast_stage<RW, RES, XREG>() && fast_stage_floats(MT, n, a.x_mode) > 0)
    stage_perm(act_src(a), fast_ps());  // constant too; the staging barrier follows
  pdl_wait();
  if (!multi && a.prob_count) {  // device-side problem count (compacted problem lists)
    const int kc = min(a.K, max(0, *a.prob_count));
    const int64_t items = (int64_t)a.row_blocks * kc * a.mtiles;
    cta_items(items, item, item_end);
  }
  if (!weights_known && item < item_end) {
    cur = decode(item);
    load_idx(cur, 0, iv, jv, sv);
  }
  if (RES) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) cb1s[i] = static_cast<const uint4*>(a.cb1)[i];
  }
  pdl_trigger();

  // greedy argmax: each warp's running best key per activation row of its current M tile
  __shared__ unsigned long long s_best[EPI == kEpiArgmax ? 8 : 1][MT];
  __shared__ int s_tile[EPI == kEpiArgmax ? 8 : 1];
  if constexpr (EPI == kEpiArgmax) {
    if (lane == 0) {
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) s_best[warp][mi] = 0ull;
      s_tile[warp] = -1;
    }
  }
  int64_t cur_xoff = -1;
  float xreg[XREG ? 64 : 1];
  float acc[RW][MT];

  while (item < item_end) {
    const int m0 = cur.mt * MT;
    const int mcount = min(MT, a.M - m0);
    const int64_t xoff = (int64_t)m0 * a.x_row_stride + (multi ? 0 : (int64_t)(cur.o / a.x_k_div) * a.x_k_stride);
    if (xoff != cur_xoff) {  // uniform over the CTA
      __syncthreads();
      stage_tile<MT>(act_src(a), xoff, mcount, xs, xl, scratch, fast_raw(), fast_ps());
      __syncthreads();
      if constexpr (XREG) {  // this lane's 8 groups -> registers (conflict-free: lanes 68 floats apart)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 lo = *reinterpret_cast<const float4*>(xs + xs_pos(li * 8 + j, 0));
          const float4 hi = *reinterpret_cast<const float4*>(xs + xs_pos(li * 8 + j, 4));
          xreg[j * 8 + 0] = lo.x; xreg[j * 8 + 1] = lo.y; xreg[j * 8 + 2] = lo.z; xreg[j * 8 + 3] = lo.w;
          xreg[j * 8 + 4] = hi.x; xreg[j * 8 + 5] = hi.y; xreg[j * 8 + 6] = hi.z; xreg[j * 8 + 7] = hi.w;
        }
      }
      cur_xoff = xoff;
    }

    // prefetch the next task's indices
    int64_t nitem = item;
    int nchunk = chunk + 1;
    if (nchunk == chunks) { nchunk = 0; nitem = item + 1; }
    uint4 nv[RW];
    uint2 njv[RW];
    float nsv[RW] = {};
    Item nxt = cur;
    if (nitem < item_end) {
      if (nitem != item) nxt = decode(nitem);
      load_idx(nxt, nchunk, nv, njv, nsv);
    }

    if (chunk == 0) {
#pragma unroll
      for (int rw = 0; rw < RW; ++rw)
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) acc[rw][mi] = 0.f;
    }
    const int g0 = (chunk * LPR + li) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float xv[MT][8];
      if constexpr (XREG) {
#pragma unroll
        for (int t = 0; t < 8; ++t) xv[0][t] = xreg[j * 8 + t];
      } else {
        const int p = xs_pos(g0 + j, 0);
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
          const float4 lo = *reinterpret_cast<const float4*>(xs + mi * xl + p);
          const float4 hi = *reinterpret_cast<const float4*>(xs + mi * xl + p + 4);
          xv[mi][0] = lo.x; xv[mi][1] = lo.y; xv[mi][2] = lo.z; xv[mi][3] = lo.w;
          xv[mi][4] = hi.x; xv[mi][5] = hi.y; xv[mi][6] = hi.z; xv[mi][7] = hi.w;
        }
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

    if (chunk == chunks - 1) {
#pragma unroll
      for (int rw = 0; rw < RW; ++rw)
#pragma unroll
        for (int mi = 0; mi < MT; ++mi)
#pragma unroll
          for (int off = LPR / 2; off > 0; off >>= 1) acc[rw][mi] += __shfl_xor_sync(0xffffffffu, acc[rw][mi], off);
      // greedy argmax (one matrix): per activation row, the warp's best (value, row) key
      unsigned long long best[EPI == kEpiArgmax ? MT : 1];
      if constexpr (EPI == kEpiArgmax) {
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) best[mi] = 0ull;
      }
      if (li == 0) {
        void* ybase = multi ? a.p_y[cur.k] : a.y;
        const int64_t yk = multi ? 0 : (int64_t)cur.o * a.y_k_stride;
#pragma unroll
        for (int rw = 0; rw < RW; ++rw) {
          const int r = cur.rb * RPC + warp * RPW + rw * RPL + sub;
          if (r < cur.out) {
            const float s = sv[rw];
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) {
              if (mi < mcount) {
                const int64_t o = yk + (int64_t)(m0 + mi) * a.y_row_stride + r;
                const float v = acc[rw][mi] * s;
                if constexpr (EPI == kEpiArgmax) {
                  const unsigned long long key = argmax_key(v, r);
                  best[mi] = key > best[mi] ? key : best[mi];
                  if (a.no_y) continue;
                }
                if (a.y_dtype == VQ2_F16) static_cast<__half*>(ybase)[o] = __float2half_rn(v);
                else if (a.y_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(ybase)[o] = __float2bfloat16_rn(v);
                else static_cast<float*>(ybase)[o] = v;
              }
            }
          }
        }
      }
      if constexpr (EPI == kEpiArgmax) {
        // the warp's best of this item joins its running best; the running bests go out (one
        // atomic per row) only when the warp moves to another M tile and at the end of the
        // CTA's items, not once per item: 64-bit atomics on one address serialise in L2
        if (lane == 0 && s_tile[warp] != m0) {
          if (s_tile[warp] >= 0) {
#pragma unroll
            for (int mi = 0; mi < MT; ++mi)
              if (s_best[warp][mi]) atomicMax(a.argmax + s_tile[warp] + mi, s_best[warp][mi]);
          }
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) s_best[warp][mi] = 0ull;
          s_tile[warp] = m0;
        }
#pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
          unsigned long long b = best[mi];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long q = __shfl_xor_sync(0xffffffffu, b, off);
            b = q > b ? q : b;
          }
          if (lane == 0 && mi < mcount && b > s_best[warp][mi]) s_best[warp][mi] = b;
        }
      }
      if constexpr (EPI == kEpiComb)  // uniform over the CTA
        combine_tail(a.comb_w, a.comb_tstart, a.comb_tcnt, a.comb_ctr, a.prob_map, static_cast<const float*>(a.y),
                     a.y_k_stride, a.comb_out, a.comb_dtype, a.comb_ks, a.row_blocks, a.out, cur.o, cur.rb, RPC,
                     li == 0);
    }
    item = nitem;
    chunk = nchunk;
    cur = nxt;
#pragma unroll
    for (int rw = 0; rw < RW; ++rw) {
      iv[rw] = nv[rw];
      if (RES) jv[rw] = njv[rw];
      sv[rw] = nsv[rw];
    }
  }
  if constexpr (EPI == kEpiArgmax) {
    if (lane == 0 && s_tile[warp] >= 0) {
#pragma unroll
      for (int mi = 0; mi < MT; ++mi)
        if (s_best[warp][mi]) atomicMax(a.argmax + s_tile[warp] + mi, s_best[warp][mi]);
    }
  }
}

// ---- host dispatch ------------------------------------------------------------------------
constexpr int kMaxXsBytes = 80 * 1024;  // activation tile cap; the rest of the SM's 256 KB stays L1
constexpr int kTcMinRows = 4;           // activation rows from which the tensor-core path is used
constexpr int64_t kTcTallRows = 16384;  // ...or from 2 rows when the matrices have this many rows

template <int LPR, int RW, int MT, bool RES, bool XREG, typename TV, int EPI = kEpiPlain>
static int launch_cfg(GemvArgs a, cudaStream_t st) {
  constexpr int RPC = 8 * RW * (32 / LPR);
  a.mtiles = (a.M + MT - 1) / MT;
  int64_t items;
  if (a.nprob > 0) {
    int rb = 0;
    for (int p = 0; p < a.nprob; ++p) {
      a.p_rb0[p] = rb;
      rb += (a.p_out[p] + RPC - 1) / RPC;
    }
    a.p_rb0[a.nprob] = rb;
    a.row_blocks = rb;
    items = (int64_t)rb * a.mtiles;
  } else {
    a.row_blocks = (a.out + RPC - 1) / RPC;
    items = (int64_t)a.row_blocks * a.K * a.mtiles;
  }
  const size_t smem = ((size_t)MT * xs_len(a.n) + kScratchFloats +
                       (variant_fast_stage<RW, RES, XREG>() ? fast_stage_floats(MT, a.n, a.x_mode) : 0)) *
                          sizeof(float) +
                      (RES ? 256 * sizeof(uint4) : 0);
  auto kern = vq_gemv_kernel<LPR, RW, MT, RES, XREG, TV, EPI>;
  // Per-device one-time attributes: dynamic shared memory opt-in and, for the small-tile
  // variants, a small shared-memory carveout so most of the SM's 256 KB serves as L1.
  static std::atomic<uint64_t> done{0};
  static std::atomic<int> blocks_per_sm{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kGemvSmemCap);
    if (e == cudaSuccess && XREG) {  // small carveout (most of the SM's memory as L1), room for 2 CTAs
      const int cta = ((xs_len(2048) + kScratchFloats + fast_extra_floats(1, 2048)) * 4 + (RES ? 4096 : 0)) + 1024;
      const int pct = (2 * cta * 100 + 228 * 1024 - 1) / (228 * 1024);
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, pct > 20 ? pct : 20);
    }
    if (e != cudaSuccess) { set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    int nb = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, 256, smem);
    blocks_per_sm.store(nb > 0 ? nb : 1);
    done.fetch_or(bit);
  }
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm.load();
  const int64_t grid = items < cap ? items : cap;
  if (grid <= 0) return VQ2_OK;
  return launch_kernel(kern, dim3((unsigned)grid), dim3(256), smem, st, a);
}

template <int LPR, int RW, bool RES, typename TV, int EPI>
static int launch_mt(const GemvArgs& a, int mt, bool xreg, cudaStream_t st) {
  if constexpr (LPR == 32) {
    if (xreg && mt == 1) return launch_cfg<LPR, RW, 1, RES, true, TV, EPI>(a, st);
  }
  switch (mt) {
    case 1: return launch_cfg<LPR, RW, 1, RES, false, TV, EPI>(a, st);
    case 2: return launch_cfg<LPR, RW, 2, RES, false, TV, EPI>(a, st);
    case 4: return launch_cfg<LPR, RW, 4, RES, false, TV, EPI>(a, st);
    default: return launch_cfg<LPR, RW, 8, RES, false, TV, EPI>(a, st);
  }
}

template <int LPR, bool RES, typename TV, int EPI>
static int launch_rw(const GemvArgs& a, int64_t total_rows, int mt, bool xreg, cudaStream_t st) {
  // Few rows (small matrices) or wide M tiles: one row per warp-load keeps many CTAs busy within
  // the register budget. Many rows at M tile 1, and expert-indexed problems at any count: two
  // rows per warp put twice the gathers in flight per lane (for MoE problems the rows are known
  // only after the routing kernel, so the CTAs should finish their shares in fewer rounds).
  if (mt == 1 && (a.nprob == 0 || total_rows >= (int64_t)sm_count() * 8 * 2 * 8 * (32 / LPR))) {
    if (xreg && LPR == 32) return launch_cfg<LPR, 2, 1, RES, LPR == 32, TV, EPI>(a, st);
    return launch_cfg<LPR, 2, 1, RES, false, TV, EPI>(a, st);
  }
  return launch_mt<LPR, 1, RES, TV, EPI>(a, mt, xreg, st);
}

template <bool RES, typename TV, int EPI>
static int launch_lpr(const GemvArgs& a, int64_t total_rows, int lpr, int mt, cudaStream_t st) {
  const bool xreg = (a.n == 2048);
  switch (lpr) {
    case 4: return launch_rw<4, RES, TV, EPI>(a, total_rows, mt, false, st);
    case 8: return launch_rw<8, RES, TV, EPI>(a, total_rows, mt, false, st);
    case 16: return launch_rw<16, RES, TV, EPI>(a, total_rows, mt, false, st);
    default: return launch_rw<32, RES, TV, EPI>(a, total_rows, mt, xreg, st);
  }
}

template <bool RES, typename TV>
static int launch_epi(const GemvArgs& a, int64_t total_rows, int lpr, int mt, cudaStream_t st) {
  if (a.argmax) return launch_lpr<RES, TV, kEpiArgmax>(a, total_rows, lpr, mt, st);
  return launch_lpr<RES, TV, kEpiPlain>(a, total_rows, lpr, mt, st);
}

template <int RW, typename TV>
static int launch_comb(const GemvArgs& a, int lpr, cudaStream_t st) {
  switch (lpr) {
    case 4: return launch_cfg<4, RW, 1, false, false, TV, kEpiComb>(a, st);
    case 8: return launch_cfg<8, RW, 1, false, false, TV, kEpiComb>(a, st);
    case 16: return launch_cfg<16, RW, 1, false, false, TV, kEpiComb>(a, st);
    default: return launch_cfg<32, RW, 1, false, false, TV, kEpiComb>(a, st);
  }
}

// Largest M tile (1, 2, 4, 8) whose fp32 activation tile fits kMaxXsBytes of shared memory.
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

static int check_act(const GemvArgs& a) {
  if (a.x_mode == VQ2_ACT_ROTATED) return VQ2_OK;
  if (a.x_mode != VQ2_ACT_RHT && a.x_mode != VQ2_ACT_SWIGLU_RHT) return VQ2_ERR_ARG;
  if (!a.perm || !a.sign) return VQ2_ERR_ARG;
  if (a.hb < 64 || a.hb > 2048 || (a.hb & (a.hb - 1)) != 0 || a.n % a.hb != 0) return VQ2_ERR_SHAPE;
  if (a.x_mode == VQ2_ACT_SWIGLU_RHT && a.x_dtype != VQ2_F32) return VQ2_ERR_DTYPE;
  return VQ2_OK;
}

int run_gemv(GemvArgs a, int64_t total_rows, bool res, int val_dtype, cudaStream_t st, void* ws, int64_t ws_bytes) {
  const int lpr = pick_lpr(a.n / 8);
  if (lpr == 0) return VQ2_ERR_SHAPE;
  if ((int64_t)xs_len(a.n) * 4 > kMaxXsBytes) return VQ2_ERR_SHAPE;  // n <= 19264
  const int st_act = check_act(a);
  if (st_act != VQ2_OK) return st_act;
  // Tensor cores from 8 activation rows, or from 2 when the matrices are tall enough to fill
  // the GPU with 128-row items (measured: lm_head at M = 4 is faster there than on CUDA cores).
  const bool tc = a.M >= kTcMinRows || (a.M >= 2 && total_rows >= kTcTallRows);
  if (tc && a.nprob > 0 && !a.argmax && ws != nullptr && ws_bytes >= gemm_tc_workspace(a.M, a.n)) {
    // batched: decode into tensor-core MMAs -- tcgen05 / TMEM when the 128-row tiles fill the
    // GPU, else the split-K mma.sync kernel
    int r = run_gemm_umma(a, res, val_dtype, ws, ws_bytes, st);
    if (r != -1) return r;
    r = run_gemm_tc(a, res, val_dtype, ws, st);
    if (r != -1) return r;
  }
  if (a.comb_w != nullptr) {  // fused combine: expert-indexed, 2 bpw, one activation row (MoE down)
    if (a.nprob > 0 || res || a.M != 1 || a.argmax) return VQ2_ERR_ARG;
    // two rows per warp (as launch_rw chooses for expert-indexed problems)
    if (val_dtype == VQ2_F16) return launch_comb<2, __half>(a, lpr, st);
    if (val_dtype == VQ2_BF16) return launch_comb<2, __nv_bfloat16>(a, lpr, st);
    return VQ2_ERR_DTYPE;
  }
  const int mt = pick_mt(a.M, a.n);
  if (val_dtype == VQ2_F16)
    return res ? launch_epi<true, __half>(a, total_rows, lpr, mt, st) : launch_epi<false, __half>(a, total_rows, lpr, mt, st);
  if (val_dtype == VQ2_BF16)
    return res ? launch_epi<true, __nv_bfloat16>(a, total_rows, lpr, mt, st)
               : launch_epi<false, __nv_bfloat16>(a, total_rows, lpr, mt, st);
  return VQ2_ERR_DTYPE;
}

}  // namespace vq2

static bool dtype_ok(int d) { return d == VQ2_F32 || d == VQ2_F16 || d == VQ2_BF16; }

extern "C" int64_t vq2_gemv_workspace(int64_t M, int64_t n) {
  if (M <= 0 || n <= 0) return -1;
  return M >= 2 ? vq2::gemm_tc_workspace(M, n) : 0;
}

extern "C" int vq2_gemv_multi(const void* x, int x_dtype, int x_mode, int64_t M, int64_t x_row_stride,
                              const int32_t* perm, const int8_t* sign, int64_t hb, float rot_scale, int64_t P,
                              const int16_t* const* idx0, const uint8_t* const* idx1, const int64_t* out,
                              const void* const* scale, const void* cb0, const void* cb1, int val_dtype,
                              void* const* y, int y_dtype, int64_t y_row_stride, int64_t n, float rs,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace vq2;
  if (!x || !idx0 || !out || !scale || !y || !cb0) return VQ2_ERR_ARG;
  if (P <= 0 || P > kMaxProbs) return VQ2_ERR_SHAPE;
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return VQ2_ERR_DTYPE;
  if (M <= 0 || n <= 0 || n % 64 != 0 || n > INT32_MAX || M > INT32_MAX) return VQ2_ERR_SHAPE;
  const int64_t xrow = x_mode == VQ2_ACT_SWIGLU_RHT ? 2 * n : n;
  if (x_row_stride < xrow) return VQ2_ERR_SHAPE;
  if (!aligned(cb0, 16) || (cb1 && !aligned(cb1, 16))) return VQ2_ERR_ALIGN;
  const bool res = idx1 != nullptr && idx1[0] != nullptr;
  if (res != (cb1 != nullptr)) return VQ2_ERR_ARG;
  GemvArgs a{};
  int64_t total_rows = 0, max_out = 0;
  for (int p = 0; p < P; ++p) {
    if (!idx0[p] || !scale[p] || !y[p]) return VQ2_ERR_ARG;
    if (res && !idx1[p]) return VQ2_ERR_ARG;
    if (!res && idx1 && idx1[p]) return VQ2_ERR_ARG;
    if (out[p] <= 0 || out[p] > INT32_MAX) return VQ2_ERR_SHAPE;
    if (!aligned(idx0[p], 16) || (res && !aligned(idx1[p], 8))) return VQ2_ERR_ALIGN;
    a.p_idx0[p] = idx0[p];
    a.p_idx1[p] = res ? idx1[p] : nullptr;
    a.p_scale[p] = scale[p];
    a.p_y[p] = y[p];
    a.p_out[p] = (int)out[p];
    total_rows += out[p];
    max_out = out[p] > max_out ? out[p] : max_out;
  }
  if (y_row_stride < max_out && M > 1) return VQ2_ERR_SHAPE;
  a.nprob = (int)P;
  a.x = x; a.x_dtype = x_dtype; a.x_mode = x_mode; a.x_row_stride = x_row_stride; a.x_k_stride = 0; a.x_k_div = 1;
  a.perm = perm; a.sign = sign; a.hb = (int)hb; a.rot_scale = rot_scale;
  a.M = (int)M; a.cb0 = cb0; a.cb1 = cb1; a.y_dtype = y_dtype; a.y_row_stride = y_row_stride;
  a.n = (int)n; a.rs = rs; a.K = 1; a.out = (int)max_out;
  return run_gemv(a, total_rows, res, val_dtype, static_cast<cudaStream_t>(stream), workspace, workspace_bytes);
}

extern "C" int vq2_gemv(const void* xr, int x_dtype, int64_t M, int64_t x_row_stride, const int16_t* idx0,
                        const uint8_t* idx1, const void* cb0, const void* cb1, const void* scale, int val_dtype,
                        void* y, int y_dtype, int64_t y_row_stride, int64_t out, int64_t n, float rs,
                        void* workspace, int64_t workspace_bytes, void* stream) {
  if (!xr || !idx0 || !cb0 || !scale || !y) return VQ2_ERR_ARG;
  if ((idx1 == nullptr) != (cb1 == nullptr)) return VQ2_ERR_ARG;
  if (out <= 0) return VQ2_ERR_SHAPE;
  if (y_row_stride < out) return VQ2_ERR_SHAPE;
  void* yp[1] = {y};
  const void* sp[1] = {scale};
  const int16_t* i0p[1] = {idx0};
  const uint8_t* i1p[1] = {idx1};
  const int64_t op[1] = {out};
  return vq2_gemv_multi(xr, x_dtype, VQ2_ACT_ROTATED, M, x_row_stride, nullptr, nullptr, 0, 1.f, 1, i0p,
                        idx1 ? i1p : nullptr, op, sp, cb0, cb1, val_dtype, yp, y_dtype, y_row_stride, n, rs,
                        workspace, workspace_bytes, stream);
}

extern "C" int vq2_moe_gemv(const void* x, int x_dtype, int x_mode, int64_t x_k_stride, int64_t x_k_div,
                            const int32_t* perm, const int8_t* sign, int64_t hb, float rot_scale,
                            const int32_t* e_ids, int64_t K, int64_t num_experts, const int16_t* idx,
                            int64_t idx_e_stride, const void* cb0, const void* scale, int64_t scale_e_stride,
                            int val_dtype, void* y, int y_dtype, int64_t out, int64_t ng, float rs,
                            void* stream) {
  using namespace vq2;
  if (!x || !e_ids || !idx || !cb0 || !scale || !y) return VQ2_ERR_ARG;
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return VQ2_ERR_DTYPE;
  if (K <= 0 || num_experts <= 0 || out <= 0 || ng <= 0 || ng % 8 != 0 || out > INT32_MAX || ng * 8 > INT32_MAX)
    return VQ2_ERR_SHAPE;
  if (x_k_stride < 0 || x_k_div <= 0 || K > INT32_MAX) return VQ2_ERR_SHAPE;
  if (idx_e_stride < out * ng || scale_e_stride < out) return VQ2_ERR_SHAPE;
  if (!aligned(idx, 16) || !aligned(cb0, 16) || idx_e_stride % 8 != 0) return VQ2_ERR_ALIGN;
  GemvArgs a{};
  a.nprob = 0;
  a.x = x; a.x_dtype = x_dtype; a.x_mode = x_mode; a.x_row_stride = 0; a.x_k_stride = x_k_stride;
  a.x_k_div = x_k_div; a.perm = perm; a.sign = sign; a.hb = (int)hb; a.rot_scale = rot_scale; a.M = 1;
  a.idx0 = idx; a.idx1 = nullptr; a.cb0 = cb0; a.cb1 = nullptr; a.scale = scale;
  a.y = y; a.y_dtype = y_dtype; a.y_row_stride = 0; a.y_k_stride = out;
  a.e_ids = e_ids; a.num_experts = num_experts; a.idx_e_stride = idx_e_stride; a.idx1_e_stride = idx_e_stride;
  a.scale_e_stride = scale_e_stride;
  a.out = (int)out; a.n = (int)(ng * 8); a.rs = rs; a.K = (int)K;
  return run_gemv(a, out * K, false, val_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int vq2_gemv_argmax(const void* x, int x_dtype, int x_mode, int64_t M, int64_t x_row_stride,
                               const int32_t* perm, const int8_t* sign, int64_t hb, float rot_scale,
                               const int16_t* idx0, const uint8_t* idx1, const void* cb0, const void* cb1,
                               const void* scale, int val_dtype, int64_t out, int64_t n, float rs, void* y,
                               int y_dtype, int64_t y_row_stride, unsigned long long* best, void* stream) {
  using namespace vq2;
  if (!x || !idx0 || !scale || !cb0 || !best) return VQ2_ERR_ARG;
  if (!dtype_ok(x_dtype) || (y && !dtype_ok(y_dtype))) return VQ2_ERR_DTYPE;
  if (M <= 0 || M > 64 || n <= 0 || n % 64 != 0 || out <= 0 || out > INT32_MAX) return VQ2_ERR_SHAPE;
  if (x_row_stride < (x_mode == VQ2_ACT_SWIGLU_RHT ? 2 * n : n) || (y && M > 1 && y_row_stride < out))
    return VQ2_ERR_SHAPE;
  if (!aligned(cb0, 16) || !aligned(idx0, 16) || (idx1 && !aligned(idx1, 8)) || (cb1 && !aligned(cb1, 16)))
    return VQ2_ERR_ALIGN;
  if ((idx1 != nullptr) != (cb1 != nullptr)) return VQ2_ERR_ARG;
  GemvArgs a{};
  a.nprob = 1;
  a.p_idx0[0] = idx0; a.p_idx1[0] = idx1; a.p_scale[0] = scale; a.p_y[0] = y; a.p_out[0] = (int)out;
  a.x = x; a.x_dtype = x_dtype; a.x_mode = x_mode; a.x_row_stride = x_row_stride; a.x_k_stride = 0; a.x_k_div = 1;
  a.perm = perm; a.sign = sign; a.hb = (int)hb; a.rot_scale = rot_scale;
  a.M = (int)M; a.cb0 = cb0; a.cb1 = cb1; a.y_dtype = y ? y_dtype : VQ2_F32; a.y_row_stride = y_row_stride;
  a.n = (int)n; a.rs = rs; a.K = 1; a.out = (int)out;
  a.argmax = best; a.no_y = (y == nullptr);
  return run_gemv(a, out, idx1 != nullptr, val_dtype, static_cast<cudaStream_t>(stream), nullptr, 0);
}
