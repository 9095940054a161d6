// Fused routed-expert FFN of one MoE layer for decode-sized batches (T * top_k <= 64): the gate_up
// GEMV (input RHT fused), the down GEMV (SwiGLU + RHT fused) and the routing-weighted combine in
// ONE persistent launch instead of four (compaction, gate_up, down, combine).
//
// Work items, handed out in this order by an atomic counter:
//   [0, np * RBG)            gate_up rows block rb of problem k (RPC_G rows each)
//   [np * RBG, + np * RBD)   down rows block rb of problem k (RPC_D rows), after all of k's gate_up
//   [.., + T)                combine of token t, after all of t's down items
// A CTA only waits on items handed out before its own, and those are held by CTAs that are
// already running and never wait on later items, so the waits always end; each is still bounded
// (kWaitPolls polls), after which the CTA records a timeout, skips the item and carries on.
// Completion is published with the split-K semaphore pattern: __syncthreads, then one thread
// fences and increments the item's counter; the waiter spins on an acquire load, then
// __syncthreads, and reads the producer's fp32 rows from L2.
// The counters live at the start of the workspace; the last CTA to finish resets them to zero,
// so they are zero at every launch once they were zero at the first.
//
// Arithmetic per output row and per combined element is the same as the unfused kernels' (same
// lanes per row, same FMA and shuffle-reduction order), so both paths give identical results.
// Semantics: reference PagedMoEExpert.forward (vq2/paged_runtime.py:491-511) and
// PackedMoEExpertUniversal.forward (vq2/load_and_test_full_35b.py:53-95).
#include <atomic>

#include "gemv_dev.cuh"

namespace vq2 {

constexpr int kFusedMaxP = kIdsByValue;  // 64 (token, expert) problems
constexpr int kFusedRW = 4;              // rows per warp-load slot
constexpr int kWaitPolls = 1 << 20;      // ~0.1-1 s at 64 ns naps: far beyond any real wait
constexpr int kFusedTimeout = 0x100;     // raised into the caller's status word on a timed-out wait
constexpr int kCtrQueue = 0, kCtrFinished = 1, kCtrTimeouts = 2, kCtrGu = 8, kCtrDn = 8 + kFusedMaxP;


__device__ __forceinline__ int ld_acquire(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0: wait until *c >= target (bounded); returns false on timeout.
__device__ bool wait_count(const int32_t* c, int target) {
  for (int it = 0; it < kWaitPolls; ++it) {
    if (ld_acquire(c) >= target) return true;
    __nanosleep(64);
  }
  return false;
}

// Rows block rb of one expert matrix: y[r] = scale[r] * sum_g dot(cb0[idx[r, g]], xs[8g:8g+8]),
// RW x (32 / LPR) rows per warp, LPR lanes per row (the GEMV kernel's decomposition at M = 1).
template <int LPR, typename TV>
struct RowsGemv {
  static constexpr int RPL = 32 / LPR, RPW = kFusedRW * RPL, RPC = 8 * RPW;

  __device__ static void load(const int16_t* idx, int rows, int ng, int rb, int chunk, uint4 (&iv)[kFusedRW],
                              uint64_t pol) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane / LPR, li = lane % LPR;
    const int g0 = (chunk * LPR + li) * 8;
#pragma unroll
    for (int rw = 0; rw < kFusedRW; ++rw) {
      const int r = rb * RPC + warp * RPW + rw * RPL + sub;
      iv[rw] = r < rows ? ld_stream_u4(idx + (int64_t)r * ng + g0, pol) : make_uint4(0, 0, 0, 0);
    }
  }

  // iv holds chunk 0's indices on entry (prefetched); later chunks are loaded here.
  __device__ static void run(const int16_t* idx, const TV* scale, int rows, int ng, int rb, const float* xs,
                             const uint4* cb0, float* y, uint4 (&iv)[kFusedRW], uint64_t pol_s, uint64_t pol_c) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane / LPR, li = lane % LPR;
    const int chunks = ng / (8 * LPR);
    float acc[kFusedRW];
#pragma unroll
    for (int rw = 0; rw < kFusedRW; ++rw) acc[rw] = 0.f;
    for (int c = 0; c < chunks; ++c) {
      if (c > 0) load(idx, rows, ng, rb, c, iv, pol_s);
      const int g0 = (c * LPR + li) * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int p = xs_pos(g0 + j, 0);
        const float4 lo = *reinterpret_cast<const float4*>(xs + p);
        const float4 hi = *reinterpret_cast<const float4*>(xs + p + 4);
        const float xv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int rw = 0; rw < kFusedRW; ++rw) {
          const uint32_t w32 = (&iv[rw].x)[j >> 1];
          const uint32_t code = (j & 1) ? (w32 >> 16) : (w32 & 0xffffu);
          float wv[8];
          decode8<TV>(ld_cb_u4(cb0 + code, pol_c), wv);
          float s = acc[rw];
#pragma unroll
          for (int t = 0; t < 8; ++t) s = fmaf(wv[t], xv[t], s);
          acc[rw] = s;
        }
      }
    }
#pragma unroll
    for (int rw = 0; rw < kFusedRW; ++rw)
#pragma unroll
      for (int off = LPR / 2; off > 0; off >>= 1) acc[rw] += __shfl_xor_sync(0xffffffffu, acc[rw], off);
    if (li == 0) {
#pragma unroll
      for (int rw = 0; rw < kFusedRW; ++rw) {
        const int r = rb * RPC + warp * RPW + rw * RPL + sub;
        if (r < rows) y[r] = acc[rw] * to_f32<TV>(scale[r]);
      }
    }
  }
};

template <int LG, int LD, typename TV>
__global__ void __launch_bounds__(256, 2) moe_fused_kernel(const MoeFusedArgs a) {
  using G = RowsGemv<LG, TV>;
  using D = RowsGemv<LD, TV>;
  extern __shared__ __align__(16) float smem[];
  __shared__ int s_pid[kFusedMaxP], s_eid[kFusedMaxP], s_cidx[kFusedMaxP];
  __shared__ int s_np, s_item, s_ok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_in = a.ng_gu * 8, n_mid = a.ng_dn * 8;
  float* xs = smem;
  float* scratch = smem + xs_len(n_in > n_mid ? n_in : n_mid);
  const uint4* cb0 = static_cast<const uint4*>(a.cb0);
  const uint64_t pol_s = policy_evict_first(), pol_c = policy_evict_last();
  const int RBG = (a.gu_rows + G::RPC - 1) / G::RPC, RBD = (a.dn_rows + D::RPC - 1) / D::RPC;
  // activation sources: token rows of h (gate_up input, RHT) and problem rows of the gate|up
  // output (down input, SwiGLU + RHT)
  const ActSrc src_in = {a.h, a.h_dtype, VQ2_ACT_RHT, n_in, a.hb_in, n_in, a.perm_in, a.sign_in, a.scale_in};
  const ActSrc src_mid = {a.y_gu, VQ2_F32, VQ2_ACT_SWIGLU_RHT, n_mid, a.hb_mid, a.gu_rows, a.perm_mid, a.sign_mid,
                          a.scale_mid};

  // Problems whose expert is in the pool, in order (warp 0, two ballots of 32).
  auto build_list = [&]() {
    if (warp == 0) {
      int base = 0;
#pragma unroll
      for (int p0 = 0; p0 < kFusedMaxP; p0 += 32) {
        const int p = p0 + lane;
        const int id = p < a.P ? (a.ids ? a.ids[p] : a.iv.v[p]) : -1;
        const bool keep = p < a.P && id >= 0 && id < a.num_experts;
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        if (keep) {
          s_pid[pos] = p;
          s_eid[pos] = id;
        }
        if (p < a.P) s_cidx[p] = keep ? pos : -1;
        base += __popc(m);
      }
      if (lane == 0) s_np = base;
    }
  };
  if (!a.ids) build_list();
  pdl_wait();
  if (a.ids) build_list();
  if (tid == 0) s_item = atomicAdd(&a.ctr[kCtrQueue], 1);
  __syncthreads();
  const int np = s_np;
  const int n_gu = np * RBG, n_dn = np * RBD, n_items = n_gu + n_dn + a.T;
  auto item_src = [&](int it, const int16_t*& idx, int& rows, int& ng, int& rb, int& k) {
    const bool gu = it < n_gu;
    const int q = gu ? it : it - n_gu;
    k = gu ? q / RBG : q / RBD;
    rb = gu ? q - k * RBG : q - k * RBD;
    const uint8_t* r = a.pool + (int64_t)s_eid[k] * a.rec;
    idx = reinterpret_cast<const int16_t*>(gu ? r : r + a.off_di);
    rows = gu ? a.gu_rows : a.dn_rows;
    ng = gu ? a.ng_gu : a.ng_dn;
  };
  auto prefetch = [&](int it, uint4 (&iv)[kFusedRW]) {
    if (it >= n_gu + n_dn) return;
    const int16_t* idx;
    int rows, ng, rb, k;
    item_src(it, idx, rows, ng, rb, k);
    if (it < n_gu) G::load(idx, rows, ng, rb, 0, iv, pol_s);
    else D::load(idx, rows, ng, rb, 0, iv, pol_s);
  };

  int item = s_item;
  uint4 iv[kFusedRW];
  prefetch(item, iv);
  int staged = INT32_MIN;  // token t (gate_up input) or -(k + 1) (down input of problem k)
  while (item < n_items) {
    __syncthreads();  // s_item consumed by every thread
    if (tid == 0) s_item = atomicAdd(&a.ctr[kCtrQueue], 1);
    __syncthreads();
    const int next = s_item;
    uint4 nv[kFusedRW];
    prefetch(next, nv);  // weights are constant: no dependency on earlier items

    if (item < n_gu + n_dn) {
      const bool gu = item < n_gu;
      const int16_t* idx;
      int rows, ng, rb, k;
      item_src(item, idx, rows, ng, rb, k);
      const int p = s_pid[k];
      const uint8_t* rec = a.pool + (int64_t)s_eid[k] * a.rec;
      if (!gu) {  // the down input needs all of problem k's gate_up rows
        if (tid == 0) {
          s_ok = 1;
          if (!wait_count(a.ctr + kCtrGu + k, RBG)) {
            s_ok = 0;
            atomicAdd(a.ctr + kCtrTimeouts, 1);
            if (a.err) atomicMax(a.err, kFusedTimeout);
          }
        }
        __syncthreads();
      }
      const int key = gu ? p / a.K : -(k + 1);
      if (key != staged) {
        __syncthreads();
        if (gu) stage_activations<1>(src_in, (int64_t)(p / a.K) * n_in, 1, xs, xs_len(n_in), scratch);
        else stage_activations<1>(src_mid, (int64_t)p * a.gu_rows, 1, xs, xs_len(n_mid), scratch);
        __syncthreads();
        staged = key;
      }
      if (gu) {
        G::run(idx, reinterpret_cast<const TV*>(rec + a.off_gs), rows, ng, rb, xs, cb0, a.y_gu + (int64_t)p * a.gu_rows,
               iv, pol_s, pol_c);
      } else if (s_ok) {
        D::run(idx, reinterpret_cast<const TV*>(rec + a.off_ds), rows, ng, rb, xs, cb0, a.y_dn + (int64_t)p * a.dn_rows,
               iv, pol_s, pol_c);
      }
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        atomicAdd(a.ctr + (gu ? kCtrGu : kCtrDn) + k, 1);
      }
    } else {  // combine of token t: out[t] = sum_j w[t, j] * y_dn[t * K + j] over computed problems
      const int t = item - n_gu - n_dn;
      if (tid == 0) {
        s_ok = 1;
        for (int j = 0; j < a.K; ++j) {
          const int k = s_cidx[t * a.K + j];
          if (k >= 0 && !wait_count(a.ctr + kCtrDn + k, RBD)) {
            s_ok = 0;
            atomicAdd(a.ctr + kCtrTimeouts, 1);
            if (a.err) atomicMax(a.err, kFusedTimeout);
            break;
          }
        }
      }
      __syncthreads();
      const int H = a.dn_rows;
      if (s_ok) {
        for (int c = tid; c < H; c += blockDim.x) {
          float s = 0.f;
          for (int j = 0; j < a.K; ++j) {
            const int p = t * a.K + j;
            if (s_cidx[p] < 0) continue;  // problem not computed here
            s = fmaf(a.w[p], __ldcg(a.y_dn + (int64_t)p * H + c), s);
          }
          const int64_t o = (int64_t)t * H + c;
          if (a.out_dtype == VQ2_F16) static_cast<__half*>(a.out)[o] = __float2half_rn(s);
          else if (a.out_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(s);
          else static_cast<float*>(a.out)[o] = s;
        }
      }
    }
    item = next;
#pragma unroll
    for (int rw = 0; rw < kFusedRW; ++rw) iv[rw] = nv[rw];
  }
  pdl_trigger();
  // The last CTA out resets the counters for the next launch (every other CTA is past its last
  // counter access by then).
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(a.ctr + kCtrFinished, 1) == (int)gridDim.x - 1) {
      for (int k = 0; k < np; ++k) {
        a.ctr[kCtrGu + k] = 0;
        a.ctr[kCtrDn + k] = 0;
      }
      a.ctr[kCtrQueue] = 0;
      a.ctr[kCtrFinished] = 0;
      __threadfence();
    }
  }
}

constexpr int64_t kFusedCtrBytes = 1024;

// The fused path has instantiations for the 35B-A3B expert shape (gate_up input 2048 -> 32 lanes
// per row, down input 512 -> 8, as the GEMV picks them), P <= 64 and fp16/bf16 weights.
bool moe_fused_eligible(const MoeFusedArgs& a, int val_dtype) {
  return a.P >= 1 && a.P <= kFusedMaxP && a.T >= 1 && a.ng_gu == 256 && a.ng_dn == 64 && a.gu_rows == 2 * 8 * a.ng_dn &&
         (val_dtype == VQ2_F16 || val_dtype == VQ2_BF16) && a.hb_in >= 64 && a.hb_mid >= 64;
}

int moe_fused_ffn(const MoeFusedArgs& a, int val_dtype, cudaStream_t st) {
  if (!moe_fused_eligible(a, val_dtype)) return VQ2_ERR_SHAPE;
  auto kern = val_dtype == VQ2_F16 ? moe_fused_kernel<32, 8, __half> : moe_fused_kernel<32, 8, __nv_bfloat16>;
  const size_t smem = ((size_t)xs_len(2048) + kScratchFloats) * sizeof(float);
  static std::atomic<uint64_t> done{0};
  static std::atomic<int> bps{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done.load() & bit)) {
    int nb = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, moe_fused_kernel<32, 8, __half>, 256, smem);
    bps.store(nb > 0 ? nb : 1);
    done.fetch_or(bit);
  }
  const int RBG = (a.gu_rows + RowsGemv<32, __half>::RPC - 1) / RowsGemv<32, __half>::RPC;
  const int RBD = (a.dn_rows + RowsGemv<8, __half>::RPC - 1) / RowsGemv<8, __half>::RPC;
  const int64_t items = (int64_t)a.P * (RBG + RBD) + a.T;
  const int64_t cap = (int64_t)sm_count() * bps.load();
  const int grid = (int)(items < cap ? items : cap);
  return launch_kernel(kern, dim3(grid), dim3(256), smem, st, a);
}

}  // namespace vq2
