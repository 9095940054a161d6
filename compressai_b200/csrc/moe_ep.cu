// Expert-parallel combine fused with the cross-GPU reduction: the routing-weighted sum of this
// rank's expert outputs and the sum over ranks in ONE kernel over NVLink peer memory, replacing
// combine -> NCCL all_reduce(SUM) -> cast.
//
// Every rank holds an identical symmetric buffer (peer-mapped; the device array `peers` has each
// rank's base address): [flags: world x kPeerFlagStride uint32][slots: 2 parities x world ranks x T_max x H
// fp32]. The [T, H] output is split into contiguous float4 ranges, one per CTA:
//   1. CTA b computes its range of this rank's partial (sum_j w[t, j] * y[t*k + j] over local
//      problems) and stores it into slot [parity][rank] of EVERY rank's buffer (posted NVLink
//      writes; no remote reads anywhere);
//   2. the lanes of warp 0, one per peer, fence at system scope, publish the call's sequence
//      number into flag [rank][b] of their peer (release stores) and wait (bounded; acquire loads
//      of the local flags) until that peer's flag [q][b] has it;
//   3. the CTA adds slots [parity][0..world) of its range from LOCAL memory in rank order (the
//      same values in the same order on every rank) and writes the output in its dtype.
// The sequence number lives in local device memory (state[0]); the last CTA to finish advances
// it (state[1] counts finished CTAs). Every rank makes the same calls, so the numbers agree; a
// rank can run at most one call ahead of another (it needs the others' flags of the current
// call), so two parity slots keep the data of the call being read stable. A wait that gives up
// raises *err and the CTA writes what it has; nothing traps.
#include <algorithm>

#include "gemv.cuh"

namespace vq2 {

__global__ void __launch_bounds__(256) moe_combine_peer_kernel(const float* __restrict__ y, const float* __restrict__ w,
                                                               const int32_t* __restrict__ ids, int64_t num_experts,
                                                               int T, int K, int H, uint8_t* const* __restrict__ peers,
                                                               int rank, int world, int64_t part_off,
                                                               int64_t slot_bytes, int32_t* __restrict__ state,
                                                               int32_t* err, int max_polls, void* out,
                                                               int out_dtype) {
  __shared__ uint32_t s_e;
  pdl_wait();
  const int b = blockIdx.x, nb = gridDim.x, tid = threadIdx.x;
  if (tid == 0) s_e = static_cast<uint32_t>(state[0]) + 1u;
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t par = e & 1u;
  const int64_t nv = (int64_t)T * H / 4, per = (nv + nb - 1) / nb, v0 = (int64_t)b * per, v1 = min(nv, v0 + per);
  // 1. local partial of this CTA's range, pushed into slot [par][rank] of every rank
  for (int64_t v = v0 + tid; v < v1; v += blockDim.x) {
    const int64_t el = v * 4, t = el / H, c = el - t * H;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < K; j0 += 8) {  // 8 problems' loads in flight, summed in problem order
      bool ok[8];
      float wp[8];
      float4 yv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t p = t * K + j0 + k;
        const int32_t id = j0 + k < K ? (ids ? ids[p] : 0) : -1;  // ids null: every problem local
        ok[k] = id >= 0 && id < num_experts;  // else computed on another rank
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t p = t * K + j0 + k;
        wp[k] = ok[k] ? (w ? w[p] : 1.f) : 0.f;  // w null: weight 1 (y is an already combined partial)
        yv[k] = ok[k] ? *reinterpret_cast<const float4*>(y + p * H + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (!ok[k]) continue;
        s.x = fmaf(wp[k], yv[k].x, s.x);
        s.y = fmaf(wp[k], yv[k].y, s.y);
        s.z = fmaf(wp[k], yv[k].z, s.z);
        s.w = fmaf(wp[k], yv[k].w, s.w);
      }
    }
    for (int r = 0; r < world; ++r)
      reinterpret_cast<float4*>(peers[r] + part_off + (par * world + rank) * slot_bytes)[v] = s;
  }
  __syncthreads();
  // 2. publish, then wait for every peer's range b of this call
  if (tid < 32) peer_flags_handshake(peers, rank, world, kPeerFlagStride, b, e, max_polls, kPeerTightPolls, err,
                                     kPeerTimeout);
  __syncthreads();
  // 3. sum of all ranks' ranges from local memory, in rank order
  const uint8_t* base = peers[rank] + part_off + par * world * slot_bytes;
  for (int64_t v = v0 + tid; v < v1; v += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(base + r * slot_bytes) + v);
      s.x += x.x;
      s.y += x.y;
      s.z += x.z;
      s.w += x.w;
    }
    const int64_t o = v * 4;
    if (out_dtype == VQ2_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(out) + o) = s;
    } else if (out_dtype == VQ2_F16) {
      __half2* d = reinterpret_cast<__half2*>(static_cast<__half*>(out) + o);
      d[0] = __floats2half2_rn(s.x, s.y);
      d[1] = __floats2half2_rn(s.z, s.w);
    } else {
      __nv_bfloat162* d = reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(out) + o);
      d[0] = __floats2bfloat162_rn(s.x, s.y);
      d[1] = __floats2bfloat162_rn(s.z, s.w);
    }
  }
  // 4. the last CTA out advances the sequence number
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(state + 1, 1) == nb - 1) {
      state[1] = 0;
      state[0] = static_cast<int32_t>(e);
      __threadfence();
    }
  }
}

int64_t peer_flag_bytes(int world) { return ((int64_t)world * kPeerFlagStride * 4 + 4095) / 4096 * 4096; }
int64_t peer_slot_bytes(int64_t max_tokens, int64_t H) { return (max_tokens * H * 4 + 255) / 256 * 256; }

int run_combine_peer(const float* y, const float* w, int64_t T, int top_k, int64_t H, const int32_t* ids,
                     int64_t num_experts, const PeerReduce& pr, void* out, int out_dtype, cudaStream_t st) {
  if (!pr.peers || !pr.epochs || pr.world < 2 || pr.rank < 0 || pr.rank >= pr.world) return VQ2_ERR_ARG;
  if (H % 4 != 0 || T * H * 4 > pr.part_bytes || pr.part_off < peer_flag_bytes(pr.world)) return VQ2_ERR_SHAPE;
  if (!aligned(out, 16) || !aligned(y, 16)) return VQ2_ERR_ALIGN;
  const int64_t nv = T * H / 4;
  const int nb = (int)std::min<int64_t>(kPeerMaxBlocks, std::max<int64_t>(1, (nv + 255) / 256));
  const int polls = pr.max_polls > 0 ? pr.max_polls : kPeerWaitPolls;
  return launch_kernel(moe_combine_peer_kernel, dim3(nb), dim3(256), 0, st, y, w, ids, num_experts, (int)T, top_k,
                       (int)H, pr.peers, pr.rank, pr.world, pr.part_off, pr.part_bytes, pr.epochs, pr.err, polls, out,
                       out_dtype);
}

}  // namespace vq2

extern "C" int64_t vq2_moe_peer_buffer_bytes(int64_t max_tokens, int64_t hidden, int64_t world) {
  if (max_tokens <= 0 || hidden <= 0 || world < 2 || world > 64) return -1;
  return vq2::peer_flag_bytes((int)world) + 2 * world * vq2::peer_slot_bytes(max_tokens, hidden);
}

extern "C" int vq2_moe_expert_ffn_ep(const void* h, int h_dtype, int64_t T, int64_t top_k, const int32_t* ids,
                                     const float* w, const void* pool, int64_t num_experts, int64_t gu_rows,
                                     int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
                                     const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in,
                                     const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid, float scale_mid,
                                     void* workspace, int64_t workspace_bytes, void* const* peers_dev, int rank,
                                     int world, int64_t max_tokens, uint32_t* epochs, int32_t* err,
                                     int64_t max_polls, void* out, int out_dtype, void* stream) {
  if (T <= 0 || top_k <= 0 || gu_rows <= 0 || dn_rows <= 0 || T > max_tokens) return VQ2_ERR_SHAPE;
  if (workspace_bytes < vq2::moe_ffn_workspace(T * top_k, gu_rows, dn_rows)) return VQ2_ERR_ARG;
  if (!peers_dev || !epochs || world < 2 || world > 64) return VQ2_ERR_ARG;
  vq2::PeerReduce pr;
  pr.peers = reinterpret_cast<uint8_t* const*>(peers_dev);
  pr.rank = rank;
  pr.world = world;
  pr.part_off = vq2::peer_flag_bytes(world);
  pr.part_bytes = vq2::peer_slot_bytes(max_tokens, gu_cols * 8);
  pr.epochs = reinterpret_cast<int32_t*>(epochs);
  pr.err = err;
  pr.max_polls = (int)std::min<int64_t>(std::max<int64_t>(max_polls, 0), INT32_MAX);
  return vq2::moe_expert_ffn(h, h_dtype, T, top_k, ids, w, pool, num_experts, gu_rows, gu_cols, dn_rows, dn_cols,
                             cb0, val_dtype, perm_in, sign_in, hb_in, scale_in, perm_mid, sign_mid, hb_mid,
                             scale_mid, workspace, out, out_dtype, static_cast<cudaStream_t>(stream), false, false,
                             nullptr, false, nullptr, nullptr, &pr);
}

extern "C" int vq2_moe_layer_ep(const void* h, int h_dtype, int64_t T, const float* logits, int64_t E, int64_t top_k,
                                const float* shared_gate, int64_t expert_lo, int64_t expert_hi, const void* pool,
                                int64_t pool_rows, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows, int64_t dn_cols,
                                const void* cb0, int val_dtype, const int32_t* perm_in, const int8_t* sign_in,
                                int64_t hb_in, float scale_in, const int32_t* perm_mid, const int8_t* sign_mid,
                                int64_t hb_mid, float scale_mid, void* workspace, int64_t workspace_bytes,
                                void* const* peers_dev, int rank, int world, int64_t max_tokens, uint32_t* epochs,
                                int32_t* err, int64_t max_polls, void* out, int out_dtype, void* stream) {
  if (T <= 0 || T > max_tokens) return VQ2_ERR_SHAPE;
  if (!peers_dev || !epochs || world < 2 || world > 64) return VQ2_ERR_ARG;
  vq2::PeerReduce pr;
  pr.peers = reinterpret_cast<uint8_t* const*>(peers_dev);
  pr.rank = rank;
  pr.world = world;
  pr.part_off = vq2::peer_flag_bytes(world);
  pr.part_bytes = vq2::peer_slot_bytes(max_tokens, gu_cols * 8);
  pr.epochs = reinterpret_cast<int32_t*>(epochs);
  pr.err = err;
  pr.max_polls = (int)std::min<int64_t>(std::max<int64_t>(max_polls, 0), INT32_MAX);
  return vq2::moe_layer(h, h_dtype, T, logits, E, top_k, shared_gate, expert_lo, expert_hi, rank, world, pool,
                        pool_rows, gu_rows, gu_cols, dn_rows, dn_cols, cb0, val_dtype, perm_in, sign_in, hb_in,
                        scale_in, perm_mid, sign_mid, hb_mid, scale_mid, workspace, workspace_bytes, out, out_dtype,
                        static_cast<cudaStream_t>(stream), &pr);
}
