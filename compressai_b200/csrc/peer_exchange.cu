// Small all-to-all exchanges over NVLink peer memory for the row-sharded lm_head (greedy decode
// with the vocabulary split across the ranks of one node), in one kernel each:
//   * mode GATHER: every rank contributes `bytes` from src; afterwards dst holds all ranks'
//     contributions in rank order (an all-gather of the ranks' hidden states);
//   * mode MAX_KEYS: every rank contributes n 64-bit greedy-argmax keys of its shard (the value
//     in the high half, 0xffffffff - local row in the low half, as the fused-argmax GEMV writes
//     them); they are rebased to global rows (local row + row_offset) and dst receives the
//     elementwise maximum over the ranks -- the global argmax with ties to the smaller row.
// Protocol (as the MoE combine over peer memory): symmetric buffers of identical layout on every
// rank, [flags: world uint32][slots: 2 parities x world x slot_bytes]; each CTA... here a single
// CTA per call: it writes its contribution into slot [parity][rank] of every peer (posted NVLink
// stores), fences at system scope, publishes the call's sequence number in flag [rank] of every
// peer, waits (bounded, acquire loads of its own flags) for every peer's flag, then reads all
// slots from local memory in rank order. The sequence number lives in local device memory and
// advances once per call; a rank can be at most one call ahead, so two parity slots keep the data
// being read stable. A wait that gives up raises *err (0x400) and the kernel uses what it has.
#include "gemv.cuh"

namespace vq2 {

constexpr int kXchgTimeout = 0x400;
constexpr int kXchgDefaultPolls = 1 << 22;

__global__ void __launch_bounds__(256) peer_exchange_kernel(const void* __restrict__ src, int64_t bytes, int mode,
                                                            int64_t row_offset, uint8_t* const* __restrict__ peers,
                                                            int rank, int world, int64_t slot_bytes,
                                                            int32_t* __restrict__ state, int32_t* err,
                                                            int max_polls, void* __restrict__ dst) {
  __shared__ uint32_t s_e;
  pdl_wait();
  const int tid = threadIdx.x;
  if (tid == 0) s_e = static_cast<uint32_t>(state[0]) + 1u;
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t par = e & 1u;
  const int64_t slots = 4096;  // flags region
  // 1. contribution into slot [par][rank] of every rank (16-byte stores; bytes % 8 == 0)
  if (mode == 0) {
    const int64_t nv = bytes / 8;
    const uint64_t* s8 = static_cast<const uint64_t*>(src);
    for (int64_t v = tid; v < nv; v += blockDim.x) {
      const uint64_t x = s8[v];
      for (int r = 0; r < world; ++r)
        reinterpret_cast<uint64_t*>(peers[r] + slots + (par * world + rank) * slot_bytes)[v] = x;
    }
  } else {
    const int64_t n = bytes / 8;
    const unsigned long long* k = static_cast<const unsigned long long*>(src);
    for (int64_t v = tid; v < n; v += blockDim.x) {
      unsigned long long key = k[v];
      if (key != 0ull) {  // rebase the local row to the global row
        const uint32_t local = 0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull);
        key = (key & 0xffffffff00000000ull) | (0xffffffffu - static_cast<uint32_t>(local + row_offset));
      }
      for (int r = 0; r < world; ++r)
        reinterpret_cast<unsigned long long*>(peers[r] + slots + (par * world + rank) * slot_bytes)[v] = key;
    }
  }
  __syncthreads();
  // 2. publish and wait (one peer per lane of warp 0)
  if (tid < 32) peer_flags_handshake(peers, rank, world, 1, 0, e, max_polls, 2048, err, kXchgTimeout);
  __syncthreads();
  // 3. read all slots from local memory in rank order
  const uint8_t* base = peers[rank] + slots + par * world * slot_bytes;
  if (mode == 0) {
    const int64_t nv = bytes / 8;
    for (int r = 0; r < world; ++r)
      for (int64_t v = tid; v < nv; v += blockDim.x)
        static_cast<uint64_t*>(dst)[r * nv + v] = __ldcg(reinterpret_cast<const unsigned long long*>(base + r * slot_bytes) + v);
  } else {
    const int64_t n = bytes / 8;
    for (int64_t v = tid; v < n; v += blockDim.x) {
      unsigned long long m = 0ull;
      for (int r = 0; r < world; ++r) {
        const unsigned long long x = __ldcg(reinterpret_cast<const unsigned long long*>(base + r * slot_bytes) + v);
        m = x > m ? x : m;
      }
      static_cast<unsigned long long*>(dst)[v] = m;
    }
  }
  __syncthreads();
  if (tid == 0) state[0] = static_cast<int32_t>(e);
}

}  // namespace vq2

extern "C" int64_t vq2_peer_exchange_buffer_bytes(int64_t max_bytes, int64_t world) {
  if (max_bytes <= 0 || world < 2 || world > 1024) return -1;
  return 4096 + 2 * world * ((max_bytes + 255) / 256 * 256);
}

extern "C" int vq2_peer_exchange(const void* src, int64_t bytes, int mode, int64_t row_offset,
                                 void* const* peers_dev, int rank, int world, int64_t max_bytes, int32_t* state,
                                 int32_t* err, int64_t max_polls, void* dst, void* stream) {
  using namespace vq2;
  if (!src || !peers_dev || !state || !dst) return VQ2_ERR_ARG;
  if (mode != 0 && mode != 1) return VQ2_ERR_ARG;
  if (world < 2 || world > 1024 || rank < 0 || rank >= world) return VQ2_ERR_ARG;
  if (bytes <= 0 || bytes % 8 != 0 || bytes > max_bytes) return VQ2_ERR_SHAPE;
  if (!aligned(src, 8) || !aligned(dst, 8)) return VQ2_ERR_ALIGN;
  const int polls = max_polls > 0 ? (int)(max_polls < INT32_MAX ? max_polls : INT32_MAX) : kXchgDefaultPolls;
  const int64_t slot = (max_bytes + 255) / 256 * 256;
  return launch_kernel(peer_exchange_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), src, bytes,
                       mode, row_offset, reinterpret_cast<uint8_t* const*>(peers_dev), rank, world, slot, state, err,
                       polls, dst);
}
