// Device-resident paging for the T = 1 decode step: the LRU slot decision of reference
// PagedMoEExpert._get_slot (vq2/paged_runtime.py:415-437) runs on the GPU, and missed expert
// records are read by the SMs straight from the pinned host image (zero-copy over PCIe) into
// their slots, so a decode step (router -> LRU -> fetch -> expert FFN, per layer) needs no host
// round trip and can be captured in one CUDA graph.
//
// LRU state of one layer, one int32 array (initialised by the host, see vq2_lru_state_ints):
//   [0] head (least recently used expert, -1 if none)  [1] tail (most recent)  [2] free count
//   [3] hits  [4] misses  [5] capacity  [6] num_experts  [7] error flag
//   [8, 8+E) expert -> slot (-1 absent)  [.., +E) prev  [.., +E) next  [.., +cap) free-slot stack
// The free stack holds range(cap) with the top at the end, so slots are taken in the order of
// Python's list.pop() on list(range(cap)); eviction takes the head (OrderedDict.popitem(last=False)).
#include "gemv.cuh"

namespace vq2 {

constexpr int kLruHdr = 8;

// The decision itself is serial (one thread). The CTA first copies the layer's state into
// shared memory with coalesced loads (when it fits kLruSmemInts), so the ~5 dependent accesses per
// id are shared-memory round trips instead of L2 ones, and copies it back at the end.
constexpr int kLruSmemInts = 12288;  // 48 KB: E up to ~4000 experts per layer

__global__ void __launch_bounds__(256) lru_step_kernel(int32_t* __restrict__ gst, const int32_t* __restrict__ ids,
                                                       int K, int32_t* __restrict__ slots,
                                                       int32_t* __restrict__ miss) {
  extern __shared__ int32_t sst[];
  pdl_wait();
  const int64_t nints = kLruHdr + 3 * (int64_t)gst[6] + gst[5];  // header: capacity, experts
  const bool in_smem = nints <= kLruSmemInts;
  int32_t* st = gst;
  if (in_smem) {
    for (int i = threadIdx.x; i < nints; i += blockDim.x) sst[i] = gst[i];
    __syncthreads();
    st = sst;
  }
  if (threadIdx.x == 0) {
    const int E = st[6];
    int32_t* e2s = st + kLruHdr;
    int32_t* prv = e2s + E;
    int32_t* nxt = prv + E;
    int32_t* fre = nxt + E;
    int head = st[0], tail = st[1], nfree = st[2], hits = st[3], misses = st[4], err = st[7];
    auto unlink = [&](int x) {
      const int p = prv[x], n = nxt[x];
      if (p >= 0) nxt[p] = n; else head = n;
      if (n >= 0) prv[n] = p; else tail = p;
    };
    auto append = [&](int x) {
      prv[x] = tail;
      nxt[x] = -1;
      if (tail >= 0) nxt[tail] = x; else head = x;
      tail = x;
    };
    int nm = 0;
    for (int k = 0; k < K; ++k) {
      const int e = ids[k];
      if (e < 0 || e >= E) {  // not an expert of this pool: contributes nothing
        slots[k] = -1;
        continue;
      }
      int s = e2s[e];
      if (s >= 0) {
        ++hits;
        unlink(e);
        append(e);
      } else {
        ++misses;
        if (nfree > 0) {
          s = fre[--nfree];
        } else if (head >= 0) {
          const int old = head;
          unlink(old);
          s = e2s[old];
          e2s[old] = -1;
          for (int j = 0; j < k; ++j)  // a slot still needed by this step must not be reused
            if (slots[j] == s) err = 1;
        } else {
          err = 1;  // capacity 0
          slots[k] = -1;
          continue;
        }
        e2s[e] = s;
        append(e);
        miss[1 + nm] = e;
        miss[1 + K + nm] = s;
        ++nm;
      }
      slots[k] = s;
    }
    miss[0] = nm;
    st[0] = head; st[1] = tail; st[2] = nfree; st[3] = hits; st[4] = misses; st[7] = err;
  }
  if (in_smem) {
    __syncthreads();
    for (int i = threadIdx.x; i < nints; i += blockDim.x) gst[i] = sst[i];
  }
}

// Copy the missed records (miss list of lru_step_kernel) from the host image into their slots:
// blockIdx.y = miss index, blockIdx.x = 16 KB piece of the record, 16-byte loads and stores.
__global__ void __launch_bounds__(256) fetch_records_kernel(const uint8_t* __restrict__ image,
                                                            const int64_t* __restrict__ rec_off, int64_t rec,
                                                            uint8_t* __restrict__ pool, int64_t capacity,
                                                            const int32_t* __restrict__ miss, int K,
                                                            int64_t num_experts) {
  pdl_wait();
  const int m = blockIdx.y;
  if (m >= miss[0]) return;
  const int e = miss[1 + m], s = miss[1 + K + m];
  if (e < 0 || e >= num_experts || s < 0 || s >= capacity) return;
  const uint4* src = reinterpret_cast<const uint4*>(image + rec_off[e]);
  uint4* dst = reinterpret_cast<uint4*>(pool + (int64_t)s * rec);
  const int64_t nv = rec / 16, v0 = (int64_t)blockIdx.x * 1024, v1 = min(nv, v0 + 1024);
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
}

}  // namespace vq2

extern "C" int64_t vq2_lru_state_ints(int64_t num_experts, int64_t capacity) {
  if (num_experts <= 0 || capacity <= 0) return -1;
  return vq2::kLruHdr + 3 * num_experts + capacity;
}

extern "C" int vq2_lru_step(int32_t* state, const int32_t* ids, int64_t K, int32_t* slots, int32_t* miss,
                            void* stream) {
  if (!state || !ids || !slots || !miss) return VQ2_ERR_ARG;
  if (K <= 0 || K > 64) return VQ2_ERR_SHAPE;
  static int attr_done[64] = {};  // per device: 48 KB of dynamic shared memory for the state copy
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    const cudaError_t e = cudaFuncSetAttribute(vq2::lru_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               vq2::kLruSmemInts * 4);
    if (e != cudaSuccess) { vq2::set_last_cuda_error(e); return VQ2_ERR_LAUNCH; }
    attr_done[dev & 63] = 1;
  }
  return vq2::launch_kernel(vq2::lru_step_kernel, dim3(1), dim3(256), (size_t)vq2::kLruSmemInts * 4,
                            static_cast<cudaStream_t>(stream), state, ids, static_cast<int>(K), slots, miss);
}

extern "C" int vq2_fetch_records(const void* image_dev, const int64_t* rec_off, int64_t rec_bytes, void* pool,
                                 int64_t capacity, const int32_t* miss, int64_t K, int64_t num_experts,
                                 void* stream) {
  if (!image_dev || !rec_off || !pool || !miss) return VQ2_ERR_ARG;
  if (K <= 0 || K > 64 || rec_bytes <= 0 || capacity <= 0 || num_experts <= 0) return VQ2_ERR_SHAPE;
  if (rec_bytes % 16 != 0 || !vq2::aligned(image_dev, 16) || !vq2::aligned(pool, 16)) return VQ2_ERR_ALIGN;
  const int64_t pieces = (rec_bytes / 16 + 1023) / 1024;
  return vq2::launch_kernel(vq2::fetch_records_kernel, dim3(static_cast<unsigned>(pieces), static_cast<unsigned>(K)),
                            dim3(256), 0, static_cast<cudaStream_t>(stream), static_cast<const uint8_t*>(image_dev),
                            rec_off, rec_bytes, static_cast<uint8_t*>(pool), capacity, miss, static_cast<int>(K),
                            num_experts);
}

extern "C" int vq2_host_device_pointer(const void* host, void** device_ptr) {
  if (!host || !device_ptr) return VQ2_ERR_ARG;
  *device_ptr = nullptr;
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0);
  if (e != cudaSuccess || d == nullptr) {
    cudaGetLastError();  // not page-locked or not mapped: report, do not leave the error pending
    vq2::set_last_cuda_error(e);
    return VQ2_ERR_ARG;
  }
  *device_ptr = d;
  return VQ2_OK;
}
