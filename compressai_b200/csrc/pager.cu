// Native executor of one paged MoE step: the copy and compute half of reference
// PagedMoEExpert.forward (vq2/paged_runtime.py:439-568) after the caller's LRU bookkeeping
// (_get_slot, :415-437) has chosen the slots. One C-ABI call issues the record copies of the
// misses on the copy stream (and, for VQ2A-coded containers, one decode launch per 8 records),
// the upload of the slot ids, and the routed-expert FFN, with the events that order them, so
// the host spends a few microseconds per layer instead of a Python call per copy.
#include <cstring>

#include "gemv.cuh"

namespace vq2 {

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return VQ2_OK;
  set_last_cuda_error(e);
  return VQ2_ERR_LAUNCH;
}

constexpr int kPagerGroup = 8;  // coded records per decode launch (4 segments each)

static int page_in(const vq2_paged_layer& L, int64_t rec, int64_t n_miss, const void* const* src,
                   const int64_t* bytes, const int32_t* slot, const int64_t* seg) {
  cudaStream_t cs = static_cast<cudaStream_t>(L.copy_stream);
  uint8_t* pool = static_cast<uint8_t*>(L.pool);
  int s = cuda_status(cudaStreamWaitEvent(cs, static_cast<cudaEvent_t>(L.compute_done), 0));
  if (s != VQ2_OK) return s;
  if (L.index_coding == 0) {
    for (int64_t i = 0; i < n_miss; ++i) {
      s = cuda_status(cudaMemcpyAsync(pool + slot[i] * rec, src[i], bytes[i], cudaMemcpyHostToDevice, cs));
      if (s != VQ2_OK) return s;
    }
  } else {
    // Coded records: the staging buffer has two halves used in turn (the turn counter is shared
    // by every layer on this copy stream); the copies of a group land in one half on the copy
    // stream, the decode stream expands them, and the next copies into that half wait for it, so
    // the copy engine keeps moving records while the SMs decode.
    cudaStream_t ds = static_cast<cudaStream_t>(L.decode_stream);
    const int64_t half = L.stage_bytes / 2;
    int64_t i = 0;
    while (i < n_miss) {  // groups that fit half the staging buffer, at most kPagerGroup records
      int64_t off[kPagerGroup + 1], g = 0, used = 0;
      while (i + g < n_miss && g < kPagerGroup && used + bytes[i + g] <= half) {
        off[g] = used;
        used += (bytes[i + g] + 255) & ~int64_t(255);
        ++g;
      }
      if (g == 0) return VQ2_ERR_SHAPE;  // one record larger than half the staging buffer
      const int turn = static_cast<int>((*L.stage_turn)++ & 1);
      uint8_t* stage = static_cast<uint8_t*>(L.stage) + turn * half;
      cudaEvent_t free_ev = static_cast<cudaEvent_t>(turn ? L.stage_free1 : L.stage_free0);
      s = cuda_status(cudaStreamWaitEvent(cs, free_ev, 0));
      if (s != VQ2_OK) return s;
      int64_t so[4 * kPagerGroup], sb[4 * kPagerGroup], d0[4 * kPagerGroup], sn[4 * kPagerGroup];
      int32_t kd[4 * kPagerGroup];
      for (int64_t r = 0; r < g; ++r) {
        s = cuda_status(cudaMemcpyAsync(stage + off[r], src[i + r], bytes[i + r], cudaMemcpyHostToDevice, cs));
        if (s != VQ2_OK) return s;
        for (int q = 0; q < 4; ++q) {
          const int64_t* e = seg + ((i + r) * 4 + q) * 5;  // src_off, src_bytes, dst_off, n, kind
          if (e[0] < 0 || e[1] < 0 || e[0] + e[1] > bytes[i + r] || e[2] < 0 || e[3] < 0 || e[2] + e[3] > rec)
            return VQ2_ERR_SHAPE;
          so[4 * r + q] = off[r] + e[0];
          sb[4 * r + q] = e[1];
          d0[4 * r + q] = slot[i + r] * rec + e[2];
          sn[4 * r + q] = e[3];
          kd[4 * r + q] = static_cast<int32_t>(e[4]);
        }
      }
      s = cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(L.stage_ready), cs));
      if (s == VQ2_OK) s = cuda_status(cudaStreamWaitEvent(ds, static_cast<cudaEvent_t>(L.stage_ready), 0));
      if (s != VQ2_OK) return s;
      s = ans_launch(stage, half, so, sb, d0, sn, kd, 4 * g, pool, L.capacity * rec, L.status, ds);
      if (s != VQ2_OK) return s;
      s = cuda_status(cudaEventRecord(free_ev, ds));
      if (s != VQ2_OK) return s;
      i += g;
    }
    return cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(L.copy_done), ds));  // decoded
  }
  return cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(L.copy_done), cs));
}

}  // namespace vq2

extern "C" int vq2_paged_moe_step(const vq2_paged_layer* layer, const void* h, int h_dtype, int64_t T, int64_t top_k,
                                  const int32_t* slots, const float* w, int64_t n_miss, const void* const* miss_src,
                                  const int64_t* miss_bytes, const int32_t* miss_slot, const int64_t* miss_seg,
                                  void* workspace, int64_t workspace_bytes, void* out, int out_dtype, void* stream) {
  using namespace vq2;
  if (!layer || !slots || (n_miss > 0 && (!miss_src || !miss_bytes || !miss_slot))) return VQ2_ERR_ARG;
  const vq2_paged_layer& L = *layer;
  if (!L.pool || !L.ids_host || !L.ids_dev || !L.copy_stream || !L.copy_done || !L.compute_done || !L.ids_done)
    return VQ2_ERR_ARG;
  if (L.index_coding != 0 &&
      (L.index_coding != 1 || !L.stage || !L.status || !L.decode_stream || !L.stage_ready || !L.stage_free0 ||
       !L.stage_free1 || !L.stage_turn || (n_miss > 0 && !miss_seg)))
    return VQ2_ERR_ARG;
  if (T <= 0 || top_k <= 0 || n_miss < 0 || L.capacity <= 0) return VQ2_ERR_SHAPE;
  const int64_t P = T * top_k;
  if (P > L.ids_cap) return VQ2_ERR_SHAPE;
  if (workspace_bytes < moe_ffn_workspace(P, L.gu_rows, L.dn_rows)) return VQ2_ERR_ARG;
  const int64_t rec = L.gu_rows * L.gu_cols * 2 + L.gu_rows * 2 + L.dn_rows * L.dn_cols * 2 + L.dn_rows * 2;
  for (int64_t i = 0; i < n_miss; ++i) {
    if (!miss_src[i] || miss_slot[i] < 0 || miss_slot[i] >= L.capacity || miss_bytes[i] <= 0) return VQ2_ERR_SHAPE;
    if (L.index_coding == 0 ? miss_bytes[i] != rec : miss_bytes[i] > L.stage_bytes / 2) return VQ2_ERR_SHAPE;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int s;
  if (n_miss > 0) {
    s = page_in(L, rec, n_miss, miss_src, miss_bytes, miss_slot, miss_seg);
    if (s != VQ2_OK) return s;
    s = cuda_status(cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(L.copy_done), 0));
    if (s != VQ2_OK) return s;
  }
  s = cuda_status(cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(L.compute_done), 0));
  if (s != VQ2_OK) return s;
  // Slot ids: up to 64 travel in the first kernel's launch parameters (a copy on `stream` would
  // queue behind the record copies on the copy engine); more go through the pinned buffer once
  // its previous upload has completed.
  const bool by_value = P <= kIdsByValue;
  if (!by_value) {
    s = cuda_status(cudaEventSynchronize(static_cast<cudaEvent_t>(L.ids_done)));
    if (s != VQ2_OK) return s;
    std::memcpy(L.ids_host, slots, static_cast<size_t>(P) * sizeof(int32_t));
    s = cuda_status(cudaMemcpyAsync(L.ids_dev, L.ids_host, static_cast<size_t>(P) * sizeof(int32_t),
                                    cudaMemcpyHostToDevice, st));
    if (s != VQ2_OK) return s;
    s = cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(L.ids_done), st));
    if (s != VQ2_OK) return s;
  }
  s = moe_expert_ffn(h, h_dtype, T, top_k, by_value ? slots : L.ids_dev, w, L.pool, L.capacity, L.gu_rows,
                     L.gu_cols, L.dn_rows, L.dn_cols, L.cb0, L.val_dtype, L.perm_in, L.sign_in, L.hb_in, L.scale_in,
                     L.perm_mid, L.sign_mid, L.hb_mid, L.scale_mid, workspace, out, out_dtype, st, by_value,
                     /*counters_zeroed=*/true, L.status, /*prefer_fused=*/true);
  if (s != VQ2_OK) return s;
  return cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(L.compute_done), st));
}
