// Routed-expert FFN of one MoE layer as one C-ABI call: gate_up GEMV (input RHT fused), down
// GEMV (SwiGLU + RHT fused), routing-weighted combine -- three launches on one stream, the two
// fp32 intermediates in a caller-provided workspace.
// Semantics: the compute part of reference PagedMoEExpert.forward (vq2/paged_runtime.py:
// 491-511, T > 1 :553-566) and PackedMoEExpertUniversal.forward
// (vq2/load_and_test_full_35b.py:53-95), in fp32 with fp16 storage.
#include <atomic>

#include "gemv.cuh"

namespace vq2 {

// Byte offsets within one expert record. 2 bpw (.vq2m payload): gu idx0 | gu scale | dn idx0 |
// dn scale. 3 bpw (promoted experts, reference tools/build_mixed_b2_container.py:50-80): each
// index entry is idx0 (int16) followed by idx1 (uint8): gu idx0 | gu idx1 | gu scale | dn idx0 |
// dn idx1 | dn scale (1,185,792 bytes at the 35B-A3B shape).
struct RecordLayout {
  int64_t gu_idx, gu_idx1, gu_scale, dn_idx, dn_idx1, dn_scale, bytes;
};

static RecordLayout record_layout(int64_t gr, int64_t gc, int64_t dr, int64_t dc, bool res = false) {
  RecordLayout r;
  r.gu_idx = 0;
  r.gu_idx1 = gr * gc * 2;
  r.gu_scale = r.gu_idx1 + (res ? gr * gc : 0);
  r.dn_idx = r.gu_scale + gr * 2;
  r.dn_idx1 = r.dn_idx + dr * dc * 2;
  r.dn_scale = r.dn_idx1 + (res ? dr * dc : 0);
  r.bytes = r.dn_scale + dr * 2;
  return r;
}

static int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

// Workspace: [counters of the fused kernel, 1 KB][gate_up out fp32 P x gu_rows][down out fp32
// P x dn_rows][compaction: ids, map, count, ids copy]. The counters sit at a fixed offset so a
// workspace reused across calls of different P keeps them.
constexpr int64_t kCtrBytes = 1024;

int64_t moe_ffn_workspace(int64_t P, int64_t gu_rows, int64_t dn_rows) {
  return kCtrBytes + align256(P * gu_rows * 4) + align256(P * dn_rows * 4) + align256(P * 12 + 4);
}

// Shared body of vq2_moe_expert_ffn and its variants: `ws` must hold moe_ffn_workspace bytes.
// ids_on_host: `ids` is a HOST array of P <= 64 ids, passed to the GPU in launch parameters.
int moe_expert_ffn(const void* h, int h_dtype, int64_t T, int64_t top_k, const int32_t* ids, const float* w,
                   const void* pool, int64_t num_experts, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows,
                   int64_t dn_cols, const void* cb0, int val_dtype, const int32_t* perm_in, const int8_t* sign_in,
                   int64_t hb_in, float scale_in, const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid,
                   float scale_mid, void* ws, void* out, int out_dtype, cudaStream_t st, bool ids_on_host,
                   bool counters_zeroed, int32_t* err, bool prefer_fused, const void* cb1, const float* add,
                   const PeerReduce* peer) {
  if (!h || !ids || !w || !pool || !cb0 || !perm_in || !sign_in || !perm_mid || !sign_mid || !ws || !out)
    return VQ2_ERR_ARG;
  if (T <= 0 || top_k <= 0 || top_k > 64 || num_experts <= 0) return VQ2_ERR_SHAPE;
  if (gu_rows <= 0 || gu_rows % 2 != 0 || gu_cols % 8 != 0 || dn_cols % 8 != 0 || gu_cols <= 0 || dn_cols <= 0)
    return VQ2_ERR_SHAPE;
  if (dn_cols * 8 != gu_rows / 2 || dn_rows != gu_cols * 8) return VQ2_ERR_SHAPE;  // SwiGLU width / hidden size
  if (h_dtype != VQ2_F32 && h_dtype != VQ2_F16 && h_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (out_dtype != VQ2_F32 && out_dtype != VQ2_F16 && out_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  const bool res = cb1 != nullptr;
  const RecordLayout L = record_layout(gu_rows, gu_cols, dn_rows, dn_cols, res);
  if (L.bytes % 16 != 0 || L.dn_idx % 16 != 0 || L.gu_idx1 % 8 != 0 || L.dn_idx1 % 8 != 0) return VQ2_ERR_ALIGN;
  if (!aligned(pool, 16) || !aligned(cb0, 16) || !aligned(ws, 256) || (res && !aligned(cb1, 16))) return VQ2_ERR_ALIGN;
  const int64_t P = T * top_k;
  if (P > 65536) return VQ2_ERR_SHAPE;
  const int64_t H = gu_cols * 8, I = gu_rows / 2;
  int32_t* ctr = static_cast<int32_t*>(ws);
  float* gu = reinterpret_cast<float*>(static_cast<char*>(ws) + kCtrBytes);
  float* yd = reinterpret_cast<float*>(reinterpret_cast<char*>(gu) + align256(P * gu_rows * 4));
  int32_t* c_ids = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(yd) + align256(P * dn_rows * 4));
  int32_t* c_map = c_ids + P;
  int32_t* c_cnt = c_map + P;
  int32_t* c_all = c_cnt + 1;  // the ids themselves when they arrive by value
  const char* base = static_cast<const char*>(pool);
  if (ids_on_host && P > kIdsByValue) return VQ2_ERR_SHAPE;

  // Decode-sized batches where launch cost dominates (the native paged step, issued eagerly from
  // the host): one fused launch (moe_fused.cu) instead of four. Inside a CUDA graph the four
  // kernels are faster on the GPU (40 vs 47 us per 35B layer at T = 1, top-8), so the generic
  // entry points keep them.
  if (prefer_fused && !res && !add && !peer && P <= kIdsByValue && moe_fused_enabled()) {
    MoeFusedArgs f{};
    f.h = h; f.h_dtype = h_dtype; f.T = (int)T; f.K = (int)top_k; f.P = (int)P;
    f.ids = ids_on_host ? nullptr : ids;
    if (ids_on_host)
      for (int64_t p = 0; p < P; ++p) f.iv.v[p] = ids[p];
    f.w = w; f.pool = static_cast<const uint8_t*>(pool); f.num_experts = num_experts; f.rec = L.bytes;
    f.off_gs = L.gu_scale; f.off_di = L.dn_idx; f.off_ds = L.dn_scale;
    f.gu_rows = (int)gu_rows; f.ng_gu = (int)gu_cols; f.dn_rows = (int)dn_rows; f.ng_dn = (int)dn_cols;
    f.cb0 = cb0; f.perm_in = perm_in; f.sign_in = sign_in; f.hb_in = (int)hb_in; f.scale_in = scale_in;
    f.perm_mid = perm_mid; f.sign_mid = sign_mid; f.hb_mid = (int)hb_mid; f.scale_mid = scale_mid;
    f.ctr = ctr; f.y_gu = gu; f.y_dn = yd; f.out = out; f.out_dtype = out_dtype; f.err = err;
    if (moe_fused_eligible(f, val_dtype)) {
      if (!counters_zeroed) {
        const cudaError_t e = cudaMemsetAsync(ctr, 0, kCtrBytes, st);
        if (e != cudaSuccess) {
          set_last_cuda_error(e);
          return VQ2_ERR_LAUNCH;
        }
      }
      return moe_fused_ffn(f, val_dtype, st);
    }
  }

  // Only problems whose expert is in the pool are computed (remote experts of an expert-parallel
  // rank are -1): compact them so the GEMV grid covers real work only.
  int s = ids_on_host ? run_compact(nullptr, P, num_experts, c_ids, c_map, c_cnt, st, ids, c_all)
                      : run_compact(ids, P, num_experts, c_ids, c_map, c_cnt, st);
  if (s != VQ2_OK) return s;
  if (ids_on_host) ids = c_all;

  GemvArgs a{};
  a.nprob = 0;
  a.x = h; a.x_dtype = h_dtype; a.x_mode = VQ2_ACT_RHT; a.x_row_stride = 0; a.x_k_stride = H; a.x_k_div = top_k;
  a.perm = perm_in; a.sign = sign_in; a.hb = (int)hb_in; a.rot_scale = scale_in; a.M = 1;
  a.idx0 = reinterpret_cast<const int16_t*>(base + L.gu_idx); a.cb0 = cb0;
  a.idx1 = res ? reinterpret_cast<const uint8_t*>(base + L.gu_idx1) : nullptr; a.cb1 = res ? cb1 : nullptr;
  a.scale = base + L.gu_scale; a.y = gu; a.y_dtype = VQ2_F32; a.y_row_stride = 0; a.y_k_stride = gu_rows;
  a.e_ids = c_ids; a.prob_count = c_cnt; a.prob_map = c_map;
  a.num_experts = num_experts; a.idx_e_stride = L.bytes / 2; a.idx1_e_stride = L.bytes; a.scale_e_stride = L.bytes / 2;
  a.out = (int)gu_rows; a.n = (int)H; a.rs = 1.f; a.K = (int)P;
  s = run_gemv(a, gu_rows * P, res, val_dtype, st);
  if (s != VQ2_OK) return s;

  GemvArgs b = a;
  b.x = gu; b.x_dtype = VQ2_F32; b.x_mode = VQ2_ACT_SWIGLU_RHT; b.x_k_stride = gu_rows; b.x_k_div = 1;
  b.perm = perm_mid; b.sign = sign_mid; b.hb = (int)hb_mid; b.rot_scale = scale_mid;
  b.idx0 = reinterpret_cast<const int16_t*>(base + L.dn_idx); b.scale = base + L.dn_scale;
  b.idx1 = res ? reinterpret_cast<const uint8_t*>(base + L.dn_idx1) : nullptr;
  b.y = yd; b.y_k_stride = dn_rows; b.out = (int)dn_rows; b.n = (int)I;
  s = run_gemv(b, dn_rows * P, res, val_dtype, st);
  if (s != VQ2_OK) return s;
  if (peer) {  // expert parallel: combine + sum over ranks in one kernel over peer memory
    if (add) return VQ2_ERR_ARG;
    return run_combine_peer(yd, w, T, (int)top_k, H, ids, num_experts, *peer, out, out_dtype, st);
  }
  return run_combine(yd, w, T, (int)top_k, H, add, out, out_dtype, st, ids, num_experts);
}

// ---- one MoE layer from router logits ------------------------------------------------------
// Workspace of moe_layer: [xrot fp32 T x H][ids, w: T x ks][compacted ids, map: P][count]
// [tstart, tcnt: T][combine counters: T x ceil(dn_rows / 8)][gate_up out fp32 P x gu_rows]
// [down out fp32 P x dn_rows], each part 256-byte aligned (P = T * ks).
struct LayerWs {
  float* xrot;
  int32_t* ids;
  float* w;
  int32_t *c_ids, *c_map, *c_cnt, *tstart, *tcnt, *ctr;
  float *gu, *yd;
  int64_t ctr_n, bytes;
};

static LayerWs layer_ws(void* base, int64_t T, int64_t ks, int64_t H, int64_t gu_rows, int64_t dn_rows) {
  LayerWs L{};
  const int64_t P = T * ks;
  char* p = static_cast<char*>(base);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* q = p ? p + off : nullptr;
    off += align256(bytes);
    return q;
  };
  L.xrot = reinterpret_cast<float*>(take(T * H * 4));
  L.ids = reinterpret_cast<int32_t*>(take(P * 4));
  L.w = reinterpret_cast<float*>(take(P * 4));
  L.c_ids = reinterpret_cast<int32_t*>(take(P * 4));
  L.c_map = reinterpret_cast<int32_t*>(take(P * 4));
  L.c_cnt = reinterpret_cast<int32_t*>(take(4));
  L.tstart = reinterpret_cast<int32_t*>(take(T * 4));
  L.tcnt = reinterpret_cast<int32_t*>(take(T * 4));
  L.ctr_n = T * ((dn_rows + 7) / 8);
  L.ctr = reinterpret_cast<int32_t*>(take(L.ctr_n * 4));
  L.gu = reinterpret_cast<float*>(take(P * gu_rows * 4));
  L.yd = reinterpret_cast<float*>(take(P * dn_rows * 4));
  L.bytes = off;
  return L;
}

int64_t moe_layer_workspace(int64_t T, int64_t ks, int64_t H, int64_t gu_rows, int64_t dn_rows) {
  return layer_ws(nullptr, T, ks, H, gu_rows, dn_rows).bytes;
}

// Router + routed (and shared) expert FFN + combine of one MoE layer: three launches (route,
// gate_up, down with the combine in its epilogue) up to kFuseCombineMaxP (token, expert)
// problems, else four (a separate combine kernel); with the cross-rank sum over peer memory the
// fourth is the peer combine.
constexpr int64_t kFuseCombineMaxP = 64;
int moe_layer(const void* h, int h_dtype, int64_t T, const float* logits, int64_t E, int64_t K,
              const float* shared_gate, int64_t lo, int64_t hi, int rank, int world, const void* pool,
              int64_t pool_rows, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0,
              int val_dtype, const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in,
              const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid, float scale_mid, void* ws,
              int64_t ws_bytes, void* out, int out_dtype, cudaStream_t st, const PeerReduce* peer) {
  if (!h || !logits || !pool || !cb0 || !perm_in || !sign_in || !perm_mid || !sign_mid || !ws || !out)
    return VQ2_ERR_ARG;
  if (T <= 0 || T > 4096 || E <= 0 || K <= 0 || K > 32 || K > E) return VQ2_ERR_SHAPE;
  if (gu_rows <= 0 || gu_rows % 2 != 0 || gu_cols <= 0 || gu_cols % 8 != 0 || dn_cols <= 0 || dn_cols % 8 != 0)
    return VQ2_ERR_SHAPE;
  if (dn_cols * 8 != gu_rows / 2 || dn_rows != gu_cols * 8) return VQ2_ERR_SHAPE;
  if (lo < 0 || hi < lo || hi > E || world <= 0 || rank < 0 || rank >= world) return VQ2_ERR_ARG;
  const int64_t ks = K + (shared_gate ? 1 : 0);
  const int64_t shared_row = hi - lo;
  if (pool_rows < shared_row + (shared_gate ? 1 : 0)) return VQ2_ERR_SHAPE;
  if (h_dtype != VQ2_F32 && h_dtype != VQ2_F16 && h_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  if (out_dtype != VQ2_F32 && out_dtype != VQ2_F16 && out_dtype != VQ2_BF16) return VQ2_ERR_DTYPE;
  const int64_t H = gu_cols * 8, I = gu_rows / 2;
  const RecordLayout R = record_layout(gu_rows, gu_cols, dn_rows, dn_cols);
  if (R.bytes % 16 != 0 || R.dn_idx % 16 != 0) return VQ2_ERR_ALIGN;
  if (!aligned(pool, 16) || !aligned(cb0, 16) || !aligned(ws, 256)) return VQ2_ERR_ALIGN;
  const LayerWs L = layer_ws(ws, T, ks, H, gu_rows, dn_rows);
  if (ws_bytes < L.bytes) return VQ2_ERR_ARG;
  const int64_t P = T * ks;

  if (T == 1) {  // one token: routing recomputed inside two launches (moe_decode.cu)
    const int s1 = run_moe_t1(h, h_dtype, logits, E, K, shared_gate, lo, hi, rank, world, pool, pool_rows, gu_rows,
                              gu_cols, dn_rows, dn_cols, cb0, val_dtype, perm_in, sign_in, hb_in, scale_in, perm_mid,
                              sign_mid, hb_mid, scale_mid, R.bytes, R.gu_idx, R.gu_scale, R.dn_idx, R.dn_scale, L.gu,
                              peer ? static_cast<void*>(L.yd) : out, peer ? VQ2_F32 : out_dtype, st);
    if (s1 != -1) {
      if (s1 != VQ2_OK || !peer) return s1;
      // the partial is already combined: one "problem" per token, weight 1, all local. (Fusing this
      // exchange into the 296 down CTAs measured slower: a system-scope fence and a peer wait per CTA.)
      return run_combine_peer(L.yd, nullptr, 1, 1, H, nullptr, 1, *peer, out, out_dtype, st);
    }
  }

  RouteArgs r{};
  r.logits = logits; r.T = (int)T; r.E = (int)E; r.K = (int)K;
  r.h = h; r.h_dtype = h_dtype; r.H = (int)H; r.gate = shared_gate;
  r.ids = L.ids; r.w = L.w; r.ks = (int)ks; r.layer = true;
  r.lo = (int)lo; r.hi = (int)hi; r.shared_row = (int)shared_row; r.rank = rank; r.world = world;
  r.perm = perm_in; r.sign = sign_in; r.hb = (int)hb_in; r.rot_scale = scale_in; r.xrot = L.xrot;
  r.c_ids = L.c_ids; r.c_map = L.c_map; r.c_cnt = L.c_cnt; r.tstart = L.tstart; r.tcnt = L.tcnt;
  // the combine rides in the down GEMV's epilogue for decode-sized batches (it saves a launch on
  // the critical path); past that its per-item fence and barriers cost more than the launch
  const bool fuse_combine = !peer && P <= kFuseCombineMaxP;
  r.zero = fuse_combine ? L.ctr : nullptr; r.zero_n = fuse_combine ? L.ctr_n : 0;
  const bool all_local = lo == 0 && hi == E && world == 1;
  r.out = (peer || all_local) ? nullptr : out; r.out_dtype = out_dtype;
  r.arrive = peer ? peer->epochs + 2 : nullptr;  // the peer state's third word: route arrivals
  int s = run_route(r, st);
  if (s != VQ2_OK) return s;

  const char* base = static_cast<const char*>(pool);
  GemvArgs a{};
  a.nprob = 0;
  a.x = L.xrot; a.x_dtype = VQ2_F32; a.x_mode = VQ2_ACT_ROTATED; a.x_row_stride = 0; a.x_k_stride = H;
  a.x_k_div = ks; a.M = 1;
  a.idx0 = reinterpret_cast<const int16_t*>(base + R.gu_idx); a.cb0 = cb0;
  a.scale = base + R.gu_scale; a.y = L.gu; a.y_dtype = VQ2_F32; a.y_row_stride = 0; a.y_k_stride = gu_rows;
  a.e_ids = L.c_ids; a.prob_count = L.c_cnt; a.prob_map = L.c_map;
  a.num_experts = pool_rows; a.idx_e_stride = R.bytes / 2; a.idx1_e_stride = R.bytes; a.scale_e_stride = R.bytes / 2;
  a.out = (int)gu_rows; a.n = (int)H; a.rs = 1.f; a.K = (int)P;
  if ((s = run_gemv(a, gu_rows * P, false, val_dtype, st)) != VQ2_OK) return s;

  GemvArgs b = a;
  b.x = L.gu; b.x_mode = VQ2_ACT_SWIGLU_RHT; b.x_k_stride = gu_rows; b.x_k_div = 1;
  b.perm = perm_mid; b.sign = sign_mid; b.hb = (int)hb_mid; b.rot_scale = scale_mid;
  b.idx0 = reinterpret_cast<const int16_t*>(base + R.dn_idx); b.scale = base + R.dn_scale;
  b.y = L.yd; b.y_k_stride = dn_rows; b.out = (int)dn_rows; b.n = (int)I;
  if (fuse_combine) {  // the routing-weighted sum of each token's problems in the down GEMV's epilogue
    b.comb_w = L.w; b.comb_tstart = L.tstart; b.comb_tcnt = L.tcnt; b.comb_ctr = L.ctr;
    b.comb_out = out; b.comb_dtype = out_dtype; b.comb_ks = (int)ks;
  }
  if ((s = run_gemv(b, dn_rows * P, false, val_dtype, st)) != VQ2_OK) return s;
  if (peer) return run_combine_peer(L.yd, L.w, T, (int)ks, H, L.ids, pool_rows, *peer, out, out_dtype, st);
  if (!fuse_combine) return run_combine(L.yd, L.w, T, (int)ks, H, nullptr, out, out_dtype, st, L.ids, pool_rows);
  return VQ2_OK;
}

}  // namespace vq2

extern "C" int64_t vq2_moe_expert_ffn_workspace(int64_t T, int64_t top_k, int64_t gu_rows, int64_t dn_rows) {
  if (T <= 0 || top_k <= 0 || gu_rows <= 0 || dn_rows <= 0) return -1;
  return vq2::moe_ffn_workspace(T * top_k, gu_rows, dn_rows);
}

extern "C" int vq2_moe_expert_ffn(const void* h, int h_dtype, int64_t T, int64_t top_k, const int32_t* ids,
                                  const float* w, const void* pool, int64_t num_experts, int64_t gu_rows,
                                  int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
                                  const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in,
                                  const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid, float scale_mid,
                                  void* workspace, int64_t workspace_bytes, void* out, int out_dtype, void* stream) {
  if (T <= 0 || top_k <= 0 || gu_rows <= 0 || dn_rows <= 0) return VQ2_ERR_SHAPE;
  if (workspace_bytes < vq2::moe_ffn_workspace(T * top_k, gu_rows, dn_rows)) return VQ2_ERR_ARG;
  return vq2::moe_expert_ffn(h, h_dtype, T, top_k, ids, w, pool, num_experts, gu_rows, gu_cols, dn_rows, dn_cols,
                             cb0, val_dtype, perm_in, sign_in, hb_in, scale_in, perm_mid, sign_mid, hb_mid,
                             scale_mid, workspace, out, out_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int vq2_moe_expert_ffn_res(const void* h, int h_dtype, int64_t T, int64_t top_k, const int32_t* ids,
                                      const float* w, const void* pool, int64_t num_experts, int64_t gu_rows,
                                      int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0,
                                      const void* cb1, int val_dtype, const int32_t* perm_in, const int8_t* sign_in,
                                      int64_t hb_in, float scale_in, const int32_t* perm_mid,
                                      const int8_t* sign_mid, int64_t hb_mid, float scale_mid, const float* add,
                                      void* workspace, int64_t workspace_bytes, void* out, int out_dtype,
                                      void* stream) {
  if (T <= 0 || top_k <= 0 || gu_rows <= 0 || dn_rows <= 0) return VQ2_ERR_SHAPE;
  if (!cb1) return VQ2_ERR_ARG;
  if (workspace_bytes < vq2::moe_ffn_workspace(T * top_k, gu_rows, dn_rows)) return VQ2_ERR_ARG;
  return vq2::moe_expert_ffn(h, h_dtype, T, top_k, ids, w, pool, num_experts, gu_rows, gu_cols, dn_rows, dn_cols,
                             cb0, val_dtype, perm_in, sign_in, hb_in, scale_in, perm_mid, sign_mid, hb_mid,
                             scale_mid, workspace, out, out_dtype, static_cast<cudaStream_t>(stream), false, false,
                             nullptr, false, cb1, add);
}

// ---- allocation-free variant -----------------------------------------------------------------
// Scratch for vq2_moe_expert_ffn_noalloc: one static device array per device that loads this
// library, held until the process exits. Every call on a device shares it, so calls that
// overlap on the GPU (different streams, no ordering between them) race on it. The two
// intermediates it holds (gate|up and down outputs) are written in full by each call before
// they are read, so nothing needs clearing between calls.
static __device__ __align__(256) unsigned char g_moe_ffn_scratch[VQ2_MOE_FFN_NOALLOC_MAX_BYTES];

namespace vq2 {

// Device address of g_moe_ffn_scratch for the current device. In host code the symbol names a
// host-side stand-in, never the device array, so its address must come from
// cudaGetSymbolAddress, called with the device current; the result is cached per device
// ordinal (a cudaDeviceReset makes it stale: documented as unsupported after a reset).
static void* noalloc_scratch(int* status) {
  static std::atomic<void*> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    *status = VQ2_ERR_LAUNCH;
    return nullptr;
  }
  void* p = dev < 64 ? cache[dev].load() : nullptr;
  if (p == nullptr) {
    e = cudaGetSymbolAddress(&p, g_moe_ffn_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_cuda_error(e);
      *status = VQ2_ERR_LAUNCH;
      return nullptr;
    }
    if (dev < 64) cache[dev].store(p);
  }
  return p;
}

}  // namespace vq2

extern "C" int vq2_moe_expert_ffn_noalloc(const void* h, int h_dtype, int64_t T, int64_t top_k, const int32_t* ids,
                                          const float* w, const void* pool, int64_t num_experts, int64_t gu_rows,
                                          int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0,
                                          int val_dtype, const int32_t* perm_in, const int8_t* sign_in,
                                          int64_t hb_in, float scale_in, const int32_t* perm_mid,
                                          const int8_t* sign_mid, int64_t hb_mid, float scale_mid, void* out,
                                          int out_dtype, void* stream) {
  if (T <= 0 || top_k <= 0 || gu_rows <= 0 || dn_rows <= 0) return VQ2_ERR_SHAPE;
  if (vq2::moe_ffn_workspace(T * top_k, gu_rows, dn_rows) > (int64_t)VQ2_MOE_FFN_NOALLOC_MAX_BYTES)
    return VQ2_ERR_SHAPE;  // more (token, expert) problems than the static scratch holds
  int status = VQ2_OK;
  void* ws = vq2::noalloc_scratch(&status);
  if (ws == nullptr) return status;
  // always the four-kernel sequence (prefer_fused false): no counters are kept in the scratch
  return vq2::moe_expert_ffn(h, h_dtype, T, top_k, ids, w, pool, num_experts, gu_rows, gu_cols, dn_rows, dn_cols,
                             cb0, val_dtype, perm_in, sign_in, hb_in, scale_in, perm_mid, sign_mid, hb_mid,
                             scale_mid, ws, out, out_dtype, static_cast<cudaStream_t>(stream), false, false,
                             nullptr, false);
}

extern "C" int64_t vq2_moe_layer_workspace(int64_t T, int64_t top_k, int has_shared, int64_t hidden, int64_t gu_rows,
                                           int64_t dn_rows) {
  if (T <= 0 || top_k <= 0 || hidden <= 0 || gu_rows <= 0 || dn_rows <= 0) return -1;
  return vq2::moe_layer_workspace(T, top_k + (has_shared ? 1 : 0), hidden, gu_rows, dn_rows);
}

extern "C" int vq2_moe_layer(const void* h, int h_dtype, int64_t T, const float* logits, int64_t E, int64_t top_k,
                             const float* shared_gate, int64_t expert_lo, int64_t expert_hi, int rank, int world,
                             const void* pool, int64_t pool_rows, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows,
                             int64_t dn_cols, const void* cb0, int val_dtype, const int32_t* perm_in,
                             const int8_t* sign_in, int64_t hb_in, float scale_in, const int32_t* perm_mid,
                             const int8_t* sign_mid, int64_t hb_mid, float scale_mid, void* workspace,
                             int64_t workspace_bytes, void* out, int out_dtype, void* stream) {
  return vq2::moe_layer(h, h_dtype, T, logits, E, top_k, shared_gate, expert_lo, expert_hi, rank, world, pool,
                        pool_rows, gu_rows, gu_cols, dn_rows, dn_cols, cb0, val_dtype, perm_in, sign_in, hb_in,
                        scale_in, perm_mid, sign_mid, hb_mid, scale_mid, workspace, workspace_bytes, out, out_dtype,
                        static_cast<cudaStream_t>(stream), nullptr);
}
