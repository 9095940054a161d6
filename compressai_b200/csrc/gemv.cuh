// Internal interface of the VQ GEMV kernel family (vq_gemv.cu), shared with the fused MoE
// entry points.
#pragma once
#include "common.cuh"

namespace vq2 {

constexpr int kMaxProbs = 8;  // matrices sharing one activation in a multi-matrix launch

struct GemvArgs {
  const void* x;          // activations, x_dtype (mode SWIGLU_RHT: fp32 [gate | up] rows)
  int x_dtype;
  int x_mode;             // VQ2_ACT_ROTATED / VQ2_ACT_RHT / VQ2_ACT_SWIGLU_RHT
  int64_t x_row_stride;   // elements between activation rows m
  int64_t x_k_stride;     // elements between activation groups of problems (0 = shared)
  int64_t x_k_div;        // problem k reads activation group k / x_k_div
  const int32_t* perm;    // rotation (modes RHT, SWIGLU_RHT)
  const int8_t* sign;
  int hb;
  float rot_scale;
  int M;                  // activation rows
  // expert-indexed problems (nprob == 0): problem k uses expert e_ids[k] of one pool
  const int16_t* idx0;    // [E, out, ng]
  const uint8_t* idx1;    // [E, out, ng] or null
  const void* scale;      // [E, out] val
  void* y;                // [K, M, out] y_dtype
  const int32_t* e_ids;   // [K] or null (problem k uses expert 0)
  const int32_t* prob_count;  // device problem count (<= K) or null: problems [count, K) are skipped
  const int32_t* prob_map;    // [K] original problem index of each (compacted) problem, or null
  int64_t num_experts;
  int64_t idx_e_stride;   // out * ng (int16 elements between experts' idx0)
  int64_t idx1_e_stride;  // bytes between experts' idx1 (3 bpw expert pools)
  int64_t scale_e_stride; // out
  int64_t y_k_stride;     // elements between problems k
  // multi-matrix problems (nprob > 0): problem p has its own weights/outputs, one shared x
  int nprob;
  const int16_t* p_idx0[kMaxProbs];
  const uint8_t* p_idx1[kMaxProbs];
  const void* p_scale[kMaxProbs];
  void* p_y[kMaxProbs];
  int p_out[kMaxProbs];
  int p_rb0[kMaxProbs + 1];  // first row block of each problem
  // common
  const void* cb0;        // [65536, 8] val
  const void* cb1;        // [256, 8] val or null
  int y_dtype;
  int64_t y_row_stride;   // elements between output rows m
  unsigned long long* argmax;  // greedy argmax per activation row m (multi mode, CUDA cores), or null
  bool no_y;                   // argmax only: outputs are not written
  // fused routing-weighted combine (expert-indexed mode; comb_w null: off): when the last of
  // token t's problems has written a row block, the CTA that wrote it sums the token's problems
  // there in problem order, out[t, r] = sum_c w[map[c]] * y[map[c], r], into comb_out
  const float* comb_w;        // [T * comb_ks] weights by original problem index
  const int32_t* comb_tstart; // [T] first compacted problem of token t
  const int32_t* comb_tcnt;   // [T] compacted problems of token t
  int32_t* comb_ctr;          // [T * row_blocks] arrival counters, zero at launch
  void* comb_out;             // [T, out] in comb_dtype
  int comb_dtype, comb_ks;
  int out;                // rows (expert-indexed mode)
  int n;
  float rs;
  int K;                  // problems (expert-indexed mode)
  int mtiles;             // M tiles
  int row_blocks;         // row blocks per (problem, M tile) (expert mode) / total (multi mode)
};

// Order-preserving 64-bit key of a router logit: larger value first, equal values to the smaller
// expert id (the router's rank rule o > l || (o == l && j < i)), -0 as +0 (as float comparison);
// 0 is below every key.
__device__ __forceinline__ unsigned long long route_key(float v, int i) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xffffffffu - static_cast<uint32_t>(i));
}

// Launch the GEMV described by `a` (expert-indexed when a.nprob == 0, multi-matrix otherwise);
// total_rows = rows of all problems (sizes the work split); res = 3 bpw.
int run_gemv(GemvArgs a, int64_t total_rows, bool res, int val_dtype, cudaStream_t st, void* ws = nullptr,
             int64_t ws_bytes = 0);

// Tensor-core batched path (vq_gemm_tc.cu) for multi-matrix problems on pre-rotated
// activations; `ws` holds gemm_tc_workspace(M, n) bytes; returns -1 when not eligible.
int run_gemm_tc(const GemvArgs& a, bool res, int val_dtype, void* ws, cudaStream_t st);
// Workspace bytes of the tensor-core path: the 16-bit hi/lo split of the [M, n] activations.
int64_t gemm_tc_workspace(int64_t M, int64_t n);
// The 16-bit operand halves of the tensor-core paths from a's activations (vq_gemm_tc.cu): hi =
// round(x), lo = round(x - hi), each [M, n]; the RHT (or SwiGLU + RHT) is applied on the way
// when a.x_mode asks for it. xl null: hi only.
int tc_operands(const GemvArgs& a, void* xh, void* xl, int val_dtype, cudaStream_t st);
// Tensor-core path on tcgen05 / TMEM / TMA (vq_gemm_umma.cu) for multi-matrix problems with
// enough 128-row tiles to fill the GPU; returns -1 when not eligible.
int run_gemm_umma(const GemvArgs& a, bool res, int val_dtype, void* ws, int64_t ws_bytes, cudaStream_t st);
// Forward RHT (or SwiGLU + RHT) of M rows into the hi / lo operand halves of the tensor-core
// GEMV (rht.cu).
int rht_split(const void* x, int x_dtype, int x_mode, int64_t x_row_stride, int64_t M, int64_t n, int64_t hb,
              const int32_t* perm, const int8_t* sign, float scale, void* xh, void* xl, int val_dtype,
              cudaStream_t st);

// Launch the routing-weighted combine out[t] = sum_j w[t, j] y[t*top_k + j] (+ add[t]) (moe.cu);
// with ids != null, rows whose id is outside [0, num_experts) are skipped.
int run_combine(const float* y, const float* w, int64_t T, int top_k, int64_t H, const float* add, void* out,
                int out_dtype, cudaStream_t st, const int32_t* ids = nullptr, int64_t num_experts = 0);

// Up to 64 problem ids passed by value in launch parameters (no upload copy needed).
constexpr int kIdsByValue = 64;
struct IdsByValue {
  int32_t v[kIdsByValue];
};

// Stable compaction of the problems whose id is in [0, num_experts): out_ids[c] = ids[p],
// out_map[c] = p, *out_count = number kept (moe.cu). One CTA; P <= 65536. With host_ids
// (a HOST array, P <= 64) the ids travel in the launch parameters and are written to
// ids_copy (device, P) for later kernels; ids is then ignored.
int run_compact(const int32_t* ids, int64_t P, int64_t num_experts, int32_t* out_ids, int32_t* out_map,
                int32_t* out_count, cudaStream_t st, const int32_t* host_ids = nullptr, int32_t* ids_copy = nullptr);

// Router of one MoE layer (moe.cu): one CTA for all T tokens; see moe_route_kernel.
struct RouteArgs {
  const float* logits;
  int T, E, K;
  const void* h;
  int h_dtype, H;
  const float* gate;     // shared-expert gate [H] fp32, or null
  int32_t* ids;          // [T, ks]
  float* w;              // [T, ks]
  int ks;                // K (+1 in layer mode with a shared expert)
  float* shared_w;       // legacy mode: [T] sigmoid gate, or null
  bool layer;            // layer mode (local ids, shared column, RHT, compaction)
  int lo, hi, shared_row, rank, world;
  const int32_t* perm;
  const int8_t* sign;
  int hb;
  float rot_scale;
  float* xrot;           // [T, H] fp32
  int32_t* c_ids;        // [T*ks] compacted pool rows
  int32_t* c_map;        // [T*ks] original problem index of each
  int32_t* c_cnt;        // [1]
  int32_t* tstart;       // [T] first compacted problem of token t
  int32_t* tcnt;         // [T] compacted problems of token t
  int32_t* zero;         // int32 words cleared for later kernels (combine counters), or null
  int64_t zero_n;
  void* out;             // layer mode: [T, H] rows of tokens without local problems are zeroed, or null
  int out_dtype;
  int32_t* arrive;       // layer mode, expert parallel: arrival counter (zero at entry, left at zero)
};

int run_route(const RouteArgs& r, cudaStream_t st);

// Cross-GPU reduction of the expert-parallel combine over peer memory (moe_ep.cu).
constexpr int kPeerMaxBlocks = 128;    // CTAs (output ranges) of the peer combine, at most
constexpr int kPeerFlagStride = 512;   // flags per rank in the symmetric buffer: CTAs of one exchange, at most
constexpr int kPeerWaitPolls = 1 << 22;  // default poll limit of a peer wait, ~1 s at 64 ns naps
constexpr int kPeerTimeout = 0x200;      // status word of a wait that gave up
constexpr int kPeerTightPolls = 2048;    // polls before napping between them

struct PeerReduce {
  uint8_t* const* peers;  // device array [world] of the symmetric buffers' base addresses
  int rank, world;
  int64_t part_off;       // bytes: flags region (world x kPeerFlagStride uint32) padded
  int64_t part_bytes;     // bytes of one (parity, rank) slot (>= T x H fp32)
  int32_t* epochs;        // local device state {sequence number, finished CTAs}, zero at first use
  int32_t* err;           // optional status word (timeouts)
  int max_polls;          // polls of a peer flag before giving up (<= 0: about a second)
};
int run_combine_peer(const float* y, const float* w, int64_t T, int top_k, int64_t H, const int32_t* ids,
                     int64_t num_experts, const PeerReduce& pr, void* out, int out_dtype, cudaStream_t st);

// Routed-expert FFN of one MoE layer (moe_ffn.cu): compaction, gate_up GEMV (input RHT),
// down GEMV (SwiGLU + RHT), combine; `ws` holds moe_ffn_workspace(T * top_k, ...) bytes.
int64_t moe_ffn_workspace(int64_t P, int64_t gu_rows, int64_t dn_rows);
int moe_expert_ffn(const void* h, int h_dtype, int64_t T, int64_t top_k, const int32_t* ids, const float* w,
                   const void* pool, int64_t num_experts, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows,
                   int64_t dn_cols, const void* cb0, int val_dtype, const int32_t* perm_in, const int8_t* sign_in,
                   int64_t hb_in, float scale_in, const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid,
                   float scale_mid, void* ws, void* out, int out_dtype, cudaStream_t st, bool ids_on_host = false,
                   bool counters_zeroed = false, int32_t* err = nullptr, bool prefer_fused = false,
                   const void* cb1 = nullptr, const float* add = nullptr, const PeerReduce* peer = nullptr);

// One MoE layer from router logits (moe_ffn.cu): route kernel, gate_up GEMV, down GEMV with the
// combine in its epilogue (or the peer combine when `peer` is given).
int64_t moe_layer_workspace(int64_t T, int64_t ks, int64_t H, int64_t gu_rows, int64_t dn_rows);
int moe_layer(const void* h, int h_dtype, int64_t T, const float* logits, int64_t E, int64_t K,
              const float* shared_gate, int64_t lo, int64_t hi, int rank, int world, const void* pool,
              int64_t pool_rows, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0,
              int val_dtype, const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in,
              const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid, float scale_mid, void* ws,
              int64_t ws_bytes, void* out, int out_dtype, cudaStream_t st, const PeerReduce* peer);

// One-token MoE layer in two launches (moe_decode.cu): routing recomputed per CTA, gate_up rows
// into `gu` ([K + 1, 1024] fp32), then the down rows over all problems with the combine, into
// `out` (out_dtype; fp32 for a rank's partial). Returns -1 when the shapes are not the specialisation's (hidden
// 2048, intermediate 512, top-k <= 8, E <= 256, 2 bpw) or VQ2_MOE_T1=0.
int run_moe_t1(const void* h, int h_dtype, const float* logits, int64_t E, int64_t K, const float* shared_gate,
               int64_t lo, int64_t hi, int rank, int world, const void* pool, int64_t pool_rows, int64_t gu_rows,
               int64_t gu_cols, int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
               const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in, float scale_in, const int32_t* perm_mid,
               const int8_t* sign_mid, int64_t hb_mid, float scale_mid, int64_t rec, int64_t off_gu_idx,
               int64_t off_gu_scale, int64_t off_dn_idx, int64_t off_dn_scale, float* gu, void* out, int out_dtype,
               cudaStream_t st);

// Fused single-launch expert FFN for T * top_k <= 64 (moe_fused.cu).
struct MoeFusedArgs {
  const void* h;
  int h_dtype, T, K, P;
  const int32_t* ids;  // device ids [P], or null: ids by value in iv
  IdsByValue iv;
  const float* w;      // [T, K]
  const uint8_t* pool; // [num_experts, rec] expert records
  int64_t num_experts, rec, off_gs, off_di, off_ds;
  int gu_rows, ng_gu, dn_rows, ng_dn;
  const void* cb0;
  const int32_t* perm_in;
  const int8_t* sign_in;
  int hb_in;
  float scale_in;
  const int32_t* perm_mid;
  const int8_t* sign_mid;
  int hb_mid;
  float scale_mid;
  int32_t* ctr;        // counters (zero between launches)
  float* y_gu;         // [P, gu_rows]
  float* y_dn;         // [P, dn_rows]
  void* out;           // [T, dn_rows]
  int out_dtype;
  int32_t* err;        // optional status word
};

bool moe_fused_eligible(const MoeFusedArgs& a, int val_dtype);
int moe_fused_ffn(const MoeFusedArgs& a, int val_dtype, cudaStream_t st);

// VQ2A decode of up to 32 segments of src into dst in one launch (rans.cu); status as
// vq2_rans_decode_segments.
int ans_launch(const uint8_t* src, int64_t src_bytes, const int64_t* src_off, const int64_t* seg_bytes,
               const int64_t* dst_off, const int64_t* seg_n, const int32_t* kind, int64_t nseg, uint8_t* dst,
               int64_t dst_bytes, int32_t* status, cudaStream_t st);

}  // namespace vq2
