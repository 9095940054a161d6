/*
 * vq2_b200.h -- C-ABI of the B200-native (sm_100a) VQ2 decode hot path.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no framework types. Every
 * entry point:
 *   - takes DEVICE pointers (except where stated) and enqueues its work on `stream`
 *     (NULL = legacy default stream); it never synchronizes and never allocates;
 *   - returns a status code (VQ2_OK = 0); on VQ2_ERR_LAUNCH the CUDA error code is kept
 *     for vq2_last_cuda_error();
 *   - is safe to capture in a CUDA graph.
 *
 * Index tensors hold the reference container layout: 16-bit stage indices are int16 holding
 * uint16 bits (masked with 0xFFFF, reference vq2/kernels.py:47,72), the optional residual
 * stage is uint8, both row-major [out, n/8]; one index selects an 8-dim codebook row.
 * Codebooks are [K, 8] and scales [out], both in the "value" dtype (fp16 or bf16).
 *
 * Reference citations are paths inside Unoalss/CompressAI.
 */
#ifndef VQ2_B200_H
#define VQ2_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define VQ2_API __attribute__((visibility("default")))
#else
#define VQ2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define VQ2_OK 0
#define VQ2_ERR_SHAPE 1    /* unsupported or inconsistent dimensions */
#define VQ2_ERR_DTYPE 2    /* unsupported dtype code */
#define VQ2_ERR_ALIGN 3    /* a pointer or stride breaks the required alignment */
#define VQ2_ERR_LAUNCH 4   /* CUDA launch/runtime error (see vq2_last_cuda_error) */
#define VQ2_ERR_TIMEOUT 5  /* a bounded device-side wait gave up */
#define VQ2_ERR_ARG 6      /* null pointer or out-of-range argument */

/* dtype codes */
#define VQ2_F16 0
#define VQ2_BF16 1
#define VQ2_F32 2

/* ABI version of this header (bumped on any signature change). */
VQ2_API int vq2_abi_version(void);
/* Static description of a status code. */
VQ2_API const char* vq2_status_string(int status);
/* cudaError_t of the most recent VQ2_ERR_LAUNCH (0 if none). */
VQ2_API int vq2_last_cuda_error(void);

/*
 * Randomized Hadamard transform, forward (inverse = 0):
 *   xr[m, b*hb + j] = out_scale * sum_i H[j, i] * x[m, perm[b*hb + i]] * sign[b*hb + i]
 * and inverse (inverse = 1), the transpose map:
 *   xr[m, perm[b*hb + j]] = out_scale * sign[b*hb + j] * sum_i H[j, i] * x[m, b*hb + i]
 * for every row m < M and block b < n/hb, H the Sylvester Hadamard matrix of order hb.
 * out_scale = hb^-0.5 gives Rot.fwd / Rot.inv; out_scale = 1 gives FastRot's unnormalised
 * variant. x: [M, n] (x_dtype, row stride x_row_stride elements); perm: int32 [n], a
 * permutation of 0..n-1; sign: int8 [n] of +-1; xr: fp32 [M, n] (row stride xr_row_stride),
 * must not alias x. hb a power of two in [64, 2048].
 * Replaces: Rot.fwd / Rot._orig_fwd / Rot.inv (vq2/vq.py:66-87) and FastRot.__call__
 * (vq2/runtime.py:57-63).
 */
VQ2_API int vq2_rht(const void* x, int x_dtype, int64_t x_row_stride, int64_t M, int64_t n,
                    int64_t hb, const int32_t* perm, const int8_t* sign, float out_scale,
                    int inverse, float* xr, int64_t xr_row_stride, void* stream);

/*
 * SwiGLU activation fused with the forward RHT of its result:
 *   act[m, j] = silu(gu[m, j]) * gu[m, I + j]      (j < I, fp32 math)
 *   xr[m, :]  = RHT_forward(act[m, :])              (as vq2_rht with inverse = 0)
 * gu: fp32 [M, 2I] (row stride gu_row_stride); xr: fp32 [M, I]. I = n is the RHT length.
 * Replaces: the torch ops `silu(gate.float()) * up.float()` and `rot_512.fwd(act)` of
 * PagedMoEExpert.forward (vq2/paged_runtime.py:501-504).
 */
VQ2_API int vq2_swiglu_rht(const float* gu, int64_t gu_row_stride, int64_t M, int64_t n,
                           int64_t hb, const int32_t* perm, const int8_t* sign, float out_scale,
                           float* xr, int64_t xr_row_stride, void* stream);

/* activation operand modes of the GEMV entry points */
#define VQ2_ACT_ROTATED 0     /* x is already rotated; used as is */
#define VQ2_ACT_RHT 1         /* x is raw; the forward RHT (perm, sign, hb, rot_scale) runs in-kernel */
#define VQ2_ACT_SWIGLU_RHT 2  /* x rows are fp32 [gate | up] of 2n: silu(gate) * up, then forward RHT */

/*
 * VQ GEMV of P <= 8 matrices sharing one activation (fp32 accumulation):
 *   xr = act(x)                      (per x_mode: as is / RHT / SwiGLU then RHT, fp32)
 *   y_p[m, r] = rs * scale_p[r] * sum_g dot(cb0[idx0_p[r, g]] (+ cb1[idx1_p[r, g]]), xr[m, 8g:8g+8])
 * x: [M, n] (mode SWIGLU_RHT: fp32 [M, 2n]) in x_dtype, row stride x_row_stride; idx0_p: int16
 * [out_p, n/8]; idx1_p: uint8 [out_p, n/8] (3 bpw, all or none); cb0: [65536, 8]; cb1: [256, 8]
 * or NULL; scale_p: [out_p]; the codebooks and scales in val_dtype (fp16/bf16); y_p: [M, out_p]
 * in y_dtype with row stride y_row_stride. idx0, idx1, out, scale and y are HOST arrays of P
 * device pointers / sizes. n % 64 == 0; idx0_p, cb0, cb1 16-byte aligned, idx1_p 8-byte aligned.
 * Replaces: the per-matrix FastRot + vq_gemv_16 / vq_gemv_16_8 sequence of PackedLinear.forward
 * (vq2/runtime.py:91-104, vq2/kernels.py:32-78, 215-230), fused and batched over matrices
 * that read the same input (q/k/v, gate/up), for any number of rows M.
 */
VQ2_API int vq2_gemv_multi(const void* x, int x_dtype, int x_mode, int64_t M, int64_t x_row_stride,
                           const int32_t* perm, const int8_t* sign, int64_t hb, float rot_scale,
                           int64_t P, const int16_t* const* idx0, const uint8_t* const* idx1,
                           const int64_t* out, const void* const* scale, const void* cb0,
                           const void* cb1, int val_dtype, void* const* y, int y_dtype,
                           int64_t y_row_stride, int64_t n, float rs, void* workspace,
                           int64_t workspace_bytes, void* stream);

/*
 * Row decode of a VQ matrix, one CTA per requested row:
 *   q[c, :] = scale[ids[c]] * (cb0[idx0[ids[c], g]] (+ cb1[idx1[ids[c], g]]))  for every group g
 * and, with perm/sign given, out[c, perm[j]] = (blockH_hb(q[c]) * inv_scale)[j] * sign[j] (the
 * inverse randomized Hadamard transform, inv_scale = hb^-1/2); without them out = q (rotated
 * space). ids: int64 [count] device; idx0 int16 [rows, n/8], idx1 uint8 or NULL, cb0/cb1/scale
 * in val_dtype; n % 256 == 0, n <= 8192; out [count, n] in out_dtype. Ids outside [0, rows) give
 * zero rows and set *bad (device int32) to 1.
 * Replaces: PackedEmbedding.forward (vq2/runtime.py:116-133: F.embedding of the codebooks, row
 * scale, Rot.inv, bf16) and the rotated-space rows of PackedLinear.weight_rows (:82-89).
 */
VQ2_API int vq2_embed_rows(const int64_t* ids, int64_t count, int64_t rows, const int16_t* idx0,
                           const uint8_t* idx1, const void* cb0, const void* cb1, const void* scale,
                           int val_dtype, int64_t n, const int32_t* perm, const int8_t* sign,
                           int64_t hb, float inv_scale, void* out, int out_dtype, int32_t* bad,
                           void* stream);

/*
 * GPU unpack of a fixed-width index stream: n symbols of `bits` (16: little-endian words; 8:
 * bytes; 4: two per byte, low nibble first; 12: two per 3 bytes, a | b << 12) from src (device,
 * src_bytes >= vq2_fixed_stream_bytes(bits, n)) into dst (device, n elements of dst_bytes = 2
 * (uint16 / int16 bits) or 1 (uint8, bits <= 8)).
 * Replaces: unpack_fixed (vq2/export.py:56-70) on the host inside decode_indices
 * (vq2/runtime.py:155-182).
 */
VQ2_API int64_t vq2_fixed_stream_bytes(int bits, int64_t n);
VQ2_API int vq2_unpack_fixed(const uint8_t* src, int64_t src_bytes, int bits, int64_t n, void* dst,
                             int dst_bytes, void* stream);

/*
 * Workspace bytes vq2_gemv_multi / vq2_gemv use for M activation rows of length n (0 for one
 * row; -1 on bad sizes). With n % 128 == 0 and M >= 4 (or M >= 2 when the matrices total
 * >= 16384 rows) the GEMV runs on the tensor cores, its 16-bit activation operand(s) held in the
 * workspace (16-byte aligned; 128-byte aligned for the tcgen05 kernel):
 *   - matrices with at least one 128-row tile per SM: tcgen05.mma with the accumulator in tensor
 *     memory, the activation tile loaded by TMA, the codebook rows gathered into swizzled shared
 *     memory (fp16 codebooks: activations rounded once to fp16, max error ~2e-4 of max|y|; bf16:
 *     hi + lo halves, two MMAs per step);
 *   - smaller matrices: mma.sync m16n8k16 fed directly by the gathers, split-K over thread-block
 *     clusters, activations as hi + lo halves (fp32-level accuracy).
 * With no workspace, or one too small, it runs on the CUDA cores.
 */
VQ2_API int64_t vq2_gemv_workspace(int64_t M, int64_t n);

/*
 * Sticky status of the tcgen05 GEMV kernel on the current device: VQ2_ERR_TIMEOUT once one of
 * its bounded on-chip waits gave up (the affected CTA freed its tensor memory and returned, its
 * outputs incomplete), else VQ2_OK; reset != 0 clears it. Synchronous (reads device memory).
 * No reference counterpart (the reference has no device-side waits).
 */
VQ2_API int vq2_tc_status(int reset);

/*
 * VQ GEMV on a pre-rotated activation, one matrix (vq2_gemv_multi with P = 1, mode ROTATED;
 * workspace as there, may be NULL):
 *   y[m, r] = rs * scale[r] * sum_g dot(cb0[idx0[r, g]] (+ cb1[idx1[r, g]]), xr[m, 8g:8g+8])
 * Replaces: vq_gemv_16 / vq_gemv_16_8 (vq2/kernels.py:215-230) and the Triton kernels
 * _vq_gemv_16 / _vq_gemv_16_8 (vq2/kernels.py:32-78), which handle M = 1 only.
 */
VQ2_API int vq2_gemv(const void* xr, int x_dtype, int64_t M, int64_t x_row_stride,
                     const int16_t* idx0, const uint8_t* idx1, const void* cb0, const void* cb1,
                     const void* scale, int val_dtype, void* y, int y_dtype, int64_t y_row_stride,
                     int64_t out, int64_t n, float rs, void* workspace, int64_t workspace_bytes,
                     void* stream);

/*
 * Greedy argmax fused into the VQ GEMV of one matrix (the lm_head): as vq2_gemv_multi with P = 1
 * (any x_mode), and best[m] = max over rows r of key(y[m, r], r), an order-preserving 64-bit key
 * (high 32 bits: the fp32 value's bits, flipped so unsigned order is numeric order; low 32 bits:
 * 0xffffffff - r, so ties go to the smaller row, as torch.argmax). best: device uint64 [M], zeroed
 * by the caller before the call (the kernel only raises it); the token of row m is
 * 0xffffffff - (best[m] & 0xffffffff). y may be NULL (argmax only; no logits written). M <= 64,
 * CUDA-core path. Replaces: the lm_head GEMV + torch argmax of the decode loop (LEGION greedy
 * decoding, legion/engine.py:288-303), with no [M, vocab] logits round trip when y is NULL.
 */
VQ2_API int vq2_gemv_argmax(const void* x, int x_dtype, int x_mode, int64_t M, int64_t x_row_stride,
                            const int32_t* perm, const int8_t* sign, int64_t hb, float rot_scale,
                            const int16_t* idx0, const uint8_t* idx1, const void* cb0,
                            const void* cb1, const void* scale, int val_dtype, int64_t out,
                            int64_t n, float rs, void* y, int y_dtype, int64_t y_row_stride,
                            unsigned long long* best, void* stream);

/*
 * Expert-indexed VQ GEMV over K problems (2 bpw):
 *   xr_k = act(x + (k / x_k_div) * x_k_stride)        (per x_mode, as in vq2_gemv_multi)
 *   y[k, r] = rs * scale[e_k, r] * sum_g dot(cb0[idx[e_k, r, g]], xr_k[8g:8g+8]),  e_k = e_ids[k]
 * x_k_stride = 0 shares one activation among all problems (gate_up of one token); x_k_div =
 * top_k maps problem t*top_k + j to token t. e_ids: int32 [K] device (slots of a paged pool or
 * ids of a resident pool; ids outside [0, num_experts) give zero rows). Expert e's indices are
 * the int16 [out, ng] block at idx + e * idx_e_stride and its scales the [out] vector at
 * scale + e * scale_e_stride (element strides; >= out * ng and >= out, so a pool may interleave
 * whole expert records); scales in val_dtype; y: [K, out] in y_dtype. ng % 8 == 0; idx, cb0
 * and every expert's index block 16-byte aligned.
 * Replaces: vq_moe_parallel_gate_up / vq_moe_parallel_down (vq2/kernels.py:246-264) and
 * _parallel_moe_gate_up_kernel / _parallel_moe_down_kernel (vq2/kernels.py:117-176), plus the
 * rot_2048.fwd / SwiGLU / rot_512.fwd torch ops around them (vq2/paged_runtime.py:495-504).
 */
VQ2_API int vq2_moe_gemv(const void* x, int x_dtype, int x_mode, int64_t x_k_stride, int64_t x_k_div,
                         const int32_t* perm, const int8_t* sign, int64_t hb, float rot_scale,
                         const int32_t* e_ids, int64_t K, int64_t num_experts, const int16_t* idx,
                         int64_t idx_e_stride, const void* cb0, const void* scale,
                         int64_t scale_e_stride, int val_dtype, void* y, int y_dtype,
                         int64_t out, int64_t ng, float rs, void* stream);

/*
 * Routing-weighted combine of per-(token, expert) rows:
 *   out[t, :] = sum_{j < top_k} w[t, j] * y[t * top_k + j, :]  (+ add[t, :] if add != NULL)
 * in fixed j order, fp32 math. y: fp32 [T*top_k, H]; w: fp32 [T, top_k]; add: fp32 [T, H]
 * or NULL; out: [T, H] in out_dtype.
 * Replaces: `(y_down * topk_w[:, None]).sum(0)` of PagedMoEExpert.forward
 * (vq2/paged_runtime.py:510) and the shared-expert add of Qwen3_5MoeSparseMoeBlock.
 */
VQ2_API int vq2_moe_combine(const float* y, const float* w, int64_t T, int64_t top_k,
                            int64_t H, const float* add, void* out, int out_dtype, void* stream);

/*
 * MoE router, per token t (one warp each):
 *   ids[t, :] = the top_k experts by logit (descending, ties to the lower id)
 *   w[t, j]   = softmax(logits[t])[ids[t, j]] / sum_j' softmax(logits[t])[ids[t, j']]
 * and, when shared_gate != NULL, shared_w[t] = sigmoid(sum_i h[t, i] * shared_gate[i]).
 * logits: fp32 [T, E] (E <= 1024); ids: int32 [T, top_k] (top_k <= 32); w: fp32 [T, top_k];
 * h: [T, H] in h_dtype; shared_gate: fp32 [H]; shared_w: fp32 [T].
 * Replaces: Qwen3_5MoeTopKRouter.forward's softmax/topk/renormalise and the
 * sigmoid(shared_expert_gate(x)) of Qwen3_5MoeSparseMoeBlock.forward (installed transformers
 * modeling_qwen3_5_moe.py:762-791), which the reference's MoE path consumes
 * (vq2/paged_runtime.py:439-444).
 */
VQ2_API int vq2_moe_route(const float* logits, int64_t T, int64_t E, int64_t top_k, int32_t* ids,
                          float* w, const void* h, int h_dtype, const float* shared_gate, int64_t H,
                          float* shared_w, void* stream);

/*
 * Routed-expert FFN of one MoE layer for T tokens with top_k experts each (P = T * top_k
 * (token, expert) problems; compaction + three kernels on `stream`):
 *   gu[p]  = GateUp_{ids[p]} . RHT_in(h[p / top_k])                  fp32 [P, gu_rows]
 *   yd[p]  = Down_{ids[p]} . RHT_mid(silu(gu[p, :I]) * gu[p, I:])     fp32 [P, dn_rows]
 *   out[t] = sum_j w[t, j] * yd[t * top_k + j]                        [T, H] in out_dtype
 * with I = gu_rows / 2 = dn_cols * 8 and H = gu_cols * 8 = dn_rows. ids: int32 [P] device,
 * rows of `pool` (expert ids of a resident pool or slots of a paged one; ids outside
 * [0, num_experts) contribute zero); w: fp32 [T, top_k]. pool: num_experts expert records
 * of the .vq2m payload layout, back to back: gate_up indices int16 [gu_rows, gu_cols], gate_up
 * scales [gu_rows], down indices int16 [dn_rows, dn_cols], down scales [dn_rows] (scales in
 * val_dtype), 16-byte aligned. RHT_in = (perm_in, sign_in, hb_in, scale_in), RHT_mid likewise
 * (as vq2_rht forward). workspace: device memory of >= vq2_moe_expert_ffn_workspace(T, top_k,
 * gu_rows, dn_rows) bytes, 256-byte aligned, holding gu and yd (after a first 1 KB used by
 * vq2_paged_moe_step's fused kernel).
 * Replaces: the compute of PagedMoEExpert.forward (vq2/paged_runtime.py:495-511, T > 1
 * :553-566) and PackedMoEExpertUniversal.forward (vq2/load_and_test_full_35b.py:53-95):
 * rot_2048.fwd, vq_moe_parallel_gate_up, SiLU*up, rot_512.fwd, vq_moe_parallel_down and the
 * weighted sum, for all T tokens at once.
 */
VQ2_API int vq2_moe_expert_ffn(const void* h, int h_dtype, int64_t T, int64_t top_k,
                               const int32_t* ids, const float* w, const void* pool,
                               int64_t num_experts, int64_t gu_rows, int64_t gu_cols,
                               int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
                               const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in,
                               float scale_in, const int32_t* perm_mid, const int8_t* sign_mid,
                               int64_t hb_mid, float scale_mid, void* workspace,
                               int64_t workspace_bytes, void* out, int out_dtype, void* stream);

/*
 * vq2_moe_expert_ffn over a pool of 3 bpw expert records (promoted "anchor" experts,
 * expert_modes["L:E"] == 3 in the .vq2m meta): each index entry is idx0 int16 [rows, cols]
 * followed by idx1 uint8 [rows, cols] (gate_up idx0 | idx1 | scales | down idx0 | idx1 | scales,
 * 1,185,792 bytes at the 35B-A3B shape), decoded as cb0[idx0] + cb1[idx1] (cb1: [256, 8]). add:
 * optional fp32 [T, H] added to the routing-weighted sum before the output conversion (the
 * regular experts' partial). Replaces the dense-bf16 promoted-expert path of reference
 * PagedMoEExpert (vq2/paged_runtime.py:357-389, 446-460) without dequantizing the weights.
 */
VQ2_API int vq2_moe_expert_ffn_res(const void* h, int h_dtype, int64_t T, int64_t top_k,
                                   const int32_t* ids, const float* w, const void* pool,
                                   int64_t num_experts, int64_t gu_rows, int64_t gu_cols,
                                   int64_t dn_rows, int64_t dn_cols, const void* cb0,
                                   const void* cb1, int val_dtype, const int32_t* perm_in,
                                   const int8_t* sign_in, int64_t hb_in, float scale_in,
                                   const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid,
                                   float scale_mid, const float* add, void* workspace,
                                   int64_t workspace_bytes, void* out, int out_dtype, void* stream);

/*
 * Router logits with the dense (unquantized) router weight: logits[t, e] = sum_i h[t, i] W[e, i],
 * fp32 accumulation. h: [T, H] in h_dtype; W: [E, H] in w_dtype (fp16/bf16); logits fp32
 * [T, E]; H % 8 == 0, h and W 16-byte aligned (rows of 16-byte multiples).
 * Replaces: the F.linear of Qwen3_5MoeTopKRouter.forward (installed transformers
 * modeling_qwen3_5_moe.py:762-764); the reference keeps the router dense (vq2/quantize_35b.py:139).
 */
VQ2_API int vq2_router_logits(const void* h, int h_dtype, int64_t T, const void* W, int w_dtype, int64_t E,
                              int64_t H, float* logits, void* stream);

/*
 * One sparse MoE layer from router logits, three launches on `stream`:
 *   1. one CTA: router (softmax over E, top_k by logit with ties to the lower id, weights
 *      renormalised over the selected), the shared expert's sigmoid gate, the mapping of expert
 *      ids to this rank's pool rows, the input RHT of every token (written once to the
 *      workspace) and the ordered list of (token, expert) problems computed here;
 *   2. gate_up GEMV over those problems;
 *   3. down GEMV (SwiGLU + RHT 512 in its prologue) whose epilogue also forms
 *      out[t] = sum_j w[t, j] * down_j(t) in problem order (the CTA completing a token's last
 *      problem in a row block sums it).
 * h: [T, H] in h_dtype (H = gu_cols * 8); logits: fp32 [T, E] (E <= 1024, top_k <= 32,
 * T <= 4096); shared_gate: fp32 [H] or NULL (no shared expert). Pool rows: experts
 * [expert_lo, expert_hi) at rows 0..hi-lo-1 and, with a shared gate, the shared expert at row
 * hi-lo; its problem for token t is computed on rank t % world (rank/world: 0/1 on one GPU).
 * Tokens with no problem on this rank get zero rows. Workspace: vq2_moe_layer_workspace bytes,
 * 256-byte aligned, no state kept between calls. out: [T, H] in out_dtype.
 * Replaces: Qwen3_5MoeSparseMoeBlock.forward's router + shared expert (installed transformers
 * modeling_qwen3_5_moe.py:762-791) around the reference's expert call
 * (vq2/load_and_test_full_35b.py:53-95, vq2/paged_runtime.py:439-511).
 */
VQ2_API int64_t vq2_moe_layer_workspace(int64_t T, int64_t top_k, int has_shared, int64_t hidden,
                                        int64_t gu_rows, int64_t dn_rows);
VQ2_API int vq2_moe_layer(const void* h, int h_dtype, int64_t T, const float* logits, int64_t E,
                          int64_t top_k, const float* shared_gate, int64_t expert_lo,
                          int64_t expert_hi, int rank, int world, const void* pool,
                          int64_t pool_rows, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows,
                          int64_t dn_cols, const void* cb0, int val_dtype, const int32_t* perm_in,
                          const int8_t* sign_in, int64_t hb_in, float scale_in,
                          const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid,
                          float scale_mid, void* workspace, int64_t workspace_bytes, void* out,
                          int out_dtype, void* stream);

/*
 * One small exchange among the ranks of a node over NVLink peer memory, one kernel (the
 * row-sharded lm_head's all-gather of hidden states and its cross-rank argmax):
 *   mode 0 (gather): dst = concat over ranks of each rank's `bytes` from src (rank order);
 *   mode 1 (argmax keys): src holds bytes/8 greedy keys of this rank's rows (as written by
 *     vq2_gemv_argmax); they are rebased to global rows (+ row_offset) and dst receives the
 *     elementwise maximum over ranks (global argmax, ties to the smaller row).
 * peers_dev: device array of `world` addresses of identical buffers of
 * vq2_peer_exchange_buffer_bytes(max_bytes, world) bytes (one per rank, peer-mapped, zeroed
 * before first use); state: local device int32 [1], zeroed before first use. bytes % 8 == 0,
 * bytes <= max_bytes. Every rank makes the same calls; a wait for a peer that gives up (after
 * max_polls polls; <= 0: about a second) raises *err (0x400) and the kernel uses what it has.
 * No counterpart in the reference (single GPU only); replaces the all_gather of logits or a
 * (max, idx) all-reduce of a row-sharded PackedLMHead (vq2/runtime.py:136-144).
 */
VQ2_API int64_t vq2_peer_exchange_buffer_bytes(int64_t max_bytes, int64_t world);
VQ2_API int vq2_peer_exchange(const void* src, int64_t bytes, int mode, int64_t row_offset,
                              void* const* peers_dev, int rank, int world, int64_t max_bytes,
                              int32_t* state, int32_t* err, int64_t max_polls, void* dst,
                              void* stream);

/*
 * Expert-parallel vq2_moe_expert_ffn whose combine also sums over the ranks of a group, in one
 * kernel over NVLink peer memory (instead of combine -> NCCL all_reduce -> cast). ids: this
 * rank's local pool rows (-1 for experts of other ranks). peers_dev: device array of `world`
 * addresses of identical symmetric buffers (one per rank, peer-mapped, vq2_moe_peer_buffer_bytes
 * bytes, zeroed before first use); epochs: local device uint32 [2] (sequence number, finished
 * CTAs), zeroed before first use.
 * Every rank must make the same sequence of calls (T <= max_tokens); a wait for a peer that
 * gives up (after max_polls polls of its flag; <= 0: about a second) raises *err (code 0x200)
 * and the kernel finishes with what it has. The output is identical on every rank.
 */
VQ2_API int64_t vq2_moe_peer_buffer_bytes(int64_t max_tokens, int64_t hidden, int64_t world);
VQ2_API int vq2_moe_expert_ffn_ep(const void* h, int h_dtype, int64_t T, int64_t top_k,
                                  const int32_t* ids, const float* w, const void* pool,
                                  int64_t num_experts, int64_t gu_rows, int64_t gu_cols,
                                  int64_t dn_rows, int64_t dn_cols, const void* cb0, int val_dtype,
                                  const int32_t* perm_in, const int8_t* sign_in, int64_t hb_in,
                                  float scale_in, const int32_t* perm_mid, const int8_t* sign_mid,
                                  int64_t hb_mid, float scale_mid, void* workspace,
                                  int64_t workspace_bytes, void* const* peers_dev, int rank,
                                  int world, int64_t max_tokens, uint32_t* epochs, int32_t* err,
                                  int64_t max_polls, void* out, int out_dtype, void* stream);

/*
 * Expert-parallel vq2_moe_layer: the same route / gate_up / down sequence on this rank's
 * experts, then the routing-weighted combine and the sum over the ranks in one kernel over
 * NVLink peer memory (peers_dev, err and max_tokens as vq2_moe_expert_ffn_ep; epochs: local
 * device int32 [4], zeroed before first use -- the combine's sequence number and CTA count and
 * the router's arrival counter). Every rank makes the same calls with the same logits and hidden
 * states; the output is identical on every rank.
 */
VQ2_API int vq2_moe_layer_ep(const void* h, int h_dtype, int64_t T, const float* logits, int64_t E,
                             int64_t top_k, const float* shared_gate, int64_t expert_lo,
                             int64_t expert_hi, const void* pool, int64_t pool_rows,
                             int64_t gu_rows, int64_t gu_cols, int64_t dn_rows, int64_t dn_cols,
                             const void* cb0, int val_dtype, const int32_t* perm_in,
                             const int8_t* sign_in, int64_t hb_in, float scale_in,
                             const int32_t* perm_mid, const int8_t* sign_mid, int64_t hb_mid,
                             float scale_mid, void* workspace, int64_t workspace_bytes,
                             void* const* peers_dev, int rank, int world, int64_t max_tokens,
                             uint32_t* epochs, int32_t* err, int64_t max_polls, void* out,
                             int out_dtype,
                             void* stream);

/* Workspace bytes vq2_moe_expert_ffn needs for T tokens x top_k experts (-1 on bad sizes). */
VQ2_API int64_t vq2_moe_expert_ffn_workspace(int64_t T, int64_t top_k, int64_t gu_rows,
                                             int64_t dn_rows);

/*
 * vq2_moe_expert_ffn without a workspace argument and without allocating anything, for
 * callers that cannot obtain device memory when they call: plugin or real-time interfaces whose
 * enqueue step must not allocate (an allocation can block on the device or fail mid-stream),
 * and hosts reaching the library through an FFI that have no device allocator of their own.
 * No counterpart in the reference (its PyTorch code always allocates).
 *
 * The intermediates live in a static device array of VQ2_MOE_FFN_NOALLOC_MAX_BYTES inside this
 * library, present on every GPU that loads it until the process exits. Limit: the call is
 * refused with VQ2_ERR_SHAPE when vq2_moe_expert_ffn_workspace(T, top_k, gu_rows, dn_rows)
 * exceeds that size (4 MiB: up to 340 (token, expert) problems at the 35B-A3B shape, e.g.
 * T = 32 at top-8 plus a shared expert). The first call on a device looks up the array's
 * device address with that device current and keeps it for the device; make that first call
 * before starting any stream capture. cudaDeviceReset discards the array with the context, so
 * after a reset the kept address is stale: do not call this entry point again in that process.
 * All calls share the array: calls that may run concurrently on the GPU (on streams with no
 * ordering between them) race on it and must be serialized by the caller. Each call overwrites
 * the intermediates in full before reading them; nothing needs clearing. It always runs the
 * four-kernel sequence (compaction, gate_up, down, combine). Otherwise identical to
 * vq2_moe_expert_ffn.
 */
#define VQ2_MOE_FFN_NOALLOC_MAX_BYTES (4u * 1024u * 1024u)
VQ2_API int vq2_moe_expert_ffn_noalloc(const void* h, int h_dtype, int64_t T, int64_t top_k,
                                       const int32_t* ids, const float* w, const void* pool,
                                       int64_t num_experts, int64_t gu_rows, int64_t gu_cols,
                                       int64_t dn_rows, int64_t dn_cols, const void* cb0,
                                       int val_dtype, const int32_t* perm_in,
                                       const int8_t* sign_in, int64_t hb_in, float scale_in,
                                       const int32_t* perm_mid, const int8_t* sign_mid,
                                       int64_t hb_mid, float scale_mid, void* out, int out_dtype,
                                       void* stream);

/*
 * Diagnostic: `blocks` x 256 threads each perform 8 * iters random 16-byte gathers of the rows
 * of a [65536, 8] fp16/bf16 codebook cb, with uniform random row indices, through
 *   mode 0: global memory (the GEMV's load form); rows <= 65536 limits the rows touched;
 *   mode 1: shared memory (each CTA stages the first 12,288 rows; rows must be 65536);
 *   mode 2: distributed shared memory of an 8-CTA cluster holding the whole table (rows 65536);
 *   modes 3 / 4: `blocks` x 1024 threads, each CTA holding one 8192-row bucket of the table and a
 *           2048-value activation row (fp32 / fp16) in shared memory; each of the 8 * iters steps
 *           is one bucketed GEMV entry (codeword read + activation read + 8-wide dot product).
 * Timing it gives the random codebook-gather rate that bounds the M = 1 VQ GEMV.
 * sink: one uint32 of device memory. No reference counterpart (measurement aid).
 */
VQ2_API int vq2_gather_probe(const void* cb, int64_t rows, int mode, int64_t blocks,
                             int64_t iters, uint32_t* sink, void* stream);

/*
 * ---- ANS-coded index streams ("VQ2A" interleaved rANS) ----
 * Replaces the entropy coding of vq2/export.py:26-36 (constriction AnsCoder over the index
 * bytes), which the reference runs on the host; here an ANS-coded container's index tensors
 * are byte streams that a paged miss copies to the device and vq2_rans_decode expands there.
 * Format (little-endian): u32 magic 0x41325156, u32 n_symbols, u32 n_chunks =
 * ceil(n_symbols / 8192), u32 0, u16 freq[2][256] (context = symbol position parity, each row
 * sums to 4096, no zero), u32 chunk_off[n_chunks + 1] (last = total size), zero pad to 16
 * bytes; chunk c = u32 state[64], u16 nwords[64], then the u16 words of stream 0, 1, ... in
 * decode order, zero pad to 16. Stream w codes chunk symbols w, w + 64, ...; rANS with 32-bit
 * state, L = 2^16, 16-bit words, 12-bit scale; a stream holds at most one word per symbol and
 * ends at state L with all its words used.
 */
/* Upper bound on the encoded size of n_symbols bytes (-1 if n_symbols is out of range). */
VQ2_API int64_t vq2_rans_bound(int64_t n_symbols);
/* Host encoder: symbols -> out (host memory, out_capacity >= vq2_rans_bound); *out_bytes = size. */
VQ2_API int vq2_rans_encode(const uint8_t* symbols, int64_t n_symbols, uint8_t* out,
                            int64_t out_capacity, int64_t* out_bytes);
/*
 * GPU decoder, asynchronous on `cuda_stream`: stream (device, stream_bytes long) -> out (device,
 * n_symbols <= out_capacity bytes). *status (device int32) must be zero before the first decode;
 * a malformed stream raises it to a nonzero code (1 magic, 2 counts, 3 frequencies, 4 chunk
 * offsets, 5 word counts, 6 words exhausted, 7 bad final state) and decodes never lower it, so
 * several decodes can share one status word that the caller reads after synchronizing. All
 * reads stay inside stream_bytes and all writes inside out[0, n_symbols) whatever the stream
 * holds. n_symbols = 0 decodes nothing and checks nothing.
 */
VQ2_API int vq2_rans_decode(const void* stream, int64_t stream_bytes, int64_t n_symbols,
                            void* out, int64_t out_capacity, int32_t* status, void* cuda_stream);
/*
 * One launch over 1..32 segments of src (device, src_bytes) into dst (device, dst_bytes):
 * segment i reads src[seg_src_off[i], + seg_src_bytes[i]) and writes dst[seg_dst_off[i],
 * + seg_n[i]); seg_kind 0 = a VQ2A stream of seg_n symbols, 1 = stored bytes (seg_src_bytes ==
 * seg_n, copied). The offset arrays are host memory. Status as for vq2_rans_decode. Used to
 * expand one ANS-coded expert record (compressed indices, stored scales) into its pool slot.
 */
VQ2_API int vq2_rans_decode_segments(const void* src, int64_t src_bytes,
                                     const int64_t* seg_src_off, const int64_t* seg_src_bytes,
                                     const int64_t* seg_dst_off, const int64_t* seg_n,
                                     const int32_t* seg_kind, int64_t nseg, void* dst,
                                     int64_t dst_bytes, int32_t* status, void* cuda_stream);

/*
 * ---- Paged MoE step (native executor) ----
 * One step of a paged MoE layer after the caller's LRU bookkeeping has chosen the slots
 * (reference PagedMoEExpert.forward, vq2/paged_runtime.py:439-568, with _get_slot :415-437 kept
 * on the host so hit/miss/slot sequences stay bit-exact):
 *   1. if n_miss > 0: copy_stream waits compute_done (earlier steps may still read the slots);
 *      record i (miss_bytes[i] bytes at host address miss_src[i], pinned for asynchrony) is
 *      copied to slot miss_slot[i] of the pool; copy_done is recorded and `stream` waits for it.
 *      With index_coding 1 (VQ2A-coded records) groups of up to 8 records are copied into one
 *      half of the staging buffer (halves taken in turn by *stage_turn, shared by the layers of
 *      one copy stream; a half is reused after stage_free0/1), and decode_stream (after
 *      stage_ready) expands each group in one launch into the slots following miss_seg (per
 *      record 4 segments of 5 int64: src_off, src_bytes, dst_off, n, kind, as
 *      vq2_rans_decode_segments); copy_done is then recorded on decode_stream;
 *   2. slots (host int32 [T * top_k]): up to 64 travel in the first kernel's launch parameters;
 *      more go through ids_host (pinned; the call first waits on the host for ids_done, the
 *      previous upload) to ids_dev on `stream`;
 *   3. the routed-expert FFN (as vq2_moe_expert_ffn, on the pool with capacity rows) runs on
 *      `stream` -- for T * top_k <= 64 at the 35B-A3B expert shape as ONE fused persistent
 *      kernel (gate_up, down and combine; work items handed out in dependency order, bounded
 *      waits), which costs the host one launch instead of four -- then compute_done is recorded.
 * All events must have been recorded once before the first call. Steps of one layer use one
 * `stream`. The workspace (vq2_moe_expert_ffn_workspace bytes) must be zeroed before the first
 * step and kept for this layer's steps: its first 1 KB holds counters of the fused FFN kernel,
 * which leaves them at zero. Decode errors raise *status (see vq2_rans_decode), as does (code
 * 0x100) a bounded wait of the fused FFN kernel that gave up.
 */
typedef struct vq2_paged_layer {
  void* pool;                      /* device [capacity, record bytes] expert records */
  int64_t capacity, gu_rows, gu_cols, dn_rows, dn_cols;
  const void* cb0;                 /* [65536, 8] in val_dtype */
  int32_t val_dtype, index_coding; /* index_coding: 0 raw records, 1 VQ2A-coded indices */
  const int32_t* perm_in;
  const int8_t* sign_in;
  int64_t hb_in;
  const int32_t* perm_mid;
  const int8_t* sign_mid;
  int64_t hb_mid;
  float scale_in, scale_mid;
  void* stage;                     /* device staging for coded records (index_coding 1) */
  int64_t stage_bytes;             /* two halves of up to 8 records each */
  int32_t* status;                 /* device decode status word (index_coding 1) */
  int64_t* stage_turn;             /* host counter shared with the other layers of copy_stream */
  void* decode_stream;             /* cudaStream_t (index_coding 1) */
  void* stage_ready;               /* cudaEvent_t (index_coding 1) */
  void* stage_free0;               /* cudaEvent_t (index_coding 1) */
  void* stage_free1;               /* cudaEvent_t (index_coding 1) */
  int32_t* ids_host;               /* pinned host int32 [ids_cap] */
  int32_t* ids_dev;                /* device int32 [ids_cap] */
  int64_t ids_cap;
  void* copy_stream;               /* cudaStream_t */
  void* copy_done;                 /* cudaEvent_t */
  void* compute_done;              /* cudaEvent_t */
  void* ids_done;                  /* cudaEvent_t */
} vq2_paged_layer;

VQ2_API int vq2_paged_moe_step(const vq2_paged_layer* layer, const void* h, int h_dtype, int64_t T,
                               int64_t top_k, const int32_t* slots, const float* w, int64_t n_miss,
                               const void* const* miss_src, const int64_t* miss_bytes,
                               const int32_t* miss_slot, const int64_t* miss_seg, void* workspace,
                               int64_t workspace_bytes, void* out, int out_dtype, void* stream);

/*
 * ---- Device-resident paging (T = 1 decode without host round trips) ----
 * The LRU decision of PagedMoEExpert._get_slot (vq2/paged_runtime.py:415-437) as a GPU kernel
 * and a fetch of missed records from the pinned host image by the SMs (zero-copy), so router ->
 * LRU -> fetch -> expert FFN of every layer can run in one CUDA graph.
 *
 * LRU state of one layer: int32 [vq2_lru_state_ints(E, cap)] = {head, tail, free count, hits,
 * misses, cap, E, error}, expert->slot [E] (-1 absent), prev [E], next [E], free-slot stack [cap]
 * (range(cap), top at the end). vq2_lru_step processes ids[0..K) in order (hit: move to most
 * recent; miss: pop a free slot, else evict the least recent), writes slots[K] and the miss
 * list miss = {count, expert[K], slot[K]} (int32 [1 + 2K]); it sets the error flag if a slot
 * needed earlier in the same step would be reused (capacity < K) -- bit-exact with the
 * reference for every step it accepts.
 */
VQ2_API int64_t vq2_lru_state_ints(int64_t num_experts, int64_t capacity);
VQ2_API int vq2_lru_step(int32_t* state, const int32_t* ids, int64_t K, int32_t* slots,
                         int32_t* miss, void* stream);
/*
 * Copy the records of a miss list into their pool slots: record e of the layer is rec_bytes at
 * image_dev + rec_off[e] (device int64 [num_experts]); image_dev is the device address of a
 * page-locked host image (vq2_host_device_pointer); rec_bytes % 16 == 0, 16-byte alignment.
 */
VQ2_API int vq2_fetch_records(const void* image_dev, const int64_t* rec_off, int64_t rec_bytes,
                              void* pool, int64_t capacity, const int32_t* miss, int64_t K,
                              int64_t num_experts, void* stream);
/* Device address of page-locked host memory (VQ2_ERR_ARG if it is not mapped). */
VQ2_API int vq2_host_device_pointer(const void* host, void** device_ptr);
/*
 * The routed-expert FFN of one token on the slots of a vq2_lru_step, with the fetch of the missed
 * records fused in: two launches (gate_up rows; down rows over all problems + the combine) that
 * read a record on this step's miss list straight from the page-locked image (image_dev +
 * rec_off[ids[k]]) and write it into its slot on the way, so the PCIe reads overlap the hits'
 * codebook gathers and no separate copy pass runs. Replaces vq2_fetch_records + the expert FFN
 * (the copy + compute of reference PagedMoEExpert.forward, vq2/paged_runtime.py:439-511, the
 * LRU decision staying in vq2_lru_step). ids, slots, miss, w: device arrays of the step (top_k
 * entries; miss as written by vq2_lru_step). Shapes: hidden 2048, expert intermediate 512
 * (RHT blocks 2048 / 512), top_k <= 8, 2 bpw records; others return VQ2_ERR_SHAPE. workspace:
 * vq2_paged_moe_t1_workspace(top_k) bytes. Outputs are bit-identical to the separate fetch + FFN.
 */
VQ2_API int64_t vq2_paged_moe_t1_workspace(int64_t top_k);
VQ2_API int vq2_paged_moe_t1(const void* h, int h_dtype, int64_t top_k, const int32_t* ids,
                             const int32_t* slots, const int32_t* miss, const float* w, const void* pool,
                             int64_t capacity, int64_t gu_rows, int64_t gu_cols, int64_t dn_rows,
                             int64_t dn_cols, const void* cb0, int val_dtype, const int32_t* perm_in,
                             const int8_t* sign_in, int64_t hb_in, float scale_in, const int32_t* perm_mid,
                             const int8_t* sign_mid, int64_t hb_mid, float scale_mid, const void* image_dev,
                             const int64_t* rec_off, int64_t num_experts, void* workspace,
                             int64_t workspace_bytes, void* out, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VQ2_B200_H */
