"""MoE expert path on VQ weights: router, resident expert pool, fused expert FFN.

One MoE layer from router logits is one C-ABI call (``vq2_moe_layer``), three launches:

1. the router kernel (one CTA for all T tokens): softmax top-k with renormalised weights, the
   shared expert's sigmoid gate, the mapping of expert ids to pool rows, the input RHT of every
   token (written once), and the ordered list of (token, expert) problems;
2. the gate_up GEMV over those problems, into fp32 [P, 1024];
3. the down GEMV with SwiGLU + the 512-point RHT in its prologue and the routing-weighted sum of
   each token's problems in its epilogue (the CTA completing a token's last problem of a row
   block sums it, in problem order).

The reference runs the same math as rot_2048.fwd -> 2-D-grid Triton gate_up -> torch SiLU*up ->
rot_512.fwd -> Triton down -> torch weighted sum (vq2/paged_runtime.py:491-511;
vq2/load_and_test_full_35b.py:53-74), with a Python loop over tokens for T > 1 (:512-568 /
:75-95), around the transformers router (modeling_qwen3_5_moe.py:762-791).

``expert_ffn`` (vq2_moe_expert_ffn) keeps the form that takes routed ids and weights, as the
reference's expert modules do (``PackedMoEExpertUniversal.forward``, the paged runtime).

Experts are stored as whole records [gu_idx int16 1024x256 | gu_scale fp16 1024 | dn_idx int16
2048x64 | dn_scale fp16 2048] (792,576 B), the .vq2m payload layout, so a pool is one
[E, 792576] byte tensor and paging an expert is one copy.
"""
import torch
import torch.nn as nn

from . import _lib, kernels, vq
from .synth import DN_COLS, DN_ROWS, GU_COLS, GU_ROWS


class ExpertRecordPool:
    """Device (or host) tensor of E expert records plus typed strided views into it:
    gu_idx [E, gu_rows, gu_cols], gu_scale [E, gu_rows], dn_idx [E, dn_rows, dn_cols],
    dn_scale [E, dn_rows]."""

    def __init__(self, E, device, gu_rows=GU_ROWS, gu_cols=GU_COLS, dn_rows=DN_ROWS, dn_cols=DN_COLS,
                 buf=None):
        self.dims = (gu_rows, gu_cols, dn_rows, dn_cols)
        o1 = gu_rows * gu_cols
        o2 = o1 + gu_rows
        o3 = o2 + dn_rows * dn_cols
        o4 = o3 + dn_rows
        self.record_bytes = 2 * o4
        if (2 * o3) % 16 or self.record_bytes % 16:
            raise ValueError("expert record layout breaks 16-byte alignment")
        self.E = E
        self.raw = buf if buf is not None else torch.empty(E, self.record_bytes, dtype=torch.uint8, device=device)
        if self.raw.shape != (E, self.record_bytes):
            raise ValueError("record buffer shape mismatch")
        w = self.raw.view(torch.int16)
        self.gu_idx = w[:, :o1].view(E, gu_rows, gu_cols)
        self.gu_scale = w[:, o1:o2].view(torch.float16)
        self.dn_idx = w[:, o2:o3].view(E, dn_rows, dn_cols)
        self.dn_scale = w[:, o3:o4].view(torch.float16)

    def set_expert(self, e, gu_idx, gu_scale, dn_idx, dn_scale):
        self.gu_idx[e].copy_(torch.as_tensor(gu_idx))
        self.gu_scale[e].copy_(torch.as_tensor(gu_scale).to(torch.float16))
        self.dn_idx[e].copy_(torch.as_tensor(dn_idx))
        self.dn_scale[e].copy_(torch.as_tensor(dn_scale).to(torch.float16))


class Expert3Pool:
    """Resident pool of promoted 3 bpw expert records (reference expert_modes == 3; record =
    gu idx0 int16 | gu idx1 uint8 | gu scale fp16 | dn idx0 int16 | dn idx1 uint8 | dn scale fp16,
    1,185,792 B at the 35B-A3B shape, tools/build_mixed_b2_container.py:50-80)."""

    def __init__(self, E, device, gu_rows=GU_ROWS, gu_cols=GU_COLS, dn_rows=DN_ROWS, dn_cols=DN_COLS):
        self.dims = (gu_rows, gu_cols, dn_rows, dn_cols)
        self.E = E
        self.record_bytes = 3 * gu_rows * gu_cols + 2 * gu_rows + 3 * dn_rows * dn_cols + 2 * dn_rows
        self.raw = torch.zeros(max(E, 1), self.record_bytes, dtype=torch.uint8, device=device)

    def set_record(self, e, rec):
        """Copy one stored 3 bpw record (host bytes, in container order) into row e."""
        self.raw[e].copy_(torch.as_tensor(rec).reshape(-1))


def expert_ffn_res(hidden, ids, weights, pool3, cb16, cb8, rot_in, rot_mid, top_k, add=None, out=None,
                   out_dtype=None):
    """expert_ffn over a pool of 3 bpw expert records (vq2_moe_expert_ffn_res): ids index rows of
    ``pool3`` (-1 = not in this pool); ``add`` (fp32 [T, H]) is added before the output cast."""
    _lib.require_cuda(hidden, ids, weights, cb16, cb8)
    T, H = hidden.shape
    gr, gc, dr, dc = pool3.dims
    h = hidden.contiguous()
    ids = ids.contiguous()
    w = weights.float().contiguous()
    out_dtype = out_dtype or hidden.dtype
    if out is None:
        out = torch.empty(T, H, dtype=out_dtype, device=h.device)
    addc = add.float().contiguous() if add is not None else None
    lib = _lib.load()
    ws_bytes = lib.vq2_moe_expert_ffn_workspace(T, top_k, gr, dr)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=h.device)
    _lib.call("vq2_moe_expert_ffn_res", _lib.ptr(h), _lib.dtype_code(h), T, top_k, _lib.ptr(ids), _lib.ptr(w),
              _lib.ptr(pool3.raw), pool3.E, gr, gc, dr, dc, _lib.ptr(cb16), _lib.ptr(cb8), _lib.dtype_code(cb16),
              _lib.ptr(rot_in.perm), _lib.ptr(rot_in.sign), rot_in.hb, float(rot_in.scale), _lib.ptr(rot_mid.perm),
              _lib.ptr(rot_mid.sign), rot_mid.hb, float(rot_mid.scale),
              _lib.ptr(addc) if addc is not None else None, _lib.ptr(ws), ws_bytes, _lib.ptr(out),
              _lib.dtype_code(out), _lib.stream_ptr(h.device))
    return out


def route(logits, top_k=8, hidden=None, shared_gate=None):
    """Router on device logits fp32 [T, E] -> (ids int32 [T, top_k], w fp32 [T, top_k]
    [, shared_w fp32 [T]]); the math of Qwen3_5MoeTopKRouter (softmax, topk, renormalise) and
    the shared expert's sigmoid gate."""
    _lib.require_cuda(logits, hidden, shared_gate)
    lg = logits.float().contiguous()
    T, E = lg.shape
    ids = torch.empty(T, top_k, dtype=torch.int32, device=lg.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=lg.device)
    sw = None
    h = None
    if shared_gate is not None:
        h = hidden.reshape(T, -1).contiguous()
        g = shared_gate.reshape(-1).float().contiguous()
        sw = torch.empty(T, dtype=torch.float32, device=lg.device)
    _lib.call("vq2_moe_route", _lib.ptr(lg), T, E, top_k, _lib.ptr(ids), _lib.ptr(w),
              _lib.ptr(h) if h is not None else None, _lib.dtype_code(h) if h is not None else 0,
              _lib.ptr(g) if shared_gate is not None else None, h.shape[1] if h is not None else 0,
              _lib.ptr(sw) if sw is not None else None, _lib.stream_ptr(lg.device))
    return (ids, w) if sw is None else (ids, w, sw)


def expert_ffn(hidden, ids, weights, pool, cb16, rot_in, rot_mid, top_k, out=None, out_dtype=None):
    """sum_j w[t, j] * Expert_{ids[t*top_k + j]}(h[t]) for T tokens: one C-ABI call
    (vq2_moe_expert_ffn, three launches) with its fp32 intermediates in a workspace from the
    caching allocator.

    hidden: [T, H]; ids: int32 [T*top_k] device (pool rows: expert ids or slots); weights:
    fp32 [T, top_k]; pool: ExpertRecordPool on the device."""
    _lib.require_cuda(hidden, ids, weights, cb16)
    T, H = hidden.shape
    gr, gc, dr, dc = pool.dims
    if H != rot_in.n or gr // 2 != rot_mid.n or ids.numel() != T * top_k or ids.dtype != torch.int32:
        raise ValueError("shape/dtype mismatch between hidden, ids, rotations and the expert pool")
    if cb16.dtype != torch.float16:
        raise ValueError("the expert pools hold fp16 scales; the codebook must be fp16")
    h = hidden.contiguous()
    ids = ids.contiguous()
    w = weights.float().contiguous()
    out_dtype = out_dtype or hidden.dtype
    if out is None:
        out = torch.empty(T, H, dtype=out_dtype, device=h.device)
    lib = _lib.load()
    ws_bytes = lib.vq2_moe_expert_ffn_workspace(T, top_k, gr, dr)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=h.device)
    _lib.call("vq2_moe_expert_ffn", _lib.ptr(h), _lib.dtype_code(h), T, top_k, _lib.ptr(ids), _lib.ptr(w),
              _lib.ptr(pool.raw), pool.E, gr, gc, dr, dc, _lib.ptr(cb16), _lib.dtype_code(cb16),
              _lib.ptr(rot_in.perm), _lib.ptr(rot_in.sign), rot_in.hb, float(rot_in.scale),
              _lib.ptr(rot_mid.perm), _lib.ptr(rot_mid.sign), rot_mid.hb, float(rot_mid.scale),
              _lib.ptr(ws), ws_bytes, _lib.ptr(out), _lib.dtype_code(out), _lib.stream_ptr(h.device))
    return out


class PackedMoEExpertUniversal(nn.Module):
    """All experts resident in HBM (reference vq2/load_and_test_full_35b.py:26-95):
    forward(hidden_states [T, 2048], topk_idx [T, k], topk_weights [T, k]) -> [T, 2048].
    The pool holds the 256 routed experts (+ the shared expert as row E when given)."""

    def __init__(self, pool, cb16, device="cuda", shared=False):
        super().__init__()
        self.pool = pool
        self.num_experts = pool.E - (1 if shared else 0)
        self.shared = shared
        self.cb16 = cb16
        self.hidden_dim = pool.dims[1] * 8
        self.intermediate_dim = pool.dims[0] // 2
        self.rot_2048 = vq.get_rot("moe_expert_2048", self.hidden_dim, device)
        self.rot_512 = vq.get_rot("moe_expert_512", self.intermediate_dim, device)

    def forward(self, hidden_states, topk_idx, topk_weights, shared_weight=None):
        T = hidden_states.shape[0]
        k = topk_idx.shape[-1]
        ids = topk_idx.reshape(T, k).to(torch.int32)
        w = topk_weights.reshape(T, k).float()
        if self.shared and shared_weight is not None:
            ids = torch.cat([ids, torch.full((T, 1), self.num_experts, dtype=torch.int32, device=ids.device)], 1)
            w = torch.cat([w, shared_weight.reshape(T, 1).float()], 1)
            k += 1
        return expert_ffn(hidden_states.reshape(T, -1), ids.reshape(-1).contiguous(), w, self.pool, self.cb16,
                          self.rot_2048, self.rot_512, k)


def moe_layer(hidden, logits, pool, cb16, rot_in, rot_mid, top_k=8, shared_gate=None, lo=0, hi=None, rank=0,
              world=1, out=None, out_dtype=None, peer=None):
    """One sparse MoE layer from router logits (vq2_moe_layer; vq2_moe_layer_ep with ``peer``).

    hidden [T, H]; logits fp32 [T, E]; pool rows: experts [lo, hi) then, when ``shared_gate``
    (fp32 [H]) is given, the shared expert; its problem for token t runs on rank t % world.
    ``peer`` (ep.PeerReduceContext): the combine also sums the ranks' partials over NVLink peer
    memory. Returns out [T, H] (hidden's dtype unless ``out_dtype``)."""
    _lib.require_cuda(hidden, logits, cb16, shared_gate)
    T, H = hidden.shape
    E = logits.shape[-1]
    hi = E if hi is None else hi
    gr, gc, dr, dc = pool.dims
    if H != rot_in.n or gr // 2 != rot_mid.n or gc * 8 != H:
        raise ValueError("shape mismatch between hidden, rotations and the expert pool")
    if cb16.dtype != torch.float16:
        raise ValueError("the expert pools hold fp16 scales; the codebook must be fp16")
    h = hidden.contiguous()
    lg = logits.float().contiguous()
    g = shared_gate.reshape(-1).float().contiguous() if shared_gate is not None else None
    out_dtype = out_dtype or hidden.dtype
    if out is None:
        out = torch.empty(T, H, dtype=out_dtype, device=h.device)
    lib = _lib.load()
    ws_bytes = lib.vq2_moe_layer_workspace(T, top_k, int(g is not None), H, gr, dr)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=h.device)
    common = (_lib.ptr(pool.raw), pool.E, gr, gc, dr, dc, _lib.ptr(cb16), _lib.dtype_code(cb16),
              _lib.ptr(rot_in.perm), _lib.ptr(rot_in.sign), rot_in.hb, float(rot_in.scale),
              _lib.ptr(rot_mid.perm), _lib.ptr(rot_mid.sign), rot_mid.hb, float(rot_mid.scale),
              _lib.ptr(ws), ws_bytes)
    if peer is None:
        _lib.call("vq2_moe_layer", _lib.ptr(h), _lib.dtype_code(h), T, _lib.ptr(lg), E, top_k, _lib.ptr(g), lo, hi,
                  rank, world, *common, _lib.ptr(out), _lib.dtype_code(out), _lib.stream_ptr(h.device))
    else:
        import ctypes
        _lib.call("vq2_moe_layer_ep", _lib.ptr(h), _lib.dtype_code(h), T, _lib.ptr(lg), E, top_k, _lib.ptr(g), lo, hi,
                  *common, ctypes.c_void_p(peer.peers_dev), peer.rank, peer.world, peer.max_tokens,
                  _lib.ptr(peer.epochs), _lib.ptr(peer.err), int(getattr(peer, "max_polls", 0)), _lib.ptr(out),
                  _lib.dtype_code(out),
                  _lib.stream_ptr(h.device))
    return out


def router_logits_fn(hidden, weight, out=None):
    """logits fp32 [T, E] = hidden [T, H] . weight [E, H]^T with the dense router weight
    (vq2_router_logits; Qwen3_5MoeTopKRouter's F.linear)."""
    _lib.require_cuda(hidden, weight)
    h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    w = weight.contiguous()
    T, H = h.shape
    E = w.shape[0]
    if out is None:
        out = torch.empty(T, E, dtype=torch.float32, device=h.device)
    _lib.call("vq2_router_logits", _lib.ptr(h), _lib.dtype_code(h), T, _lib.ptr(w), _lib.dtype_code(w), E, H,
              _lib.ptr(out), _lib.stream_ptr(h.device))
    return out


class MoEBlock(nn.Module):
    """Sparse MoE block (Qwen3_5MoeSparseMoeBlock math) on VQ experts: router from logits (or a
    dense router weight), top-k routed experts + the always-on shared expert weighted by
    sigmoid(shared_gate . h), all resident; one vq2_moe_layer call (three launches) per layer."""

    def __init__(self, experts, router_weight=None, shared_gate=None, top_k=8):
        super().__init__()
        self.experts = experts
        self.router_weight = router_weight
        self.shared_gate = shared_gate
        self.top_k = top_k

    def forward(self, hidden_states, router_logits=None):
        if router_logits is None:
            router_logits = router_logits_fn(hidden_states, self.router_weight)
        ex = self.experts
        gate = self.shared_gate if (self.shared_gate is not None and ex.shared) else None
        return moe_layer(hidden_states, router_logits, ex.pool, ex.cb16, ex.rot_2048, ex.rot_512, self.top_k,
                         shared_gate=gate, lo=0, hi=ex.num_experts)
