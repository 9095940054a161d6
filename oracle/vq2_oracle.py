"""CPU oracle for the VQ2 decode hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this module, and only as the checker or the timed CPU baseline. The product path
(``compressai_b200``) never imports it and has no CPU fallback.

Every function restates, in numpy (fp64 unless stated), an algorithm of the reference
project Unoalss/CompressAI; the docstrings cite the reference file:line they follow. The
oracle is pinned against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``; checked by ``tests/test_oracle_golden.py``).

The only non-numpy dependency is torch's CPU random generator, which the reference uses to
draw each rotation's permutation and signs (``vq2/vq.py:51-54``); the same generator is the
only way to reproduce those draws bit for bit.
"""
import hashlib
import struct
from collections import OrderedDict

import numpy as np

D = 8        # vector dimension (vq2/vq.py:15)
HB = 2048    # Hadamard block (vq2/vq.py:16)


# --------------------------------------------------------------------------------------------
# Rotation (randomized Hadamard transform)
# --------------------------------------------------------------------------------------------
def tag_seed(tag):
    """int(md5(tag)[:8], 16) -- vq2/vq.py:40-41."""
    return int(hashlib.md5(tag.encode()).hexdigest()[:8], 16)


def rot_hb(n):
    """Hadamard block size rule of Rot.__init__ -- vq2/vq.py:48-49."""
    m = min(HB, n)
    hb = m if (n % m == 0 and (m & (m - 1)) == 0) else HB
    assert n % hb == 0, f"n={n} is not a multiple of hb={hb}"
    return hb


def rot_params(tag, n):
    """(perm int64[n], sign float64[n] of +-1, hb) drawn like Rot.__init__ -- vq2/vq.py:47-57."""
    import torch
    g = torch.Generator().manual_seed(tag_seed(tag))
    perm = torch.randperm(n, generator=g).numpy().astype(np.int64)
    sign = (torch.randint(0, 2, (n,), generator=g).double() * 2 - 1).numpy()
    return perm, sign, rot_hb(n)


def hadamard(n):
    """Sylvester Hadamard matrix H_{2k} = [[H, H], [H, -H]] -- vq2/vq.py:22-27."""
    assert n & (n - 1) == 0
    H = np.ones((1, 1))
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return H


def rht_fwd(x, perm, sign, hb):
    """x' = blockH(x[..., perm] * sign) * hb^-0.5 on the last dim -- Rot._orig_fwd/_blk,
    vq2/vq.py:66-76 (Rot.fwd, :78-82, computes the same map)."""
    x = np.asarray(x, dtype=np.float64)
    y = x[..., perm] * sign
    sh = y.shape
    y = y.reshape(*sh[:-1], sh[-1] // hb, hb) @ hadamard(hb)
    return (y * hb ** -0.5).reshape(sh)


def rht_inv(y, perm, sign, hb):
    """Inverse rotation -- Rot.inv, vq2/vq.py:84-87."""
    y = np.asarray(y, dtype=np.float64)
    sh = y.shape
    z = (y.reshape(*sh[:-1], sh[-1] // hb, hb) @ hadamard(hb)) * hb ** -0.5
    z = z.reshape(sh) * sign
    out = np.empty_like(z)
    out[..., perm] = z
    return out


# --------------------------------------------------------------------------------------------
# Dequantize-then-matmul (the reference's definition of the GEMV)
# --------------------------------------------------------------------------------------------
def cfg_keys(cfg):
    """Codebook keys per stage: "16", "16_8" -- vq.cfg_key, vq2/vq.py:109-110."""
    return ["_".join(str(b) for b in cfg[: i + 1]) for i in range(len(cfg))]


def as_index(a, bits):
    """Stored indices -> codebook rows; 16-bit stages are int16 holding uint16 bits
    (runtime._as_index, vq2/runtime.py:32-35; kernels.py:47,72 mask with 0xFFFF)."""
    a = np.asarray(a).astype(np.int64)
    return a & 0xFFFF if bits > 8 else a


def rotated_rows(idx_list, cfg, cbs, scale):
    """Q = (sum_i cb_i[idx_i]) * scale[:, None], the rotated-space weight rows --
    QMat.dequant, vq2/vq.py:283-290."""
    out, ng = np.asarray(idx_list[0]).shape
    rec = 0
    for i, key in enumerate(cfg_keys(cfg)):
        cb = np.asarray(cbs[key], dtype=np.float64)
        rec = rec + cb[as_index(idx_list[i], cfg[i])]
    return rec.reshape(out, ng * D) * np.asarray(scale, dtype=np.float64)[:, None]


def dequant(idx_list, cfg, cbs, scale, perm, sign, hb):
    """W = Rot.inv(Q) -- QMat.dequant, vq2/vq.py:283-292 (fp64 here)."""
    return rht_inv(rotated_rows(idx_list, cfg, cbs, scale), perm, sign, hb)


def gemv_ref(x, idx_list, cfg, cbs, scale, perm, sign, hb):
    """y = x . W^T with W = QMat.dequant(...) -- the dequantize-then-matmul of
    PackedLinear's generic path (vq2/runtime.py:82-89,105-110). Uses x.W^T = fwd(x).Q^T
    (Rot is orthogonal) so large matrices need no n x n inverse rotation."""
    xr = rht_fwd(np.asarray(x, dtype=np.float64), perm, sign, hb)
    Q = rotated_rows(idx_list, cfg, cbs, scale)
    return xr @ Q.T


def vq_gemv_legacy(xr, idx0, cb0, scale, rs, idx1=None, cb1=None):
    """y = rs * scale * sum_g (cb0[i0] (+cb1[i1])) . xr[g] on a PRE-ROTATED xr --
    _vq_gemv_16 / _vq_gemv_16_8, vq2/kernels.py:32-78."""
    idx0 = as_index(idx0, 16)
    out, ng = idx0.shape
    xg = np.asarray(xr, dtype=np.float64).reshape(ng, D)
    rec = np.asarray(cb0, dtype=np.float64)[idx0]
    if idx1 is not None:
        rec = rec + np.asarray(cb1, dtype=np.float64)[np.asarray(idx1).astype(np.int64)]
    acc = np.einsum("org,rg->o", rec, xg)
    return acc * np.asarray(scale, dtype=np.float64) * rs


def moe_gate_up_ref(xr, slots, pool_idx, cb16, pool_scale, rs=1.0):
    """Per active expert k: y[k] = rs * sc * sum cb16[idx] . xr -- vq_moe_parallel_gate_up_cpu,
    vq2/paged_runtime.py:19-29 (fp64 here)."""
    return np.stack([vq_gemv_legacy(xr, pool_idx[s], cb16, pool_scale[s], rs) for s in slots])


def moe_down_ref(act_r, slots, pool_idx, cb16, pool_scale, rs=1.0):
    """Per active expert k, its own activation row -- vq_moe_parallel_down_cpu,
    vq2/paged_runtime.py:31-41 (fp64 here)."""
    return np.stack([vq_gemv_legacy(act_r[k], pool_idx[s], cb16, pool_scale[s], rs)
                     for k, s in enumerate(slots)])


# --------------------------------------------------------------------------------------------
# MoE layer
# --------------------------------------------------------------------------------------------
def router_ref(logits, top_k=8):
    """softmax(fp32) -> topk -> renormalise, as transformers Qwen3_5MoeTopKRouter.forward
    (modeling_qwen3_5_moe.py:762-770 of the installed transformers 5.5.0). Uses the same torch
    CPU ops so ids and fp32 weights are those of the reference router."""
    import torch
    lg = torch.as_tensor(np.asarray(logits, dtype=np.float32))
    p = torch.nn.functional.softmax(lg, dtype=torch.float, dim=-1)
    v, i = torch.topk(p, top_k, dim=-1)
    v = v / v.sum(dim=-1, keepdim=True)
    return i.numpy().astype(np.int64), v.numpy()


def silu(v):
    return v / (1.0 + np.exp(-v))


def moe_layer_ref(h, ids, w, experts, cb16, rot2048, rot512, shared=None, shared_w=None, cb8=None):
    """One MoE layer for T tokens, fp64: per token, per selected expert, gate_up -> silu(gate)*up
    -> RHT512 -> down, then the routing-weighted sum -- PagedMoEExpert.forward,
    vq2/paged_runtime.py:491-511 (T=1) and :553-566 (T>1), with the CPU expert kernels
    (:19-41) and Rot.fwd (vq.py:78-82). ``experts(e)`` returns (gu_idx, gu_scale, dn_idx,
    dn_scale), or for a promoted 3 bpw expert (gu_idx0, gu_idx1, gu_scale, dn_idx0, dn_idx1,
    dn_scale) decoded as cb16[idx0] + cb8[idx1] (reference PagedMoEExpert promoted path,
    vq2/paged_runtime.py:357-389, 446-460, here without the bf16 rounding of its dense weights).
    ``shared`` (same tuple) with per-token weight ``shared_w`` adds the always-on shared expert as
    Qwen3_5MoeSparseMoeBlock.forward does (modeling_qwen3_5_moe.py:781-791)."""
    h = np.asarray(h, dtype=np.float64)
    T = h.shape[0]
    out = np.zeros((T, h.shape[1]))
    for t in range(T):
        xr = rht_fwd(h[t], *rot2048)
        plist = [(experts(int(e)), float(wk)) for e, wk in zip(ids[t], w[t])]
        if shared is not None:
            plist.append((shared, float(shared_w[t])))
        for ex, wk in plist:
            if len(ex) == 6:
                gu_i, gu_i1, gu_s, dn_i, dn_i1, dn_s = ex
            else:
                (gu_i, gu_s, dn_i, dn_s), gu_i1, dn_i1 = ex, None, None
            y_gu = vq_gemv_legacy(xr, gu_i, cb16, gu_s, 1.0, gu_i1, cb8)
            half = y_gu.shape[0] // 2
            act = silu(y_gu[:half]) * y_gu[half:]
            act_r = rht_fwd(act, *rot512)
            out[t] += wk * vq_gemv_legacy(act_r, dn_i, cb16, dn_s, 1.0, dn_i1, cb8)
    return out


# --------------------------------------------------------------------------------------------
# LRU expert cache (host decision, must be bit-exact)
# --------------------------------------------------------------------------------------------
class LRUSlotOracle:
    """Slot assignment of PagedMoEExpert._get_slot, vq2/paged_runtime.py:415-437:
    hit -> move_to_end; miss -> free_slots.pop() (LIFO over range(capacity)) else evict the
    least recently used (popitem(last=False)) and reuse its slot."""

    def __init__(self, capacity):
        self.capacity = capacity
        self.expert_to_slot = {}
        self.free_slots = list(range(capacity))
        self.access_order = OrderedDict()
        self.hits = 0
        self.misses = 0
        self.activated = set()

    def get_slot(self, e):
        self.activated.add(e)
        if e in self.expert_to_slot:
            self.hits += 1
            self.access_order.move_to_end(e)
            return self.expert_to_slot[e], True
        self.misses += 1
        if self.free_slots:
            slot = self.free_slots.pop()
        else:
            ev, _ = self.access_order.popitem(last=False)
            slot = self.expert_to_slot.pop(ev)
        self.expert_to_slot[e] = slot
        self.access_order[e] = None
        return slot, False


# --------------------------------------------------------------------------------------------
# .vq2m container
# --------------------------------------------------------------------------------------------
VQ2M_HEADER = "<4sHHHH QQQQQ 12s"   # vq2/paged_runtime.py:94, vq2/pack_35b_to_vq2m.py:236-242
VQ2M_ENTRY = "<QIQIQIQI"            # vq2/paged_runtime.py:45, vq2/pack_35b_to_vq2m.py:24


def parse_vq2m(buf):
    """Header + per-layer expert table + JSON meta -- PagedModelStore.__init__,
    vq2/paged_runtime.py:89-123."""
    import json
    (magic, version, nl, ne, _, toff, tlen, moff, mlen, pstart, _) = struct.unpack(VQ2M_HEADER, buf[:64])
    if magic != b"VQ2M" or version != 1:
        raise ValueError("invalid .vq2m")
    ents = list(struct.iter_unpack(VQ2M_ENTRY, buf[toff:toff + tlen]))
    table = [ents[ln * ne:(ln + 1) * ne] for ln in range(nl)]
    meta = json.loads(bytes(buf[moff:moff + mlen]).decode("utf-8"))
    return dict(num_layers=nl, num_experts=ne, payload_start=pstart, table=table, meta=meta)
