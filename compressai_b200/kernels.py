"""Kernel entry points with the signatures of reference ``vq2/kernels.py``, backed by the sm_100a
C-ABI library (no Triton, no CPU fallback).

Reference-compatible functions (same argument order and meaning):
  vq_gemv_16(xr, i0, cb0, scale, out, n, rs=1.0) -> y[out]               (kernels.py:224-230)
  vq_gemv_16_8(xr, i0, i1, cb0, cb1, scale, out, n, rs=1.0) -> y[out]    (kernels.py:215-221)
  vq_moe_parallel_gate_up(xr, topk_ids, gate_up_idx, cb16, gate_up_scale, y_out,
                          OUT=1024, NG=256, rs=1.0)                      (kernels.py:246-254)
  vq_moe_parallel_down(act_r, topk_ids, down_idx, cb16, down_scale, y_out,
                       OUT=2048, NG=64, rs=1.0)                          (kernels.py:256-264)
Differences: the output dtype is the codebook's dtype (the reference always returns bf16,
because its codebooks are bf16); xr may be fp32/fp16/bf16; any number of leading rows of xr
is accepted by the dense GEMVs (the reference's Triton path is batch-1 only).

Extra entry points used by the runtime: ``vq_gemv`` (batched, any output dtype),
``gemv_multi`` (several matrices sharing one activation, with the input RHT or SwiGLU+RHT
fused into the kernel prologue), ``moe_gemv``, ``swiglu_rht`` and ``moe_combine``.
"""
import ctypes

import torch

from . import _lib

HAVE_TRITON = _lib.available()   # name kept for importers: "fused GPU kernels available"
TC_MIN_ROWS = 4                  # activation rows from which the tensor-core GEMV is used
HAVE_CUDA_KERNELS = HAVE_TRITON
FUSED_KERNELS_ENABLED = True


def patch_transformers_kernels():
    """Kept so the reference's callers import unchanged (vq2/kernels.py:572): the reference swaps
    its Triton kernels into the transformers attention / DeltaNet / norm blocks here. Those blocks
    are outside this library's decode path (they run as the transformers modules), so this leaves
    them untouched and returns False."""
    return False


def optimize_deltanet_layers(model):
    """Kept for import compatibility (vq2/kernels.py:443): the reference fuses the DeltaNet input
    projections for its Triton path; with VQ weights those projections are PackedLinear modules
    already, so the model is returned unchanged."""
    return model


def set_fused_kernels_enabled(enabled: bool):
    """Kept for API compatibility (vq2/kernels.py:16-20); the CUDA kernels are always used."""
    global FUSED_KERNELS_ENABLED
    FUSED_KERNELS_ENABLED = bool(enabled)


def _check_vals(*ts):
    dt = ts[0].dtype
    if dt not in (torch.float16, torch.bfloat16):
        raise ValueError(f"codebook/scale dtype must be float16 or bfloat16, got {dt}")
    for t in ts[1:]:
        if t is not None and t.dtype != dt:
            raise ValueError(f"codebooks and scales must share one dtype ({dt} vs {t.dtype})")


def _c(t):
    return t if t is None or t.is_contiguous() else t.contiguous()


def vq_gemv(xr, i0, cb0, scale, i1=None, cb1=None, rs=1.0, out_dtype=None, y=None):
    """y[..., out] = rs * scale * sum_g (cb0[i0] (+cb1[i1])) . xr  for pre-rotated xr [..., n].

    fp32 accumulation; ``out_dtype`` defaults to the codebook dtype."""
    _lib.require_cuda(xr, i0, i1, cb0, cb1, scale)
    if i0.dtype != torch.int16 or (i1 is not None and i1.dtype != torch.uint8):
        raise ValueError("indices must be int16 (stage 1) and uint8 (residual)")
    _check_vals(cb0, cb1, scale)
    out, ng = i0.shape
    n = ng * 8
    if xr.shape[-1] != n:
        raise ValueError(f"xr last dim {xr.shape[-1]} != n={n}")
    x2 = xr.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    out_dtype = out_dtype or cb0.dtype
    if y is None:
        y = torch.empty(*xr.shape[:-1], out, dtype=out_dtype, device=xr.device)
    elif y.dtype != out_dtype or not y.is_contiguous():
        raise ValueError("y must be contiguous with dtype out_dtype")
    i0, i1, cb0, cb1, scale = _c(i0), _c(i1), _c(cb0), _c(cb1), _c(scale)
    ws = _workspace(M, n, xr.device)
    _lib.call("vq2_gemv", _lib.ptr(x2), _lib.dtype_code(x2), M, x2.stride(0), _lib.ptr(i0), _lib.ptr(i1),
              _lib.ptr(cb0), _lib.ptr(cb1), _lib.ptr(scale), _lib.dtype_code(cb0), _lib.ptr(y),
              _lib.dtype_code(y), out, out, n, float(rs), _lib.ptr(ws), ws.numel() if ws is not None else 0,
              _lib.stream_ptr(xr.device))
    return y


def _workspace(M, n, device):
    """Device workspace of the batched (tensor-core) GEMV, from the caching allocator."""
    nb = _lib.load().vq2_gemv_workspace(M, n)
    return torch.empty(nb, dtype=torch.uint8, device=device) if nb > 0 else None


def vq_gemv_16_8(xr, i0, i1, cb0, cb1, scale, out, n, rs=1.0):
    """3 bpw GEMV (stage-16 + residual-8 codebooks) -- vq2/kernels.py:215-221."""
    if i0.shape != (out, n // 8):
        raise ValueError(f"i0 shape {tuple(i0.shape)} != ({out}, {n // 8})")
    return vq_gemv(xr.reshape(-1, n), i0, cb0, scale, i1=i1, cb1=cb1, rs=rs).reshape(*xr.shape[:-1], out)


def vq_gemv_16(xr, i0, cb0, scale, out, n, rs=1.0):
    """2 bpw GEMV -- vq2/kernels.py:224-230."""
    if i0.shape != (out, n // 8):
        raise ValueError(f"i0 shape {tuple(i0.shape)} != ({out}, {n // 8})")
    return vq_gemv(xr.reshape(-1, n), i0, cb0, scale, rs=rs).reshape(*xr.shape[:-1], out)


def _ids32(ids):
    ids = ids.reshape(-1)
    if ids.dtype != torch.int32:
        ids = ids.to(torch.int32)
    return ids.contiguous()


def gemv_argmax(x, mat, cb0, cb1=None, rot=None, mode=None, rs=1.0, y=None, keys=False):
    """Greedy argmax over the rows of one VQ matrix, fused into its GEMV (vq2_gemv_argmax):
    returns int64 [M] row indices (ties to the smaller row); with ``y`` (a [M, out] tensor) the
    logits are written too; with ``keys`` the raw 64-bit (value, row) keys are returned instead
    (for a cross-rank maximum). M <= 64."""
    i0, i1, sc = mat
    _lib.require_cuda(x, i0, i1, sc, cb0, cb1)
    if mode is None:
        mode = _lib.VQ2_ACT_RHT if rot is not None else _lib.VQ2_ACT_ROTATED
    out, ng = i0.shape
    n = ng * 8
    xin = 2 * n if mode == _lib.VQ2_ACT_SWIGLU_RHT else n
    x2 = x.reshape(-1, xin).contiguous()
    M = x2.shape[0]
    _check_vals(cb0, cb1 if i1 is not None else None, sc)
    i0, i1, sc = _c(i0), _c(i1), _c(sc)   # held for the call: a temporary's memory could be reused
    best = torch.zeros(M, dtype=torch.int64, device=x.device)
    if y is not None and (y.shape[-1] != out or not y.is_contiguous()):
        raise ValueError("y must be contiguous [M, out]")
    _lib.call("vq2_gemv_argmax", _lib.ptr(x2), _lib.dtype_code(x2), int(mode), M, x2.stride(0),
              _lib.ptr(rot.perm) if rot is not None else None, _lib.ptr(rot.sign) if rot is not None else None,
              int(rot.hb) if rot is not None else 0, float(rot.scale) if rot is not None else 1.0,
              _lib.ptr(i0), _lib.ptr(i1) if i1 is not None else None, _lib.ptr(cb0),
              _lib.ptr(cb1) if i1 is not None else None, _lib.ptr(sc), _lib.dtype_code(cb0), out, n,
              float(rs), _lib.ptr(y) if y is not None else None, _lib.dtype_code(y) if y is not None else 0, out,
              _lib.ptr(best), _lib.stream_ptr(x.device))
    return best if keys else 0xFFFFFFFF - (best & 0xFFFFFFFF)


def gemv_multi(x, mats, cb0, cb1=None, rot=None, mode=None, rs=1.0, out_dtype=None, ys=None, y_row_stride=None):
    """P <= 8 VQ matrices sharing one activation in ONE launch.

    x: [..., n] (mode SWIGLU_RHT: fp32 [..., 2n]); mats: list of (idx0 int16 [out_p, n/8],
    idx1 uint8 or None, scale [out_p]); rot: a vq.Rot applied in-kernel when mode is RHT or
    SWIGLU_RHT (default: RHT when rot is given). Returns the list of outputs [..., out_p]
    (or writes the given ``ys``)."""
    if not 1 <= len(mats) <= 8:
        raise ValueError("gemv_multi takes 1..8 matrices")
    _lib.require_cuda(x, cb0, cb1)
    if mode is None:
        mode = _lib.VQ2_ACT_RHT if rot is not None else _lib.VQ2_ACT_ROTATED
    ng = mats[0][0].shape[1]
    n = ng * 8
    xin = 2 * n if mode == _lib.VQ2_ACT_SWIGLU_RHT else n
    if x.shape[-1] != xin:
        raise ValueError(f"activation last dim {x.shape[-1]} != {xin}")
    if mode != _lib.VQ2_ACT_ROTATED and (rot is None or rot.n != n):
        raise ValueError("a rotation of size n is required for modes RHT / SWIGLU_RHT")
    x2 = x.reshape(-1, xin)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    res = mats[0][1] is not None
    _check_vals(cb0, cb1 if res else None, *[m[2] for m in mats])
    i0s, i1s, scs, outs = [], [], [], []
    for i0, i1, sc in mats:
        _lib.require_cuda(i0, i1, sc)
        if i0.dtype != torch.int16 or i0.shape[1] != ng or (i1 is not None) != res:
            raise ValueError("matrices must share n and bpw; stage-1 indices are int16")
        if i1 is not None and (i1.dtype != torch.uint8 or i1.shape != i0.shape):
            raise ValueError("residual indices must be uint8 [out, n/8]")
        i0s.append(_c(i0)); i1s.append(_c(i1)); scs.append(_c(sc)); outs.append(i0.shape[0])
    out_dtype = out_dtype or cb0.dtype
    lead = x.shape[:-1]
    shaped = ys is None
    if ys is None:
        ys = [torch.empty(M, o, dtype=out_dtype, device=x.device) for o in outs]
        y_row_stride = None
    if y_row_stride is None:
        if M > 1 and len(set(outs)) > 1:
            raise ValueError("matrices of different heights need an explicit y_row_stride for M > 1")
        y_row_stride = outs[0]
    for y, o in zip(ys, outs):
        if y.dtype != out_dtype or y.stride(-1) != 1:
            raise ValueError("outputs must have dtype out_dtype and unit inner stride")
        if y.numel() < o or (M > 1 and (y.dim() < 2 or y.shape[-2] < M)):
            raise ValueError("output too small")
    P = len(mats)
    ws = _workspace(M, n, x.device)   # batched (tensor-core) path: the transformed, split operand
    _lib.call("vq2_gemv_multi", _lib.ptr(x2), _lib.dtype_code(x2), int(mode), M, x2.stride(0),
              _lib.ptr(rot.perm) if rot is not None else None, _lib.ptr(rot.sign) if rot is not None else None,
              int(rot.hb) if rot is not None else 0, float(rot.scale) if rot is not None else 1.0, P,
              _lib.ptr_array(ctypes.c_void_p, [i.data_ptr() for i in i0s]),
              _lib.ptr_array(ctypes.c_void_p, [i.data_ptr() for i in i1s]) if res else None,
              _lib.ptr_array(ctypes.c_int64, outs),
              _lib.ptr_array(ctypes.c_void_p, [t.data_ptr() for t in scs]),
              _lib.ptr(cb0), _lib.ptr(cb1) if res else None, _lib.dtype_code(cb0),
              _lib.ptr_array(ctypes.c_void_p, [y.data_ptr() for y in ys]), _lib.dtype_code(ys[0]),
              int(y_row_stride), n, float(rs), _lib.ptr(ws), ws.numel() if ws is not None else 0,
              _lib.stream_ptr(x.device))
    if shaped:
        ys = [y.reshape(*lead, y.shape[-1]) for y in ys]
    return ys


def moe_gemv(x, ids, pool_idx, cb16, pool_scale, y, x_k_stride, x_k_div=1, rs=1.0, rot=None, mode=None):
    """Expert-indexed GEMV: y[k] = rs * scale[e_k] * sum cb16[idx[e_k]] . act(x[k // x_k_div]).

    ``act`` is the identity (mode ROTATED), the forward RHT ``rot`` (mode RHT) or SwiGLU then
    ``rot`` (mode SWIGLU_RHT, x rows fp32 [gate | up]). ``pool_idx`` [E, OUT, NG] and
    ``pool_scale`` [E, OUT] may be strided views (e.g. into a pool of whole expert records)
    as long as each expert's block is contiguous."""
    _lib.require_cuda(x, ids, pool_idx, cb16, pool_scale, y)
    if pool_idx.dtype != torch.int16 or pool_idx.dim() != 3:
        raise ValueError("pool_idx must be int16 [E, OUT, NG]")
    _check_vals(cb16, pool_scale)
    if mode is None:
        mode = _lib.VQ2_ACT_RHT if rot is not None else _lib.VQ2_ACT_ROTATED
    E, OUT, NG = pool_idx.shape
    if pool_idx.stride(2) != 1 or pool_idx.stride(1) != NG or pool_scale.stride(-1) != 1:
        raise ValueError("each expert's index block [OUT, NG] and scale vector must be contiguous")
    idx_es = pool_idx.stride(0)
    sc_es = pool_scale.stride(0) if pool_scale.dim() == 2 else OUT
    ids = _ids32(ids)
    K = ids.numel()
    if y.shape[0] < K or y.numel() < K * OUT or not y.is_contiguous():
        raise ValueError(f"y must be contiguous with at least [{K}, {OUT}] elements")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    if mode != _lib.VQ2_ACT_ROTATED and (rot is None or rot.n != NG * 8):
        raise ValueError("a rotation of size n is required for modes RHT / SWIGLU_RHT")
    if pool_scale.shape[0] != E or pool_scale.shape[-1] != OUT:
        raise ValueError("pool_scale must be [E, OUT]")
    _lib.call("vq2_moe_gemv", _lib.ptr(x), _lib.dtype_code(x), int(mode), int(x_k_stride), int(x_k_div),
              _lib.ptr(rot.perm) if rot is not None else None, _lib.ptr(rot.sign) if rot is not None else None,
              int(rot.hb) if rot is not None else 0, float(rot.scale) if rot is not None else 1.0,
              _lib.ptr(ids), K, E, _lib.ptr(pool_idx), idx_es, _lib.ptr(cb16), _lib.ptr(pool_scale), sc_es,
              _lib.dtype_code(cb16), _lib.ptr(y), _lib.dtype_code(y), OUT, NG, float(rs),
              _lib.stream_ptr(x.device))
    return y


def vq_moe_parallel_gate_up(xr, topk_ids, gate_up_idx, cb16, gate_up_scale, y_out, OUT=1024, NG=256, rs=1.0):
    """Gate+up projections of the K active experts on one shared activation -- vq2/kernels.py:246-254."""
    if gate_up_idx.shape[1:] != (OUT, NG):
        raise ValueError("gate_up_idx must be [E, OUT, NG]")
    moe_gemv(xr.reshape(-1), topk_ids, gate_up_idx, cb16, gate_up_scale, y_out, x_k_stride=0, rs=rs)


def vq_moe_parallel_down(act_r, topk_ids, down_idx, cb16, down_scale, y_out, OUT=2048, NG=64, rs=1.0):
    """Down projections, expert k on its own activation row act_r[k] -- vq2/kernels.py:256-264."""
    if down_idx.shape[1:] != (OUT, NG):
        raise ValueError("down_idx must be [E, OUT, NG]")
    moe_gemv(act_r.contiguous(), topk_ids, down_idx, cb16, down_scale, y_out, x_k_stride=NG * 8, rs=rs)


def swiglu_rht(gu, rot, out=None):
    """act = silu(gu[:, :I]) * gu[:, I:], then rot.fwd(act), all fp32. gu: fp32 [M, 2I]."""
    _lib.require_cuda(gu)
    if gu.dtype != torch.float32 or gu.dim() != 2 or gu.shape[1] != 2 * rot.n or gu.stride(1) != 1:
        raise ValueError("gu must be fp32 [M, 2n] with unit inner stride")
    M = gu.shape[0]
    if out is None:
        out = torch.empty(M, rot.n, dtype=torch.float32, device=gu.device)
    _lib.call("vq2_swiglu_rht", _lib.ptr(gu), gu.stride(0), M, rot.n, rot.hb, _lib.ptr(rot.perm),
              _lib.ptr(rot.sign), float(rot.scale), _lib.ptr(out), out.stride(0), _lib.stream_ptr(gu.device))
    return out


def moe_combine(y, w, top_k, add=None, out=None, out_dtype=torch.float16):
    """out[t] = sum_j w[t, j] * y[t*top_k + j] (+ add[t]); y fp32 [T*top_k, H], w fp32 [T, top_k]."""
    _lib.require_cuda(y, w, add)
    if y.dtype != torch.float32 or w.dtype != torch.float32 or (add is not None and add.dtype != torch.float32):
        raise ValueError("moe_combine takes fp32 y, w and add")
    T = w.shape[0]
    H = y.shape[-1]
    if y.numel() != T * top_k * H:
        raise ValueError("y must be [T*top_k, H]")
    if out is None:
        out = torch.empty(T, H, dtype=out_dtype, device=y.device)
    y, w, add = _c(y), _c(w), _c(add)   # keep references alive across the launch
    _lib.call("vq2_moe_combine", _lib.ptr(y), _lib.ptr(w), T, top_k, H, _lib.ptr(add), _lib.ptr(out),
              _lib.dtype_code(out), _lib.stream_ptr(y.device))
    return out


def gather_rate(cb, mode=0, rows=None, iters=256, blocks_per_sm=8, reps=5):
    """Measured random 16-byte codebook-row gathers per second on cb's device (diagnostic;
    mode 0 global memory, 1 shared memory, 2 cluster distributed shared memory; modes 3 / 4:
    bucketed GEMV entries per second -- codeword and fp32 / fp16 activation both from shared
    memory, one 1024-thread CTA per SM)."""
    _lib.require_cuda(cb)
    dev = cb.device
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * blocks_per_sm if mode == 0 else (sms // 8 * 8 if mode == 2 else sms)
    threads = 1024 if mode in (3, 4) else 256
    rows = rows or cb.shape[0]
    sink = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _lib.stream_ptr(dev)
    args = (_lib.ptr(cb), rows, mode, blocks, iters, _lib.ptr(sink), st)
    _lib.call("vq2_gather_probe", *args)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        _lib.call("vq2_gather_probe", *args)
    e1.record()
    e1.synchronize()
    return reps * blocks * threads * iters * 8 / (e0.elapsed_time(e1) / 1e3)
