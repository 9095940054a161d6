"""The reference's CPU decode path, restated for the timed CPU baseline -- TEST/BENCH
INFRASTRUCTURE ONLY (imported by ``bench.py``'s cpu_baseline leg and ``--impl reference``
arm, never by the product).

* ``vq_gemv_cpu_streaming``: gather the codebook rows of every index then contract with the
  grouped activation, in torch fp32 on the host cores -- the "streaming" CPU GEMV of reference
  scratch/test_cpu_vq_gemv.py:53-70, with the int16 -> uint16 mask of
  vq2/paged_runtime.py:25.
* ``rht_cpu``: Rot._orig_fwd (vq2/vq.py:66-76) in torch fp32.
* ``moe_gate_up_cpu`` / ``moe_down_cpu``: vq_moe_parallel_gate_up_cpu / _down_cpu
  (vq2/paged_runtime.py:19-41), fp32 outputs.
"""
import torch


def vq_gemv_cpu_streaming(xr, idx, cb, scale, rs=1.0):
    """y[out] = rs * scale * einsum('org,rg->o', cb[idx], xr.view(NG, 8))."""
    ng = idx.shape[1]
    xg = xr.reshape(ng, 8)
    rec = cb[(idx.to(torch.int32) & 0xFFFF).long()]
    acc = torch.einsum("org,rg->o", rec, xg)
    return acc * scale * rs


_H = {}


def _hadamard(hb):
    if hb not in _H:
        H = torch.ones(1, 1)
        while H.shape[0] < hb:
            H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
        _H[hb] = H
    return _H[hb]


def rht_cpu(x, perm, sign, hb):
    y = x[..., perm] * sign
    sh = y.shape
    y = y.reshape(*sh[:-1], sh[-1] // hb, hb) @ _hadamard(hb)
    return (y * hb ** -0.5).reshape(sh)


def moe_gate_up_cpu(xr, slots, pool_idx, cb16, pool_scale, rs=1.0):
    xg = xr.reshape(-1, 8)
    out = []
    for s in slots:
        idx = (pool_idx[s].to(torch.int32) & 0xFFFF).long()
        out.append(torch.einsum("org,rg->o", cb16[idx], xg) * pool_scale[s].float() * rs)
    return torch.stack(out)


def moe_down_cpu(act_r, slots, pool_idx, cb16, pool_scale, rs=1.0):
    out = []
    for k, s in enumerate(slots):
        idx = (pool_idx[s].to(torch.int32) & 0xFFFF).long()
        out.append(torch.einsum("org,rg->o", cb16[idx], act_r[k].reshape(-1, 8)) * pool_scale[s].float() * rs)
    return torch.stack(out)
