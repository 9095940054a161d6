"""Rotation and codebook plumbing of the VQ2 format, mirroring reference ``vq2/vq.py``.

``Rot`` draws the same permutation and signs as the reference (``vq2/vq.py:47-57``: torch's CPU
generator seeded by ``tag_seed(tag)``, ``randperm`` then ``randint``), keeps them on the
device as int32/int8, and applies the transform with the CUDA kernel ``vq2_rht`` (fp32
arithmetic). Only CUDA tensors are accepted; there is no CPU path.
"""
import hashlib

import torch

from . import _lib

D = 8        # vector dimension (vq2/vq.py:15)
HB = 2048    # Hadamard block (vq2/vq.py:16)


def tag_seed(tag):
    """Per-tag rotation seed: int(md5(tag)[:8], 16) (vq2/vq.py:40-41)."""
    return int(hashlib.md5(tag.encode()).hexdigest()[:8], 16)


def cfg_key(cfg, i):
    """Codebook key of stage i, e.g. "16", "16_8" (vq2/vq.py:109-110)."""
    return "_".join(str(b) for b in cfg[: i + 1])


def cfg_bpw(cfg):
    return sum(cfg) / D


def hadamard_block(n):
    """Hadamard block size of a length-n rotation (rule of vq2/vq.py:48-49)."""
    m = min(HB, n)
    hb = m if (n % m == 0 and (m & (m - 1)) == 0) else HB
    if n % hb != 0:
        raise ValueError(f"n={n} is not a multiple of hb={hb}")
    return hb


def _rows(x, n):
    if x.shape[-1] != n:
        raise ValueError(f"last dim {x.shape[-1]} != rotation size {n}")
    x2 = x.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


class Rot:
    """x' = R^T x on the last dimension: permutation, random signs, blocked Sylvester
    Hadamard of order hb, times hb^-0.5 (vq2/vq.py:44-87). Orthogonal: inv(fwd(x)) == x."""

    def __init__(self, n, seed, device="cuda"):
        self.n = n
        self.hb = hadamard_block(n)
        self.nb = n // self.hb
        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(n, generator=g)
        sign = torch.randint(0, 2, (n,), generator=g) * 2 - 1
        self.perm_cpu = perm
        self.sign_cpu = sign.to(torch.int8)
        self.device = torch.device(device)
        self.perm = perm.to(device=self.device, dtype=torch.int32)
        self.sign = self.sign_cpu.to(self.device)
        self.scale = self.hb ** -0.5

    def _run(self, x, inverse, out_scale, out=None):
        _lib.require_cuda(x)
        x2 = _rows(x, self.n)
        M = x2.shape[0]
        if out is None:
            out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        o2 = out.view(-1, self.n)
        _lib.call("vq2_rht", _lib.ptr(x2), _lib.dtype_code(x2), x2.stride(0), M, self.n, self.hb,
                  _lib.ptr(self.perm), _lib.ptr(self.sign), out_scale, int(inverse), _lib.ptr(o2),
                  o2.stride(0), _lib.stream_ptr(x.device))
        return out

    def fwd_f32(self, x, out=None, unnormalised=False):
        """Forward rotation with an fp32 result (the decode path's working precision)."""
        return self._run(x, False, 1.0 if unnormalised else self.scale, out)

    def inv_f32(self, y, out=None):
        return self._run(y, True, self.scale, out)

    def fwd(self, x):
        """Rot.fwd (vq2/vq.py:78-82): result in x's dtype, computed in fp32."""
        y = self.fwd_f32(x)
        return y if x.dtype == torch.float32 else y.to(x.dtype)

    def inv(self, y):
        """Rot.inv (vq2/vq.py:84-87): result in y's dtype, computed in fp32."""
        x = self.inv_f32(y)
        return x if y.dtype == torch.float32 else x.to(y.dtype)


_ROTS = {}


def get_rot(tag, n, device="cuda"):
    """Cached Rot per (tag, n, device) (vq2/vq.py:96-103)."""
    k = (tag, n, str(torch.device(device)))
    if k not in _ROTS:
        _ROTS[k] = Rot(n, tag_seed(tag), device)
    return _ROTS[k]


class Codebooks:
    """Dictionary {key: tensor[K, 8]} of universal codebooks (vq2/vq.py:153-167)."""

    def __init__(self, d=None):
        self.cb = d or {}

    def get(self, cfg, i):
        return self.cb[cfg_key(cfg, i)]

    def to(self, dev, dtype=None):
        self.cb = {k: v.to(device=dev, dtype=dtype or v.dtype).contiguous() for k, v in self.cb.items()}
        return self

    def state(self):
        return {k: v.cpu() for k, v in self.cb.items()}
