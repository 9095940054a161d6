"""Compressed-weight decode runtime, mirroring reference ``vq2/runtime.py``.

``PackedLinear`` is a drop-in ``nn.Linear`` whose weight stays VQ-compressed in HBM. Its
forward is ONE kernel launch: the fp32 input rotation runs in the GEMV kernel's prologue, then
the codebook-decode GEMV, for any number of rows M (the reference's fused path is batch-1 only,
vq2/runtime.py:92; larger M fall back to dequantize-then-matmul there, :105-110). Scales and
codebooks stay in their container dtype (fp16); the output takes the input's dtype.
``PackedLinearGroup`` runs modules that share an input (q/k/v, gate/up) as one launch.
"""
import os

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, kernels
from . import vq

RS = vq.HB ** -0.5   # the unnormalised-rotation scale folded into legacy GEMV calls (vq2/runtime.py:66)


def _as_index(a, bits):
    """Stored indices -> int32 codebook rows (vq2/runtime.py:32-35)."""
    a = a.to(torch.int32)
    return a & 0xFFFF if bits > 8 else a


class _RotCache:
    """Last (input tensor, version) -> fp32 rotation, shared by all modules with the same Rot."""

    def __init__(self):
        self.x = None
        self.ver = -1
        self.y = None


_CACHES = {}


def rotate_cached(rot, x, unnormalised=False):
    key = (id(rot), unnormalised)
    c = _CACHES.get(key)
    if c is None:
        c = _CACHES[key] = _RotCache()
    if c.x is x and c.ver == x._version:
        return c.y
    y = rot.fwd_f32(x, unnormalised=unnormalised)
    c.x, c.ver, c.y = x, x._version, y
    return y


class FastRot:
    """Decode rotation: permutation + signs + UNnormalised Hadamard; the hb^-0.5 goes into the
    GEMV's rs. The result is reused while the same tensor (identity and version) comes back
    (vq2/runtime.py:37-63). Returns fp32 (the reference returns bf16)."""
    _ALL = {}

    def __init__(self, rot, device):
        self.rot = rot
        self.perm = rot.perm
        self.sign = rot.sign
        self.nb = rot.nb

    @classmethod
    def get(cls, tag, n, device, rot):
        k = (tag, n, str(device))
        if k not in cls._ALL:
            cls._ALL[k] = cls(rot, device)
        return cls._ALL[k]

    def __call__(self, x):
        return rotate_cached(self.rot, x.reshape(-1), unnormalised=True)


class PackedLinear(nn.Module):
    """nn.Linear replacement over VQ indices (vq2/runtime.py:70-113).

    shape=(out, n); cfg=(16,) (2 bpw) or (16, 8) (3 bpw); idx: list of index tensors per stage
    ([out, n/8] int16, uint8); scale: [out]; cbs: dict {"16": [65536, 8], "16_8": [256, 8]}
    in fp16 (or bf16) on the device, shared between modules."""

    def __init__(self, shape, cfg, tag, idx, scale, cbs, device):
        super().__init__()
        self.out, self.n = shape
        self.cfg, self.tag = tuple(cfg), tag
        if self.cfg not in ((16,), (16, 8)):
            raise ValueError(f"unsupported cfg {cfg}: the decode kernels take (16,) or (16, 8)")
        self.keys = [vq.cfg_key(self.cfg, i) for i in range(len(self.cfg))]
        cb_dtype = cbs[self.keys[0]].dtype
        for i, a in enumerate(idx):
            a = torch.as_tensor(a)
            a = a.to(torch.int16) if i == 0 else a.to(torch.uint8)
            self.register_buffer(f"idx{i}", a.to(device).contiguous(), persistent=False)
        self.register_buffer("scale", torch.as_tensor(scale).to(device=device, dtype=cb_dtype).contiguous(),
                             persistent=False)
        self._cbs = [cbs]
        self.rot = vq.get_rot(tag, self.n, device)

    def weight_rows(self, r0, r1):
        """Rotated-space rows [r0, r1) in the codebook dtype, decoded on the GPU by the row-decode
        kernel (vq2_embed_rows without the inverse transform): scale[r] * (sum of the stages'
        codewords), the reference's dequantized rows (vq2/runtime.py:82-89)."""
        ids = torch.arange(r0, r1, dtype=torch.int64, device=self.idx0.device)
        cb0, cb1 = self.codebooks()
        return decode_rows(self, ids, cb0, cb1, inverse=False, out_dtype=cb0.dtype)

    def mat(self):
        return (self.idx0, getattr(self, "idx1", None), self.scale)

    def codebooks(self):
        cbs = self._cbs[0]
        return cbs[self.keys[0]], (cbs[self.keys[1]] if len(self.keys) > 1 else None)

    def forward(self, x):
        """y = x W^T: the input rotation runs in the GEMV kernel's prologue (fp32), one launch."""
        cb0, cb1 = self.codebooks()
        out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16, torch.float32) else torch.float16
        return kernels.gemv_multi(x, [self.mat()], cb0, cb1, rot=self.rot, out_dtype=out_dtype)[0]

    def greedy(self, x, logits=None):
        """argmax over this layer's outputs for each row of x, fused into the GEMV (no logits
        round trip unless ``logits`` [M, out] is given to be filled): int64 [M]."""
        cb0, cb1 = self.codebooks()
        return kernels.gemv_argmax(x, self.mat(), cb0, cb1, rot=self.rot, y=logits)

    def nbytes(self):
        return sum(b.numel() * b.element_size() for b in self.buffers())


class PackedLinearGroup:
    """Several PackedLinear modules that read the same input (q/k/v, gate/up) run as ONE
    multi-matrix launch: one input rotation per CTA, one launch instead of one per matrix.
    The modules must share n, cfg, rotation tag and codebooks."""

    def __init__(self, mods):
        if not 1 <= len(mods) <= 8:
            raise ValueError("a group holds 1..8 modules")
        m0 = mods[0]
        for m in mods[1:]:
            if (m.n, m.cfg, m.rot) != (m0.n, m0.cfg, m0.rot) or m._cbs[0] is not m0._cbs[0]:
                raise ValueError("grouped modules must share n, cfg, rotation and codebooks")
        self.mods = list(mods)

    def __call__(self, x, out_dtype=None):
        m0 = self.mods[0]
        cb0, cb1 = m0.codebooks()
        out_dtype = out_dtype or (x.dtype if x.dtype in (torch.float16, torch.bfloat16, torch.float32)
                                  else torch.float16)
        return kernels.gemv_multi(x, [m.mat() for m in self.mods], cb0, cb1, rot=m0.rot, out_dtype=out_dtype)


class PackedSwiGLUMLP(nn.Module):
    """down(silu(gate(x)) * up(x)) over PackedLinear weights in TWO launches: gate and up as
    one multi-matrix GEMV (input RHT in its prologue, fp32 [M, 2I] output), then down with the
    SwiGLU and its input RHT in the prologue. Same math as the Qwen MLP block the reference
    wraps (transformers Qwen3_5MoeMLP; vq2/paged_runtime.py:501-504 for the expert form)."""

    def __init__(self, gate, up, down):
        super().__init__()
        if gate.out != up.out or down.n != gate.out:
            raise ValueError("gate/up rows must equal down's input size")
        self.gate, self.up, self.down = gate, up, down
        self._gu = PackedLinearGroup([gate, up])

    def forward(self, x):
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        M, inter = x2.shape[0], self.gate.out
        gu = torch.empty(M, 2 * inter, dtype=torch.float32, device=x.device)
        m0 = self.gate
        cb0, cb1 = m0.codebooks()
        kernels.gemv_multi(x2, [self.gate.mat(), self.up.mat()], cb0, cb1, rot=m0.rot, out_dtype=torch.float32,
                           ys=[gu, gu[:, inter:]], y_row_stride=2 * inter)
        d = self.down
        cbd0, cbd1 = d.codebooks()
        out_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16, torch.float32) else torch.float16
        y = kernels.gemv_multi(gu, [d.mat()], cbd0, cbd1, rot=d.rot, mode=kernels._lib.VQ2_ACT_SWIGLU_RHT,
                               out_dtype=out_dtype)[0]
        return y.reshape(*lead, d.out)


def decode_rows(lin, ids, cb0, cb1, inverse, out_dtype):
    """Rows `ids` of PackedLinear `lin`, dequantized on the GPU (vq2_embed_rows): rotated-space
    rows, or with ``inverse`` the original-space rows Rot.inv(q) (the embedding lookup)."""
    _lib.require_cuda(ids, cb0, cb1)
    flat = ids.reshape(-1).to(torch.int64).contiguous()
    out = torch.empty(flat.numel(), lin.n, dtype=out_dtype, device=flat.device)
    if flat.numel() == 0:
        return out.reshape(*ids.shape, lin.n)
    bad = torch.zeros(1, dtype=torch.int32, device=flat.device)
    i1 = getattr(lin, "idx1", None)
    rot = lin.rot if inverse else None
    _lib.call("vq2_embed_rows", _lib.ptr(flat), flat.numel(), lin.out, _lib.ptr(lin.idx0), _lib.ptr(i1),
              _lib.ptr(cb0), _lib.ptr(cb1 if i1 is not None else None), _lib.ptr(lin.scale), _lib.dtype_code(cb0),
              lin.n, _lib.ptr(rot.perm) if rot else None, _lib.ptr(rot.sign) if rot else None,
              rot.hb if rot else 0, float(rot.scale) if rot else 1.0, _lib.ptr(out), _lib.dtype_code(out),
              _lib.ptr(bad), _lib.stream_ptr(flat.device))
    return out.reshape(*ids.shape, lin.n)


class PackedEmbedding(nn.Module):
    """Embedding lookup over a VQ-compressed (tied) embedding matrix: each token's row is decoded
    on the GPU in fp32 -- codewords, row scale, inverse rotation -- in one kernel launch
    (vq2_embed_rows), returned in bf16 as the reference does (vq2/runtime.py:116-133). ``cbs32``:
    the embedding codebooks (the reference passes fp32 copies; the values are those of the
    stored fp16/bf16 codebooks, which the kernel reads directly)."""

    def __init__(self, lin, cbs32=None, out_dtype=torch.bfloat16):
        super().__init__()
        self.lin = lin
        self.out_dtype = out_dtype

    def forward(self, ids):
        cb0, cb1 = self.lin.codebooks()
        return decode_rows(self.lin, ids, cb0, cb1, inverse=True, out_dtype=self.out_dtype)


class PackedLMHead(nn.Module):
    """lm_head tied to the embedding: shares its compressed indices (vq2/runtime.py:136-144)."""

    def __init__(self, lin):
        super().__init__()
        self.lin = lin

    def forward(self, x):
        return self.lin(x)

    def greedy(self, x, logits=None):
        """Next-token ids (greedy) from hidden states x [M, H]: the VQ GEMV with the argmax in
        its epilogue (vq2_gemv_argmax)."""
        return self.lin.greedy(x, logits)


# --------------------------------------------------------------------------------------------
# containers
# --------------------------------------------------------------------------------------------
def unpack_fixed(buf, bits, n):
    """Fixed-width index unpacking, 16/8/4/12 bits (vq2/export.py:56-70)."""
    buf = np.asarray(buf)
    if bits == 16:
        return buf.view(np.uint16)[:n].astype(np.int64)
    if bits == 8:
        return buf[:n].astype(np.int64)
    if bits == 4:
        b = buf.astype(np.uint32)
        out = np.empty(len(b) * 2, dtype=np.int64)
        out[0::2] = b & 15
        out[1::2] = b >> 4
        return out[:n]
    if bits == 12:
        b = buf.reshape(-1, 3).astype(np.uint32)
        w = b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)
        out = np.empty(len(w) * 2, dtype=np.int64)
        out[0::2] = w & 4095
        out[1::2] = w >> 12
        return out[:n]
    raise ValueError(bits)


def unpack_fixed_gpu(buf, bits, n, device="cuda"):
    """unpack_fixed on the GPU (vq2_unpack_fixed): a fixed-width stream (host or device uint8) ->
    a device tensor of n symbols, int16 holding uint16 bits for 12/16-bit streams, uint8 else."""
    src = torch.as_tensor(buf).reshape(-1).to(device=device, dtype=torch.uint8).contiguous()
    dt = torch.int16 if bits > 8 else torch.uint8
    out = torch.empty(n, dtype=dt, device=device)
    if n:
        _lib.call("vq2_unpack_fixed", _lib.ptr(src), src.numel(), bits, n, _lib.ptr(out), out.element_size(),
                  _lib.stream_ptr(torch.device(device)))
    return out


def decode_indices(C, device=None):
    """Container dict -> {name: [index tensor per stage]} (vq2/runtime.py:155-182). Fixed-width
    streams are unpacked on the GPU when ``device`` is a CUDA device (vq2_unpack_fixed; the
    tensors stay there), else on the host; ANS streams (coded with the third-party
    `constriction` package) cannot be decoded without it and raise."""
    idx = {nm: [None] * len(C["meta"][nm]["cfg"]) for nm in C["names"]}
    gpu = device is not None and torch.device(device).type == "cuda"
    for key, e in C["streams"].items():
        bits = e["bits"]
        n = int(sum(e["sizes"]))
        if e["mode"] == "ans":
            raise NotImplementedError("ANS-coded .vq2 streams need `constriction`, which is not installed; "
                                      "convert to .vq2r (raw indices) first")
        fx = e["fixed"].numpy() if isinstance(e["fixed"], torch.Tensor) else e["fixed"]
        if gpu:
            t_all = unpack_fixed_gpu(fx, bits, n, device)
        else:
            sym = unpack_fixed(fx, bits, n)
            arr = sym.astype(np.uint8) if bits <= 8 else sym.astype(np.uint16).view(np.int16)
            t_all = torch.from_numpy(np.ascontiguousarray(arr))
        owners = [nm for nm in C["names"]
                  if key in [vq.cfg_key(C["meta"][nm]["cfg"], i) for i in range(len(C["meta"][nm]["cfg"]))]]
        off = 0
        for nm, sz in zip(owners, e["sizes"]):
            cfg_ = C["meta"][nm]["cfg"]
            i = [vq.cfg_key(cfg_, j) for j in range(len(cfg_))].index(key)
            idx[nm][i] = t_all[off:off + sz].view(C["meta"][nm]["shape"][0], -1).clone()
            off += sz
    return idx


def read_container(path, device=None):
    """Read a .vq2 (fixed-width streams) or .vq2r (raw indices) dict (vq2/runtime.py:185-193);
    with a CUDA ``device`` the fixed-width streams are unpacked there."""
    C = torch.load(path, weights_only=False)
    if C.get("format") == "vq2r":
        return C
    idx = decode_indices(C, device)
    scales = {nm: (s if isinstance(s, torch.Tensor) else torch.from_numpy(s)) for nm, s in C["scales"].items()}
    return dict(format="vq2r", names=C["names"], meta=C["meta"], idx=idx, scales=scales,
                codebooks=C["codebooks"], codebooks_embed=C.get("codebooks_embed", C["codebooks"]),
                dense=C.get("dense", {}))


def convert_to_runtime(src, dst):
    """Decode once and save raw indices (vq2/runtime.py:196-200)."""
    torch.save(read_container(src), dst)
    return os.path.getsize(dst)


def build_packed_linears(C, device, cb_dtype=torch.float16):
    """{name: PackedLinear} for every quantized matrix of a container dict (the module
    construction loop of vq2/runtime.py:231-241, without the HF model around it)."""
    cbs = {k: v.to(device=device, dtype=cb_dtype).contiguous() for k, v in C["codebooks"].items()}
    mods = {}
    for nm in C["names"]:
        m = C["meta"][nm]
        mods[nm] = PackedLinear(m["shape"], m["cfg"], m["tag"], C["idx"][nm], C["scales"][nm], cbs, device)
    return mods


def _set_module(model, name, new):
    parent = model
    parts = name.split(".")
    for p in parts[:-1]:
        parent = getattr(parent, p)
    setattr(parent, parts[-1], new)


@torch.no_grad()
def load_packed(path, device="cuda", config=None, cb_dtype=torch.float16):
    """Load a .vq2/.vq2r container into a transformers causal LM whose quantized linears stay
    compressed on the GPU (vq2/runtime.py:214-246): every name in the container becomes a
    PackedLinear (an ``embed_tokens`` name a PackedEmbedding, and a tied lm_head a
    PackedLMHead over the same indices), the ``dense`` tensors are copied in, and the model moves
    to ``device``. The reference reads the HF config from its model directory; here ``config``
    is a transformers config, a directory holding one, or None for $VQ2_MODEL_DIR."""
    from transformers import AutoConfig, AutoModelForCausalLM
    if config is None:
        config = os.environ.get("VQ2_MODEL_DIR")
        if config is None:
            raise ValueError("load_packed needs the model's config (argument or VQ2_MODEL_DIR)")
    if isinstance(config, (str, os.PathLike)):
        config = AutoConfig.from_pretrained(str(config), trust_remote_code=True)
    C = read_container(path, device)
    try:
        from transformers.initialization import no_init_weights
    except ImportError:  # older transformers
        from transformers.modeling_utils import no_init_weights
    with no_init_weights():
        model = AutoModelForCausalLM.from_config(config, dtype=torch.bfloat16).eval()
    for p in model.parameters():
        p.requires_grad_(False)
    params = dict(model.named_parameters())
    for n, v in C.get("dense", {}).items():
        params[n].data.copy_(v)
    cbs = {k: v.to(device=device, dtype=cb_dtype).contiguous() for k, v in C["codebooks"].items()}
    cbs_emb = {k: v.to(device=device, dtype=cb_dtype).contiguous()
               for k, v in C.get("codebooks_embed", C["codebooks"]).items()}
    emb = None
    for nm in C["names"]:
        m = C["meta"][nm]
        is_emb = nm.endswith("embed_tokens")
        pl = PackedLinear(m["shape"], m["cfg"], m["tag"], C["idx"][nm], C["scales"][nm], cbs_emb if is_emb else cbs,
                          device)
        C["idx"][nm] = None
        if is_emb:
            emb = pl
            _set_module(model, nm, PackedEmbedding(pl))
        else:
            _set_module(model, nm, pl)
    if emb is not None and getattr(config.get_text_config(), "tie_word_embeddings", True):
        model.lm_head = PackedLMHead(emb)
    return model.to(device)


def packed_bytes(model):
    """Bytes of the compressed weights (PackedLinear buffers) held by ``model``."""
    return sum(m.nbytes() for m in model.modules() if isinstance(m, PackedLinear))


def report_memory(model, tag=""):
    """Print allocated / peak device memory and the packed weight bytes (vq2/runtime.py:258-263)."""
    if not torch.cuda.is_available():
        return
    torch.cuda.synchronize()
    print(f"[mem{tag}] allocated {torch.cuda.memory_allocated() / 2**20:.0f} MiB | peak "
          f"{torch.cuda.max_memory_allocated() / 2**20:.0f} MiB | packed weights {packed_bytes(model) / 2**20:.0f} MiB")
