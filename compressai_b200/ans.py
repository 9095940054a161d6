"""ANS-coded index streams: host encoder and GPU decoder of the "VQ2A" interleaved rANS format.

The reference entropy-codes a stage's indices with constriction on the host and decodes them
once at load time (vq2/export.py:26-36, vq2/runtime.py:155-182). Here the coding unit is a byte
stream (an int16 index tensor viewed as bytes: even positions are the low bytes, odd the high
bytes, one adaptive-free static model per parity), encoded on the host by the C-ABI encoder and
decoded on the GPU, so an ANS-coded expert is paged in compressed and expanded in HBM. The format
is stated in include/vq2_b200.h; decoded bytes equal the encoder's input bit for bit.
"""
import ctypes

import numpy as np
import torch

from . import _lib

SEG_ANS = 0
SEG_STORED = 1

ERRORS = {1: "bad magic", 2: "symbol/chunk count mismatch", 3: "invalid frequency table",
          4: "chunk offset out of range", 5: "word counts exceed the chunk", 6: "renormalisation words exhausted",
          7: "bad final state"}


class ANSDecodeError(ValueError):
    pass


def bound(n):
    """Upper bound on the encoded size of n bytes."""
    b = _lib.load().vq2_rans_bound(int(n))
    if b < 0:
        raise ValueError(f"cannot ANS-code {n} bytes")
    return int(b)


def encode(data):
    """Encode the bytes of ``data`` (numpy array or CPU tensor of any dtype, C order) into a
    VQ2A stream (np.uint8)."""
    if isinstance(data, torch.Tensor):
        data = data.detach().cpu().contiguous().numpy()
    sym = np.ascontiguousarray(data).reshape(-1).view(np.uint8)
    cap = bound(sym.size)
    out = np.empty(cap, dtype=np.uint8)
    got = ctypes.c_int64(0)
    _lib.check(_lib.load().vq2_rans_encode(sym.ctypes.data if sym.size else None, sym.size, out.ctypes.data, cap,
                                           ctypes.byref(got)), "vq2_rans_encode")
    return out[:got.value].copy()


def new_status(device):
    """A zeroed device status word for the decoders."""
    return torch.zeros(1, dtype=torch.int32, device=device)


def decode(stream, n, out=None, status=None):
    """Decode a VQ2A stream held in device memory (uint8 tensor) into ``n`` bytes on the current
    stream. Asynchronous: a malformed stream raises ``status`` (check_status reads it)."""
    if not stream.is_cuda or stream.dtype != torch.uint8 or not stream.is_contiguous():
        raise ValueError("decode: stream must be a contiguous uint8 CUDA tensor")
    if out is None:
        out = torch.empty(int(n), dtype=torch.uint8, device=stream.device)
    if status is None:
        status = new_status(stream.device)
    if not out.is_cuda or not out.is_contiguous():
        raise ValueError("decode: out must be a contiguous CUDA tensor")
    _lib.call("vq2_rans_decode", _lib.ptr(stream), stream.numel(), int(n), _lib.ptr(out), out.numel() * out.element_size(),
              _lib.ptr(status), _lib.stream_ptr(stream.device))
    return out, status


def decode_segments(src, segments, dst, status, stream=None):
    """One launch expanding ``segments`` [(src_off, src_bytes, dst_off, n, kind), ...] (at most
    32) of the device buffer ``src`` into the device buffer ``dst`` (kind SEG_ANS or SEG_STORED)."""
    nseg = len(segments)
    arr = [np.ascontiguousarray([s[i] for s in segments], dtype=np.int64) for i in range(4)]
    kind = np.ascontiguousarray([s[4] for s in segments], dtype=np.int32)
    st = stream.cuda_stream if stream is not None else _lib.stream_ptr(src.device)
    _lib.call("vq2_rans_decode_segments", _lib.ptr(src), src.numel() * src.element_size(), arr[0].ctypes.data,
              arr[1].ctypes.data, arr[2].ctypes.data, arr[3].ctypes.data, kind.ctypes.data, nseg, _lib.ptr(dst),
              dst.numel() * dst.element_size(), _lib.ptr(status), st)


def check_status(status):
    """Synchronize on ``status`` and raise ANSDecodeError if a decode flagged its stream."""
    code = int(status.item())
    if code:
        raise ANSDecodeError(f"malformed ANS stream: {ERRORS.get(code, 'unknown error')} (code {code})")
