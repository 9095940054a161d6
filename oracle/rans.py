"""TEST INFRASTRUCTURE ONLY: ctypes wrapper and build recipe for oracle/rans_oracle.c, the plain-C
restatement of the "VQ2A" interleaved rANS format used for ANS-coded expert indices.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use it, as the checker. The C file is
compiled with gcc into oracle/_build/librans_oracle.so (git-ignored, travels with the working
tree); `build()` is called by __graft_entry__.build() and lazily on first use.

The reference entropy-codes indices with the third-party `constriction` package
(vq2/export.py:26-36: a Categorical model over one stage's indices, AnsCoder.encode_reverse /
decode). constriction is not installed here and no reference test pins its stream bytes, so the
stream format is this repository's own and only the decoded indices are compared with the
reference (they must equal the encoder's input bit for bit).
"""
import ctypes
import os
import shutil
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "rans_oracle.c")
OUTDIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUTDIR, "librans_oracle.so")

_lib = None


def build(force=False):
    """Compile rans_oracle.c with gcc (when the .so is missing or older than the source)."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc is required to build the rANS oracle")
    os.makedirs(OUTDIR, exist_ok=True)
    tmp = LIB + ".tmp"
    subprocess.run([cc, "-O2", "-std=c99", "-shared", "-fPIC", "-Wall", "-o", tmp, SRC], check=True)
    os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build())
        lib.oracle_bound.argtypes = [ctypes.c_int64]
        lib.oracle_bound.restype = ctypes.c_int64
        lib.oracle_encode.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64]
        lib.oracle_encode.restype = ctypes.c_int64
        lib.oracle_decode.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64]
        lib.oracle_decode.restype = ctypes.c_int
        lib.oracle_quantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.oracle_quantize.restype = None
        _lib = lib
    return _lib


def bound(n):
    return int(_load().oracle_bound(int(n)))


def encode(sym):
    """uint8 symbols -> encoded stream (np.uint8)."""
    sym = np.ascontiguousarray(sym, dtype=np.uint8).reshape(-1)
    cap = bound(sym.size)
    out = np.zeros(cap, dtype=np.uint8)
    n = _load().oracle_encode(sym.ctypes.data, sym.size, out.ctypes.data, cap)
    if n < 0:
        raise ValueError("oracle_encode failed")
    return out[:n].copy()


def decode(stream, n):
    """Encoded stream -> (status, symbols); status 0 = well-formed, else the error code."""
    stream = np.ascontiguousarray(stream, dtype=np.uint8).reshape(-1)
    out = np.zeros(max(int(n), 1), dtype=np.uint8)
    st = _load().oracle_decode(stream.ctypes.data, stream.size, out.ctypes.data, int(n))
    return int(st), out[:n]


def quantize(counts):
    """256 symbol counts -> the 256 quantized frequencies (sum 4096) the format stores."""
    c = np.ascontiguousarray(counts, dtype=np.uint64)
    f = np.zeros(256, dtype=np.uint16)
    _load().oracle_quantize(c.ctypes.data, f.ctypes.data)
    return f
