"""C-ABI library: loads without a GPU, exports every symbol the header declares, validates
arguments before touching the device."""
import ctypes
import re

import pytest

from compressai_b200 import _lib


def _declared():
    txt = open(_lib.HEADER_PATH).read()
    return sorted(set(re.findall(r"VQ2_API\s+(?:const\s+)?\w+\*?\s+(vq2_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    names = _declared()
    assert "vq2_gemv" in names and "vq2_rht" in names and "vq2_moe_gemv" in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/vq2_b200.h"


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for nm in _declared():
        assert hasattr(lib, nm), nm
    assert lib.vq2_abi_version() == _lib.ABI_VERSION


def test_status_strings():
    lib = _lib.load()
    assert lib.vq2_status_string(0) == b"ok"
    assert b"shape" in lib.vq2_status_string(1)
    assert lib.vq2_status_string(99) == b"unknown status"


def test_argument_validation_without_device():
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # null activation
    assert lib.vq2_gemv(None, 2, 1, 2048, p, None, p, None, p, 0, p, 0, 2048, 2048, 2048, 1.0, None, 0, None) == _lib.VQ2_ERR_ARG
    # n not a multiple of 64
    assert lib.vq2_gemv(p, 2, 1, 2040, p, None, p, None, p, 0, p, 0, 2048, 2048, 2040, 1.0, None, 0, None) == _lib.VQ2_ERR_SHAPE
    # bad dtype code
    assert lib.vq2_gemv(p, 7, 1, 2048, p, None, p, None, p, 0, p, 0, 2048, 2048, 2048, 1.0, None, 0, None) == _lib.VQ2_ERR_DTYPE
    # misaligned index pointer
    q = ctypes.c_void_p(18)
    assert lib.vq2_gemv(p, 2, 1, 2048, q, None, p, None, p, 0, p, 0, 2048, 2048, 2048, 1.0, None, 0, None) == _lib.VQ2_ERR_ALIGN
    # residual index without residual codebook
    assert lib.vq2_gemv(p, 2, 1, 2048, p, p, p, None, p, 0, p, 0, 2048, 2048, 2048, 1.0, None, 0, None) == _lib.VQ2_ERR_ARG
    # RHT block size not a power of two
    assert lib.vq2_rht(p, 2, 2048, 1, 2048, 1000, p, p, 1.0, 0, p, 2048, None) == _lib.VQ2_ERR_SHAPE
    # moe: zero experts
    assert lib.vq2_moe_gemv(p, 2, 0, 0, 1, None, None, 0, 1.0, p, 8, 0, p, 262144, p, p, 1024, 0, p, 2, 1024,
                            256, 1.0, None) == _lib.VQ2_ERR_SHAPE
    # fused RHT mode without a rotation
    assert lib.vq2_moe_gemv(p, 2, 1, 0, 1, None, None, 2048, 1.0, p, 8, 16, p, 262144, p, p, 1024, 0, p, 2, 1024,
                            256, 1.0, None) == _lib.VQ2_ERR_ARG
    # expert stride smaller than one expert
    assert lib.vq2_moe_gemv(p, 2, 0, 0, 1, None, None, 0, 1.0, p, 8, 16, p, 1000, p, p, 1024, 0, p, 2, 1024,
                            256, 1.0, None) == _lib.VQ2_ERR_SHAPE
    # multi-matrix: too many matrices
    arr = (ctypes.c_void_p * 9)(*([16] * 9))
    outs = (ctypes.c_int64 * 9)(*([64] * 9))
    assert lib.vq2_gemv_multi(p, 2, 0, 1, 2048, None, None, 0, 1.0, 9, arr, None, outs, arr, p, None, 0, arr, 0,
                              64, 2048, 1.0, None, 0, None) == _lib.VQ2_ERR_SHAPE
    assert lib.vq2_gemv_workspace(1, 2048) == 0 and lib.vq2_gemv_workspace(4, 2048) == 2 * 4 * 2048 * 2 and lib.vq2_gemv_workspace(16, 2048) == 2 * 16 * 2048 * 2
    assert lib.vq2_moe_combine(p, p, 1, 0, 2048, None, p, 0, None) == _lib.VQ2_ERR_SHAPE


def test_status_mapping_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.VQ2_ERR_SHAPE, "x")
    with pytest.raises(_lib.VQ2Error):
        _lib.check(_lib.VQ2_ERR_TIMEOUT, "x")


def test_cpu_tensors_are_rejected():
    import torch
    from compressai_b200 import kernels
    x = torch.zeros(2048)
    i0 = torch.zeros(2048, 256, dtype=torch.int16)
    cb = torch.zeros(65536, 8, dtype=torch.float16)
    sc = torch.zeros(2048, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        kernels.vq_gemv_16(x, i0, cb, sc, 2048, 2048)
