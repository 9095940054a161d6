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


def test_paged_layer_struct_matches_header():
    """The ctypes mirror of vq2_paged_layer declares the header's fields in order with the
    natural C layout (pointers and int64 at 8-byte boundaries)."""
    txt = open(_lib.HEADER_PATH).read()
    body = txt[txt.index("typedef struct vq2_paged_layer {"):txt.index("} vq2_paged_layer;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S).split("{", 1)[1]
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if decl:
            names += [n.strip().lstrip("*") for n in re.sub(r"^(const\s+)?\w+\*?\s+", "", decl).split(",")]
    assert names == [f for f, _ in _lib.PagedLayer._fields_]
    # sizes and offsets as the C compiler lays the struct out
    import os
    import shutil
    import subprocess
    import tempfile
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    d = tempfile.mkdtemp()
    src = os.path.join(d, "layout.c")
    with open(src, "w") as f:
        f.write("#include <stdio.h>\n#include <stddef.h>\n#include \"vq2_b200.h\"\nint main(void){"
                f"printf(\"%zu\", sizeof(vq2_paged_layer));"
                + "".join(f"printf(\" %zu\", offsetof(vq2_paged_layer, {n}));" for n in names) + "return 0;}")
    exe = os.path.join(d, "layout")
    subprocess.run([cc, "-I", os.path.dirname(_lib.HEADER_PATH), src, "-o", exe], check=True)
    got = [int(v) for v in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert got[0] == ctypes.sizeof(_lib.PagedLayer)
    assert got[1:] == [getattr(_lib.PagedLayer, n).offset for n in names]


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


def test_paged_step_validation_without_device():
    lib = _lib.load()
    slots = (ctypes.c_int32 * 8)()
    layer = _lib.PagedLayer()  # null pool, events, ...
    assert lib.vq2_paged_moe_step(None, None, 0, 1, 8, slots, None, 0, None, None, None, None, None, 0, None, 0,
                                  None) == _lib.VQ2_ERR_ARG
    assert lib.vq2_paged_moe_step(ctypes.byref(layer), None, 0, 1, 8, slots, None, 0, None, None, None, None, None,
                                  0, None, 0, None) == _lib.VQ2_ERR_ARG
    p = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    layer = _lib.PagedLayer(pool=256, capacity=4, gu_rows=1024, gu_cols=256, dn_rows=2048, dn_cols=64, ids_host=256,
                            ids_dev=256, ids_cap=8, copy_stream=256, copy_done=256, compute_done=256, ids_done=256)
    big = lib.vq2_moe_expert_ffn_workspace(2, 8, 1024, 2048)
    # more problems than the id buffers hold
    assert lib.vq2_paged_moe_step(ctypes.byref(layer), p, 0, 2, 8, slots, p, 0, None, None, None, None, p, big, p, 0,
                                  None) == _lib.VQ2_ERR_SHAPE
    # a miss aimed outside the pool, and one of the wrong size
    src = (ctypes.c_void_p * 1)(256)
    ws = lib.vq2_moe_expert_ffn_workspace(1, 8, 1024, 2048)
    for slot, nb in ((4, 792576), (0, 1000)):
        bad_slot = (ctypes.c_int32 * 1)(slot)
        nbytes = (ctypes.c_int64 * 1)(nb)
        assert lib.vq2_paged_moe_step(ctypes.byref(layer), p, 0, 1, 8, slots, p, 1, src, nbytes, bad_slot, None, p,
                                      ws, p, 0, None) == _lib.VQ2_ERR_SHAPE
    # coded records without a staging buffer
    layer.index_coding = 1
    assert lib.vq2_paged_moe_step(ctypes.byref(layer), p, 0, 1, 8, slots, p, 0, None, None, None, None, p, ws, p, 0,
                                  None) == _lib.VQ2_ERR_ARG


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
