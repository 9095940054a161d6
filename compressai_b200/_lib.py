"""ctypes binding of the C-ABI library ``lib/libvq2_b200.so`` (declared in include/vq2_b200.h).

The library is loaded on first use. There is no fallback: if it is missing or fails to load,
every compute entry point raises. Status codes from the C-ABI are mapped to Python
exceptions: shape/dtype/alignment/argument errors -> ValueError, launch/timeout -> RuntimeError.
"""
import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("VQ2_B200_LIB", os.path.join(_HERE, "lib", "libvq2_b200.so"))
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "vq2_b200.h")

VQ2_OK, VQ2_ERR_SHAPE, VQ2_ERR_DTYPE, VQ2_ERR_ALIGN, VQ2_ERR_LAUNCH, VQ2_ERR_TIMEOUT, VQ2_ERR_ARG = range(7)
VQ2_F16, VQ2_BF16, VQ2_F32 = 0, 1, 2
VQ2_ACT_ROTATED, VQ2_ACT_RHT, VQ2_ACT_SWIGLU_RHT = 0, 1, 2

_DTYPE_CODE = {torch.float16: VQ2_F16, torch.bfloat16: VQ2_BF16, torch.float32: VQ2_F32}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> argtypes (restype is int unless stated); must match include/vq2_b200.h
SIGNATURES = {
    "vq2_abi_version": [],
    "vq2_status_string": [_i32],
    "vq2_last_cuda_error": [],
    "vq2_rht": [_p, _i32, _i64, _i64, _i64, _i64, _p, _p, _f32, _i32, _p, _i64, _p],
    "vq2_swiglu_rht": [_p, _i64, _i64, _i64, _i64, _p, _p, _f32, _p, _i64, _p],
    "vq2_gemv_multi": [_p, _i32, _i32, _i64, _i64, _p, _p, _i64, _f32, _i64, _p, _p, _p, _p, _p, _p, _i32, _p,
                       _i32, _i64, _i64, _f32, _p, _i64, _p],
    "vq2_gemv_workspace": [_i64, _i64],
    "vq2_tc_status": [_i32],
    "vq2_router_logits": [_p, _i32, _i64, _p, _i32, _i64, _i64, _p, _p],
    "vq2_peer_exchange_buffer_bytes": [_i64, _i64],
    "vq2_peer_exchange": [_p, _i64, _i32, _i64, _p, _i32, _i32, _i64, _p, _p, _i64, _p, _p],
    "vq2_fixed_stream_bytes": [_i32, _i64],
    "vq2_unpack_fixed": [_p, _i64, _i32, _i64, _p, _i32, _p],
    "vq2_embed_rows": [_p, _i64, _i64, _p, _p, _p, _p, _p, _i32, _i64, _p, _p, _i64, _f32, _p, _i32, _p, _p],
    "vq2_gemv_argmax": [_p, _i32, _i32, _i64, _i64, _p, _p, _i64, _f32, _p, _p, _p, _p, _p, _i32, _i64, _i64, _f32, _p,
                        _i32, _i64, _p, _p],
    "vq2_gemv": [_p, _i32, _i64, _i64, _p, _p, _p, _p, _p, _i32, _p, _i32, _i64, _i64, _i64, _f32, _p, _i64, _p],
    "vq2_moe_gemv": [_p, _i32, _i32, _i64, _i64, _p, _p, _i64, _f32, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _i32,
                     _p, _i32, _i64, _i64, _f32, _p],
    "vq2_moe_combine": [_p, _p, _i64, _i64, _i64, _p, _p, _i32, _p],
    "vq2_gather_probe": [_p, _i64, _i32, _i64, _i64, _p, _p],
    "vq2_moe_route": [_p, _i64, _i64, _i64, _p, _p, _p, _i32, _p, _i64, _p, _p],
    "vq2_moe_expert_ffn": [_p, _i32, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i32, _p, _p, _i64,
                           _f32, _p, _p, _i64, _f32, _p, _i64, _p, _i32, _p],
    "vq2_moe_expert_ffn_workspace": [_i64, _i64, _i64, _i64],
    "vq2_moe_expert_ffn_noalloc": [_p, _i32, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i32, _p, _p,
                                   _i64, _f32, _p, _p, _i64, _f32, _p, _i32, _p],
    "vq2_paged_moe_t1_workspace": [_i64],
    "vq2_paged_moe_t1": [_p, _i32, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i32, _p, _p, _i64,
                         _f32, _p, _p, _i64, _f32, _p, _p, _i64, _p, _i64, _p, _i32, _p],
    "vq2_rans_bound": [_i64],
    "vq2_rans_encode": [_p, _i64, _p, _i64, _p],
    "vq2_rans_decode": [_p, _i64, _i64, _p, _i64, _p, _p],
    "vq2_rans_decode_segments": [_p, _i64, _p, _p, _p, _p, _p, _i64, _p, _i64, _p, _p],
    "vq2_moe_expert_ffn_res": [_p, _i32, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i32, _p, _p,
                               _i64, _f32, _p, _p, _i64, _f32, _p, _p, _i64, _p, _i32, _p],
    "vq2_moe_peer_buffer_bytes": [_i64, _i64, _i64],
    "vq2_moe_expert_ffn_ep": [_p, _i32, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i32, _p, _p, _i64,
                              _f32, _p, _p, _i64, _f32, _p, _i64, _p, _i32, _i32, _i64, _p, _p, _i64, _p, _i32, _p],
    "vq2_moe_layer_workspace": [_i64, _i64, _i32, _i64, _i64, _i64],
    "vq2_moe_layer": [_p, _i32, _i64, _p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _p, _i64, _i64, _i64, _i64, _i64,
                      _p, _i32, _p, _p, _i64, _f32, _p, _p, _i64, _f32, _p, _i64, _p, _i32, _p],
    "vq2_moe_layer_ep": [_p, _i32, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _i32,
                         _p, _p, _i64, _f32, _p, _p, _i64, _f32, _p, _i64, _p, _i32, _i32, _i64, _p, _p, _i64, _p, _i32,
                         _p],
    "vq2_lru_state_ints": [_i64, _i64],
    "vq2_lru_step": [_p, _p, _i64, _p, _p, _p],
    "vq2_fetch_records": [_p, _p, _i64, _p, _i64, _p, _i64, _i64, _p],
    "vq2_host_device_pointer": [_p, _p],
    "vq2_paged_moe_step": [_p, _p, _i32, _i64, _i64, _p, _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _i32, _p],
}


class PagedLayer(ctypes.Structure):
    """Mirror of ``vq2_paged_layer`` (include/vq2_b200.h), field for field."""
    _fields_ = [("pool", _p), ("capacity", _i64), ("gu_rows", _i64), ("gu_cols", _i64), ("dn_rows", _i64),
                ("dn_cols", _i64), ("cb0", _p), ("val_dtype", ctypes.c_int32), ("index_coding", ctypes.c_int32),
                ("perm_in", _p), ("sign_in", _p), ("hb_in", _i64), ("perm_mid", _p), ("sign_mid", _p),
                ("hb_mid", _i64), ("scale_in", _f32), ("scale_mid", _f32), ("stage", _p), ("stage_bytes", _i64),
                ("status", _p), ("stage_turn", _p), ("decode_stream", _p), ("stage_ready", _p), ("stage_free0", _p),
                ("stage_free1", _p), ("ids_host", _p), ("ids_dev", _p), ("ids_cap", _i64), ("copy_stream", _p),
                ("copy_done", _p), ("compute_done", _p), ("ids_done", _p)]
ABI_VERSION = 2

_lib = None
_lock = threading.Lock()


class VQ2Error(RuntimeError):
    pass


def load():
    """Load the library once (thread-safe) and bind every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise VQ2Error(f"compressai_b200 CUDA library not built: {LIB_PATH} is missing "
                           "(run `python -m compressai_b200.build`); there is no CPU fallback")
        lib = ctypes.CDLL(LIB_PATH)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = (ctypes.c_char_p if name == "vq2_status_string" else
                          ctypes.c_int64 if name.endswith(("_workspace", "_bound", "_ints", "_bytes")) else ctypes.c_int)
        if lib.vq2_abi_version() != ABI_VERSION:
            raise VQ2Error(f"ABI version mismatch: library {lib.vq2_abi_version()}, python {ABI_VERSION}")
        _lib = lib
    return _lib


def available():
    """True when the CUDA library exists and loads (the reference's HAVE_TRITON role)."""
    try:
        load()
        return True
    except (OSError, VQ2Error):
        return False


def check(status, what):
    if status == VQ2_OK:
        return
    lib = load()
    msg = f"{what}: {lib.vq2_status_string(status).decode()} (status {status})"
    if status in (VQ2_ERR_SHAPE, VQ2_ERR_DTYPE, VQ2_ERR_ALIGN, VQ2_ERR_ARG):
        raise ValueError(msg)
    if status == VQ2_ERR_LAUNCH:
        msg += f", cudaError {lib.vq2_last_cuda_error()}"
    raise VQ2Error(msg)


def call(name, *args):
    """Call a C-ABI entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def dtype_code(t):
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def ptr_array(ctype, values):
    """Host array of pointers/sizes for the multi-matrix entry points."""
    arr = (ctype * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


def stream_ptr(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    """The product path is CUDA-only: CPU tensors are an error, not a fallback."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("compressai_b200 kernels take CUDA tensors only (no CPU fallback); "
                             f"got a tensor on {t.device}")
