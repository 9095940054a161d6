"""The allocation-free MoE expert FFN entry point (vq2_moe_expert_ffn_noalloc).

It exists for callers that cannot obtain device memory when they call in -- plugin interfaces
whose enqueue step must not block on an allocation, or hosts reaching the library through an
FFI without a device allocator. Its scratch is a static device array inside the library, so
this test checks it against the workspace-taking entry point, vq2_moe_expert_ffn, over the
C-ABI on two calls in a row with different inputs (the second call must not see anything left
over by the first), against the fp64 oracle once, at the largest accepted problem count (340
(token, expert) problems) and that the first count past the static scratch is refused. Kept in
its own file, collected last.
"""
import numpy as np
import pytest
import torch

from compressai_b200 import _lib, moe, synth, vq
from oracle import vq2_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-6   # same kernels and launch shapes on both paths: results agree to fp32 rounding


def _setup():
    E = 12
    pool = moe.ExpertRecordPool(E, DEV)
    for e in range(E):
        pool.set_expert(e, *[torch.from_numpy(a) for a in synth.synth_expert(77, e)])
    cb = torch.from_numpy(synth.random_codebooks(3)["16"]).to(DEV)
    r_in = vq.get_rot("moe_expert_2048", 2048, DEV)
    r_mid = vq.get_rot("moe_expert_512", 512, DEV)
    return E, pool, cb, r_in, r_mid


def _args(h, T, K, ids, w, E, pool, cb, r_in, r_mid):
    return [_lib.ptr(h), _lib.dtype_code(h), T, K, _lib.ptr(ids), _lib.ptr(w), _lib.ptr(pool.raw), E, 1024, 256,
            2048, 64, _lib.ptr(cb), _lib.VQ2_F16, _lib.ptr(r_in.perm), _lib.ptr(r_in.sign), r_in.hb,
            float(r_in.scale), _lib.ptr(r_mid.perm), _lib.ptr(r_mid.sign), r_mid.hb, float(r_mid.scale)]


@pytest.mark.parametrize("shapes", [[(4, 8), (2, 5)], [(34, 10), (1, 3)]])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(shapes):
    """Two calls in a row; the second list starts at the largest accepted size (34 x 10 = 340
    problems, 4,183,040 of the 4,194,304 scratch bytes)."""
    lib = _lib.load()
    E, pool, cb, r_in, r_mid = _setup()
    st = _lib.stream_ptr(DEV)
    rng = np.random.default_rng(5)
    for call, (T, K) in enumerate(shapes):
        h = torch.from_numpy(rng.standard_normal((T, 2048)).astype(np.float16)).to(DEV)
        ids = torch.from_numpy(rng.integers(0, E, size=T * K).astype(np.int32)).to(DEV)
        w = torch.from_numpy(rng.random((T, K)).astype(np.float32)).to(DEV)
        base = _args(h, T, K, ids, w, E, pool, cb, r_in, r_mid)

        ref = torch.empty(T, 2048, dtype=torch.float32, device=DEV)
        ws_bytes = lib.vq2_moe_expert_ffn_workspace(T, K, 1024, 2048)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        _lib.check(lib.vq2_moe_expert_ffn(*base, _lib.ptr(ws), ws_bytes, _lib.ptr(ref), _lib.VQ2_F32, st),
                   "vq2_moe_expert_ffn")

        out = torch.full((T, 2048), float("nan"), dtype=torch.float32, device=DEV)
        _lib.check(lib.vq2_moe_expert_ffn_noalloc(*base, _lib.ptr(out), _lib.VQ2_F32, st),
                   "vq2_moe_expert_ffn_noalloc")
        torch.cuda.synchronize()
        r, o = ref.cpu().numpy().astype(np.float64), out.cpu().numpy().astype(np.float64)
        assert np.isfinite(o).all(), f"call {call}: output not fully written"
        err = np.abs(o - r).max() / max(np.abs(r).max(), 1e-30)
        assert err <= TOL, f"call {call}: max rel err {err}"


def test_noalloc_matches_oracle():
    """One call against the fp64 oracle of the reference's expert path (1e-3, fp16 output)."""
    lib = _lib.load()
    E, pool, cb, r_in, r_mid = _setup()
    cb_np = synth.random_codebooks(3)["16"]
    rng = np.random.default_rng(9)
    T, K = 3, 8
    h_np = rng.standard_normal((T, 2048)).astype(np.float16)
    ids_np = rng.integers(0, E, size=(T, K)).astype(np.int32)
    w_np = rng.random((T, K)).astype(np.float32)
    h = torch.from_numpy(h_np).to(DEV)
    ids = torch.from_numpy(ids_np.reshape(-1)).to(DEV)
    w = torch.from_numpy(w_np).to(DEV)
    out = torch.empty(T, 2048, dtype=torch.float16, device=DEV)
    _lib.check(lib.vq2_moe_expert_ffn_noalloc(*_args(h, T, K, ids, w, E, pool, cb, r_in, r_mid), _lib.ptr(out),
                                              _lib.VQ2_F16, _lib.stream_ptr(DEV)), "vq2_moe_expert_ffn_noalloc")
    torch.cuda.synchronize()
    ref = O.moe_layer_ref(h_np, ids_np, w_np, lambda e: synth.synth_expert(77, e), cb_np,
                          O.rot_params("moe_expert_2048", 2048), O.rot_params("moe_expert_512", 512))
    y = out.float().cpu().numpy().astype(np.float64)
    assert np.abs(y - ref).max() / np.abs(ref).max() <= 1e-3


@pytest.mark.parametrize("T,K", [(31, 11), (64, 8)])
def test_noalloc_refuses_problems_beyond_its_scratch(T, K):
    """341 problems (the first count past the 4 MiB scratch) and 512 are refused."""
    lib = _lib.load()
    E, pool, cb, r_in, r_mid = _setup()
    assert lib.vq2_moe_expert_ffn_workspace(T, K, 1024, 2048) > 4 * 1024 * 1024
    assert lib.vq2_moe_expert_ffn_workspace(34, 10, 1024, 2048) <= 4 * 1024 * 1024
    h = torch.zeros(T, 2048, dtype=torch.float16, device=DEV)
    ids = torch.zeros(T * K, dtype=torch.int32, device=DEV)
    w = torch.zeros(T, K, dtype=torch.float32, device=DEV)
    out = torch.empty(T, 2048, dtype=torch.float32, device=DEV)
    st = lib.vq2_moe_expert_ffn_noalloc(*_args(h, T, K, ids, w, E, pool, cb, r_in, r_mid), _lib.ptr(out),
                                        _lib.VQ2_F32, _lib.stream_ptr(DEV))
    assert st == _lib.VQ2_ERR_SHAPE
