"""CUDA kernels vs the CPU oracle (oracle/vq2_oracle.py), through the C-ABI.

Tolerances: fp32 RHT vs the fp64 oracle 1e-5 relative to max|ref|; GEMV outputs in fp16
max|y - ref| / max|ref| <= 1e-3; bf16 outputs 4e-3 (bf16 rounding
alone is 2^-9 of |y|).
"""
import numpy as np
import pytest
import torch

from compressai_b200 import kernels, synth, vq
from oracle import vq2_oracle as O
from tests.conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL_F16 = 1e-3
TOL_BF16 = 4e-3


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.fixture(scope="module")
def cbs():
    try:
        d = golden("codebooks.npz")
        return {"16": d["cb16"], "16_8": d["cb16_8"]}
    except pytest.skip.Exception:
        return synth.random_codebooks(1)


def dev_cbs(cbs, dtype=torch.float16):
    return {k: torch.from_numpy(v.astype(np.float32)).to(DEV, dtype).contiguous() for k, v in cbs.items()}


# ------------------------------------------------------------------------------------------ RHT
@pytest.mark.parametrize("tag,n", [("dense_q", 2048), ("moe_expert_512", 512), ("mlp_down", 6144),
                                   ("small_1024", 1024), ("t64", 64), ("t128", 128), ("t256", 256)])
@pytest.mark.parametrize("M", [1, 3, 17])
def test_rht_forward_inverse(tag, n, M):
    rot = vq.get_rot(tag, n, DEV)
    perm, sign, hb = O.rot_params(tag, n)
    assert np.array_equal(rot.perm_cpu.numpy(), perm)
    x = torch.randn(M, n, generator=torch.Generator().manual_seed(n + M))
    y = rot.fwd_f32(x.to(DEV)).cpu().numpy()
    ref = O.rht_fwd(x.numpy(), perm, sign, hb)
    assert rel_err(y, ref) < 1e-5
    z = rot.inv_f32(torch.from_numpy(ref.astype(np.float32)).to(DEV)).cpu().numpy()
    assert rel_err(z, x.numpy()) < 1e-5
    # unnormalised (FastRot) variant
    yu = rot.fwd_f32(x.to(DEV), unnormalised=True).cpu().numpy()
    assert rel_err(yu, ref * hb ** 0.5) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rht_input_dtypes(dtype):
    rot = vq.get_rot("attn", 2048, DEV)
    x = torch.randn(2, 2048, generator=torch.Generator().manual_seed(3)).to(dtype)
    y = rot.fwd_f32(x.to(DEV)).cpu().numpy()
    ref = O.rht_fwd(x.float().numpy(), *O.rot_params("attn", 2048))
    assert rel_err(y, ref) < 1e-5


def test_rht_matches_reference_golden():
    d = golden("rot.npz")
    for tag, n in [("dense_q", 2048), ("mlp_down", 6144), ("moe_expert_512", 512), ("small_1024", 1024)]:
        key = f"{tag}_{n}"
        rot = vq.get_rot(tag, n, DEV)
        x = torch.from_numpy(d[f"x_{key}"]).to(DEV)
        assert rel_err(rot.fwd_f32(x).cpu().numpy(), d[f"fwd_{key}"]) < 1e-5
        assert rel_err(rot.inv_f32(x).cpu().numpy(), d[f"inv_{key}"]) < 1e-5


def test_swiglu_rht():
    rot = vq.get_rot("moe_expert_512", 512, DEV)
    gu = torch.randn(9, 1024, generator=torch.Generator().manual_seed(4))
    out = kernels.swiglu_rht(gu.to(DEV), rot).cpu().numpy()
    g, u = gu[:, :512].double().numpy(), gu[:, 512:].double().numpy()
    ref = O.rht_fwd(O.silu(g) * u, *O.rot_params("moe_expert_512", 512))
    assert rel_err(out, ref) < 2e-5


# ----------------------------------------------------------------------------------------- GEMV
def run_packed(idx, scale, x, tag, cbs_dev, out_dtype=None):
    """Rotate x (fp32 RHT) then GEMV, as PackedLinear.forward does."""
    out, ng = idx[0].shape
    n = ng * 8
    rot = vq.get_rot(tag, n, DEV)
    xr = rot.fwd_f32(torch.from_numpy(np.asarray(x)).to(DEV))
    i0 = torch.from_numpy(np.ascontiguousarray(idx[0])).to(DEV)
    i1 = torch.from_numpy(np.ascontiguousarray(idx[1])).to(DEV) if len(idx) > 1 else None
    sc = torch.from_numpy(np.asarray(scale)).to(DEV, cbs_dev["16"].dtype)
    y = kernels.vq_gemv(xr, i0, cbs_dev["16"], sc, i1=i1, cb1=cbs_dev["16_8"] if i1 is not None else None,
                        out_dtype=out_dtype or torch.float16)
    return y.float().cpu().numpy()


def test_gemv_golden_cases(cbs):
    d = golden("gemv.npz")
    cbd = dev_cbs(cbs)
    names = sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_meta")})
    assert "cfg1" in names
    for nm in names:
        out, n, nst, M = d[f"{nm}_meta"]
        idx = [d[f"{nm}_idx0"]] + ([d[f"{nm}_idx1"]] if nst > 1 else [])
        y = run_packed(idx, d[f"{nm}_scale"], d[f"{nm}_x"], str(d[f"{nm}_tag"]), cbd)
        err = rel_err(y, d[f"{nm}_y"])
        assert err < TOL_F16, (nm, err)


@pytest.mark.parametrize("out,n,bits,M", [
    (2048, 2048, (16,), 1), (2048, 2048, (16, 8), 1), (6144, 2048, (16,), 4), (2048, 6144, (16,), 1),
    (2048, 6144, (16, 8), 4), (1000, 2048, (16,), 16), (512, 2048, (16, 8), 64), (300, 512, (16,), 3),
    (128, 256, (16,), 2), (2048, 2048, (16,), 64), (40, 4096, (16, 8), 9),
])
def test_gemv_random_vs_oracle(cbs, out, n, bits, M):
    idx, scale = synth.random_matrix(out * 7 + n, out, n, bits)
    x = np.random.default_rng(M).standard_normal((M, n)).astype(np.float16)
    tag = f"rand_{n}"
    y = run_packed(idx, scale, x, tag, dev_cbs(cbs))
    perm, sign, hb = O.rot_params(tag, n)
    ref = O.gemv_ref(x.astype(np.float64), idx, bits, cbs, scale, perm, sign, hb)
    assert rel_err(y, ref) < TOL_F16


@pytest.mark.parametrize("out_dtype,tol", [(torch.bfloat16, TOL_BF16), (torch.float32, 2e-5)])
def test_gemv_output_dtypes(cbs, out_dtype, tol):
    idx, scale = synth.random_matrix(5, 512, 2048)
    x = np.random.default_rng(0).standard_normal((2, 2048)).astype(np.float32)
    y = run_packed(idx, scale, x, "dense_q", dev_cbs(cbs), out_dtype=out_dtype)
    ref = O.gemv_ref(x, idx, (16,), cbs, scale, *O.rot_params("dense_q", 2048))
    assert rel_err(y, ref) < tol


def test_legacy_signatures_bf16(cbs):
    """vq_gemv_16 / vq_gemv_16_8 with the reference's bf16 codebooks/scales and rs = 2048^-0.5."""
    idx, scale = synth.random_matrix(9, 1024, 2048, (16, 8))
    cbd = dev_cbs(cbs, torch.bfloat16)
    xr = torch.randn(2048, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    i0 = torch.from_numpy(idx[0]).to(DEV)
    i1 = torch.from_numpy(idx[1]).to(DEV)
    sc = torch.from_numpy(scale).to(DEV, torch.bfloat16)
    rs = 2048 ** -0.5
    y2 = kernels.vq_gemv_16(xr, i0, cbd["16"], sc, 1024, 2048, rs)
    y3 = kernels.vq_gemv_16_8(xr, i0, i1, cbd["16"], cbd["16_8"], sc, 1024, 2048, rs)
    assert y2.dtype == torch.bfloat16 and y2.shape == (1024,)
    cb16 = cbd["16"].float().cpu().numpy()
    cb8 = cbd["16_8"].float().cpu().numpy()
    scf = sc.float().cpu().numpy()
    xf = xr.float().cpu().numpy()
    assert rel_err(y2.float().cpu(), O.vq_gemv_legacy(xf, idx[0], cb16, scf, rs)) < TOL_BF16
    assert rel_err(y3.float().cpu(), O.vq_gemv_legacy(xf, idx[0], cb16, scf, rs, idx[1], cb8)) < TOL_BF16


# ------------------------------------------------------------------------------------ MoE GEMV
def _pool(E, seed):
    ex = [synth.synth_expert(seed, e) for e in range(E)]
    return [np.stack([x[i] for x in ex]) for i in range(4)]


def test_moe_legacy_gate_up_down(cbs):
    E = 12
    gu_i, gu_s, dn_i, dn_s = _pool(E, 3)
    cbd = dev_cbs(cbs)
    slots = np.array([3, 0, 11, 7, 7, 2, 9, 5], dtype=np.int32)
    xr = torch.randn(2048, generator=torch.Generator().manual_seed(2)).to(DEV, torch.float16)
    y_gu = torch.empty(8, 1024, device=DEV, dtype=torch.float16)
    kernels.vq_moe_parallel_gate_up(xr, torch.from_numpy(slots).to(DEV), torch.from_numpy(gu_i).to(DEV), cbd["16"],
                                    torch.from_numpy(gu_s).to(DEV), y_gu)
    ref = O.moe_gate_up_ref(xr.float().cpu().numpy(), slots, gu_i, cbs["16"], gu_s)
    assert rel_err(y_gu.float().cpu(), ref) < TOL_F16
    act = torch.randn(8, 512, generator=torch.Generator().manual_seed(5)).to(DEV, torch.float16)
    y_dn = torch.empty(8, 2048, device=DEV, dtype=torch.float16)
    kernels.vq_moe_parallel_down(act, torch.from_numpy(slots).to(DEV), torch.from_numpy(dn_i).to(DEV), cbd["16"],
                                 torch.from_numpy(dn_s).to(DEV), y_dn)
    ref = O.moe_down_ref(act.float().cpu().numpy(), slots, dn_i, cbs["16"], dn_s)
    assert rel_err(y_dn.float().cpu(), ref) < TOL_F16


def test_moe_gemv_out_of_range_ids_give_zero_rows(cbs):
    gu_i, gu_s, _, _ = _pool(4, 1)
    cbd = dev_cbs(cbs)
    ids = torch.tensor([1, -1, 4, 2], dtype=torch.int32, device=DEV)
    x = torch.randn(2048, device=DEV)
    y = torch.full((4, 1024), 7.0, device=DEV)
    kernels.moe_gemv(x, ids, torch.from_numpy(gu_i).to(DEV), cbd["16"], torch.from_numpy(gu_s).to(DEV), y,
                     x_k_stride=0)
    y = y.cpu()
    assert torch.all(y[1] == 0) and torch.all(y[2] == 0)
    assert torch.any(y[0] != 0) and torch.any(y[3] != 0)


def test_moe_combine():
    T, K, H = 3, 8, 2048
    y = torch.randn(T * K, H, device=DEV)
    w = torch.rand(T, K, device=DEV)
    add = torch.randn(T, H, device=DEV)
    out = kernels.moe_combine(y, w, K, add=add, out_dtype=torch.float32)
    ref = (y.view(T, K, H).double() * w.double()[:, :, None]).sum(1) + add.double()
    assert rel_err(out.cpu(), ref.cpu()) < 1e-6


# ------------------------------------------------------------------ fused prologues / multi
def _dev_mat(idx, scale, dtype=torch.float16):
    i0 = torch.from_numpy(np.ascontiguousarray(idx[0])).to(DEV)
    i1 = torch.from_numpy(np.ascontiguousarray(idx[1])).to(DEV) if len(idx) > 1 else None
    return (i0, i1, torch.from_numpy(np.asarray(scale)).to(DEV, dtype))


def test_packed_linear_fused_rht_golden(cbs):
    """PackedLinear.forward (RHT fused in the GEMV prologue) on the reference-quantized cases."""
    from compressai_b200 import runtime
    d = golden("gemv.npz")
    cbd = dev_cbs(cbs)
    names = sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_meta")})
    for nm in names:
        out, n, nst, M = d[f"{nm}_meta"]
        cfg = (16,) if nst == 1 else (16, 8)
        idx = [torch.from_numpy(d[f"{nm}_idx0"])] + ([torch.from_numpy(d[f"{nm}_idx1"])] if nst > 1 else [])
        lin = runtime.PackedLinear((int(out), int(n)), cfg, str(d[f"{nm}_tag"]), idx,
                                   torch.from_numpy(d[f"{nm}_scale"]), cbd, DEV)
        y = lin(torch.from_numpy(d[f"{nm}_x"]).to(DEV)).float().cpu().numpy()
        assert rel_err(y, d[f"{nm}_y"]) < TOL_F16, nm


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("bits", [(16,), (16, 8)])
def test_gemv_multi_shared_input(cbs, M, bits):
    """q/k/v-style group: 3 matrices of different heights, one input, one launch."""
    from compressai_b200 import runtime
    cbd = dev_cbs(cbs)
    outs = [2048, 512, 768]
    mods = []
    mats_np = []
    for j, o in enumerate(outs):
        idx, scale = synth.random_matrix(100 + j, o, 2048, bits)
        mats_np.append((idx, scale))
        mods.append(runtime.PackedLinear((o, 2048), bits, "attn_in", [torch.from_numpy(i) for i in idx],
                                         torch.from_numpy(scale), cbd, DEV))
    x = np.random.default_rng(M).standard_normal((M, 2048)).astype(np.float16)
    ys = runtime.PackedLinearGroup(mods)(torch.from_numpy(x).to(DEV)) if M == 1 else \
        [m(torch.from_numpy(x).to(DEV)) for m in mods]
    perm, sign, hb = O.rot_params("attn_in", 2048)
    for (idx, scale), y in zip(mats_np, ys):
        ref = O.gemv_ref(x, idx, bits, cbs, scale, perm, sign, hb)
        assert rel_err(y.float().cpu().numpy().reshape(ref.shape), ref) < TOL_F16
    if M > 1:  # grouped with an explicit output row stride
        yb = torch.empty(M, sum(outs), device=DEV, dtype=torch.float16)
        offs = np.cumsum([0] + outs)
        cb0, cb1 = mods[0].codebooks()
        kernels.gemv_multi(torch.from_numpy(x).to(DEV), [m.mat() for m in mods], cb0, cb1, rot=mods[0].rot,
                           ys=[yb[:, offs[j]:offs[j + 1]] for j in range(3)], y_row_stride=sum(outs))
        for j, (idx, scale) in enumerate(mats_np):
            ref = O.gemv_ref(x, idx, bits, cbs, scale, perm, sign, hb)
            assert rel_err(yb[:, offs[j]:offs[j + 1]].float().cpu().numpy(), ref) < TOL_F16


@pytest.mark.parametrize("M", [1, 4])
def test_packed_swiglu_mlp(cbs, M):
    from compressai_b200 import runtime
    cbd = dev_cbs(cbs)
    gi, gs = synth.random_matrix(1, 6144, 2048)
    ui, us = synth.random_matrix(2, 6144, 2048)
    di, ds = synth.random_matrix(3, 2048, 6144)
    mk = lambda idx, sc, o, n, tag: runtime.PackedLinear((o, n), (16,), tag, [torch.from_numpy(idx[0])],
                                                         torch.from_numpy(sc), cbd, DEV)
    mlp = runtime.PackedSwiGLUMLP(mk(gi, gs, 6144, 2048, "mlp_in"), mk(ui, us, 6144, 2048, "mlp_in"),
                                  mk(di, ds, 2048, 6144, "mlp_down"))
    x = np.random.default_rng(7).standard_normal((M, 2048)).astype(np.float16)
    y = mlp(torch.from_numpy(x).to(DEV)).float().cpu().numpy()
    r_in = O.rot_params("mlp_in", 2048)
    g = O.gemv_ref(x, gi, (16,), cbs, gs, *r_in)
    u = O.gemv_ref(x, ui, (16,), cbs, us, *r_in)
    ref = O.gemv_ref(O.silu(g) * u, di, (16,), cbs, ds, *O.rot_params("mlp_down", 6144))
    assert rel_err(y, ref) < TOL_F16


def test_moe_gemv_fused_modes(cbs):
    """Expert-indexed GEMVs with the RHT (gate_up) and SwiGLU+RHT (down) prologues."""
    E = 10
    gu_i, gu_s, dn_i, dn_s = _pool(E, 5)
    cbd = dev_cbs(cbs)
    r2048 = vq.get_rot("moe_expert_2048", 2048, DEV)
    r512 = vq.get_rot("moe_expert_512", 512, DEV)
    T, K = 3, 4
    ids = np.array([[1, 4, 9, 0], [4, 4, 2, 7], [3, 8, 5, 6]], dtype=np.int32)
    h = np.random.default_rng(3).standard_normal((T, 2048)).astype(np.float16)
    ids_d = torch.from_numpy(ids.reshape(-1)).to(DEV)
    gu = torch.empty(T * K, 1024, device=DEV)
    kernels.moe_gemv(torch.from_numpy(h).to(DEV), ids_d, torch.from_numpy(gu_i).to(DEV), cbd["16"],
                     torch.from_numpy(gu_s).to(DEV), gu, x_k_stride=2048, x_k_div=K, rot=r2048)
    y_dn = torch.empty(T * K, 2048, device=DEV)
    kernels.moe_gemv(gu, ids_d, torch.from_numpy(dn_i).to(DEV), cbd["16"], torch.from_numpy(dn_s).to(DEV), y_dn,
                     x_k_stride=1024, rot=r512, mode=2)
    rot2048 = O.rot_params("moe_expert_2048", 2048)
    rot512 = O.rot_params("moe_expert_512", 512)
    for t in range(T):
        xr = O.rht_fwd(h[t].astype(np.float64), *rot2048)
        for j in range(K):
            e = ids[t, j]
            g = O.vq_gemv_legacy(xr, gu_i[e], cbs["16"], gu_s[e], 1.0)
            assert rel_err(gu[t * K + j].cpu().numpy(), g) < 2e-5
            act_r = O.rht_fwd(O.silu(g[:512]) * g[512:], *rot512)
            ref = O.vq_gemv_legacy(act_r, dn_i[e], cbs["16"], dn_s[e], 1.0)
            assert rel_err(y_dn[t * K + j].cpu().numpy(), ref) < 2e-5


@pytest.mark.parametrize("M", [8, 24, 64, 100])
@pytest.mark.parametrize("bits", [(16,), (16, 8)])
@pytest.mark.parametrize("cbdt", [torch.float16, torch.bfloat16])
def test_tensor_core_batched_gemv(cbs, M, bits, cbdt):
    """M >= 8 runs on the tensor cores (activations split hi + lo): fp32 outputs agree with the
    fp64 oracle to fp32-accumulation accuracy, for fp16 and bf16 codebooks, 2 and 3 bpw."""
    out, n = 300, 2048
    idx, scale = synth.random_matrix(M + len(bits), out, n, bits)
    cbd = dev_cbs(cbs, cbdt)
    cb_np = {k: v.float().cpu().numpy() for k, v in cbd.items()}   # the values the kernel sees
    sc = torch.from_numpy(scale).to(DEV, cbdt)
    x = np.random.default_rng(M).standard_normal((M, n)).astype(np.float32)
    xr = torch.from_numpy(x).to(DEV)
    i0 = torch.from_numpy(idx[0]).to(DEV)
    i1 = torch.from_numpy(idx[1]).to(DEV) if len(bits) > 1 else None
    y = kernels.vq_gemv(xr, i0, cbd["16"], sc, i1=i1, cb1=cbd["16_8"] if i1 is not None else None,
                        out_dtype=torch.float32).cpu().numpy()
    ref = np.stack([O.vq_gemv_legacy(x[m], idx[0], cb_np["16"], sc.float().cpu().numpy(), 1.0,
                                     idx[1] if len(bits) > 1 else None, cb_np["16_8"]) for m in range(M)])
    assert rel_err(y, ref) < 3e-5


@pytest.mark.parametrize("out,n,M,tol", [(2048, 6144, 16, 3e-5), (9000, 1024, 24, 3e-5), (40000, 2048, 8, 1e-3),
                                         (130, 256, 64, 3e-5)])
def test_tensor_core_split_k_shapes(cbs, out, n, M, tol):
    """Split-K over thread-block clusters (items that fill less than half the GPU: S = 8, 4, and
    K too short to split) agrees with the fp64 oracle to fp32 accuracy (hi + lo operands); the
    40000-row matrix has a 128-row tile per SM and runs on the tcgen05 kernel (fp16 operand:
    1e-3)."""
    idx, scale = synth.random_matrix(out + n, out, n)
    cbd = dev_cbs(cbs)
    sc = torch.from_numpy(scale).to(DEV)
    x = np.random.default_rng(out).standard_normal((M, n)).astype(np.float32)
    y = kernels.vq_gemv(torch.from_numpy(x).to(DEV), torch.from_numpy(idx[0]).to(DEV), cbd["16"], sc,
                        out_dtype=torch.float32).cpu().numpy()
    cb_np = cbd["16"].float().cpu().numpy()
    ref = np.stack([O.vq_gemv_legacy(x[m], idx[0], cb_np, scale.astype(np.float32), 1.0) for m in range(M)])
    assert rel_err(y, ref) < tol


def test_tensor_core_path_without_workspace_falls_back_exactly(cbs):
    """vq2_gemv with M >= 8 but no workspace runs the CUDA-core kernel: same result."""
    from compressai_b200 import _lib
    idx, scale = synth.random_matrix(3, 256, 2048)
    cbd = dev_cbs(cbs)
    x = torch.randn(16, 2048, device=DEV)
    i0 = torch.from_numpy(idx[0]).to(DEV)
    sc = torch.from_numpy(scale).to(DEV)
    y_tc = kernels.vq_gemv(x, i0, cbd["16"], sc, out_dtype=torch.float32)
    y_cc = torch.empty(16, 256, device=DEV)
    _lib.call("vq2_gemv", _lib.ptr(x), _lib.VQ2_F32, 16, 2048, _lib.ptr(i0), None, _lib.ptr(cbd["16"]), None,
              _lib.ptr(sc), _lib.VQ2_F16, _lib.ptr(y_cc), _lib.VQ2_F32, 256, 256, 2048, 1.0, None, 0,
              _lib.stream_ptr(DEV))
    assert rel_err(y_cc.cpu().numpy(), y_tc.cpu().numpy()) < 3e-5


def test_greedy_argmax_matches_reference_on_golden(cbs):
    """vq2_gemv_argmax (keys and ids) on every golden case -- matrices quantized by the
    reference's own quantizer, y computed by the reference's dequantize + fp64 matmul -- picks the
    reference's argmax row for every activation row; a row whose reference logit is within the
    GEMV tolerance of the maximum counts as a tie."""
    from compressai_b200 import runtime
    d = golden("gemv.npz")
    cbd = dev_cbs(cbs)
    names = sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_meta")})
    checked = 0
    for nm in names:
        out, n, nst, M = (int(v) for v in d[f"{nm}_meta"])
        bits = (16, 8) if nst > 1 else (16,)
        idx = [d[f"{nm}_idx0"]] + ([d[f"{nm}_idx1"]] if nst > 1 else [])
        lin = runtime.PackedLinear((out, n), bits, str(d[f"{nm}_tag"]),
                                   [torch.from_numpy(np.ascontiguousarray(a)) for a in idx],
                                   torch.from_numpy(np.asarray(d[f"{nm}_scale"])), cbd, DEV)
        x = torch.from_numpy(np.asarray(d[f"{nm}_x"])).to(DEV)
        got = lin.greedy(x).cpu().numpy()
        ref = np.asarray(d[f"{nm}_y"], dtype=np.float64).reshape(M, out)
        tol = TOL_F16 * np.abs(ref).max()
        for m in range(M):
            assert ref[m, got[m]] >= ref[m].max() - tol, (nm, m, int(got[m]), int(ref[m].argmax()))
            checked += 1
    assert checked >= len(names)


@pytest.mark.parametrize("M,bits,ties", [(1, (16,), False), (3, (16, 8), False), (2, (16,), True)])
def test_lm_head_fused_greedy_argmax(cbs, M, bits, ties):
    """vq2_gemv_argmax: the argmax of each activation row equals torch.argmax of the GEMV's own
    logits (ties to the smaller row), with and without the logits written."""
    from compressai_b200 import runtime
    out, n = 20000, 2048
    idx, scale = synth.random_matrix(M + 50, out, n, bits)
    if ties:   # three identical rows with a large scale: equal maximal logits at 123, 7000, 19999
        idx = [a.copy() for a in idx]
        for a in idx:
            a[7000] = a[123]
            a[19999] = a[123]
        scale = scale.copy()
        scale[[123, 7000, 19999]] = 100.0
    cbd = dev_cbs(cbs)
    lin = runtime.PackedLinear((out, n), bits, "lm_head_t", [torch.from_numpy(a) for a in idx],
                               torch.from_numpy(scale), cbd, DEV)
    x = torch.randn(M, n, device=DEV).half()
    logits = lin(x).float()
    if ties:   # make row 123's logit positive for every activation row, so its twins tie at the max
        x = torch.where((logits[:, 123] < 0)[:, None], -x, x)
        logits = lin(x).float()
    got = lin.greedy(x)
    y = torch.empty(M, out, device=DEV, dtype=torch.float32)
    got2 = lin.greedy(x, logits=y)
    # the fused kernel's own fp32 logits decide; lin(x) may run on tensor cores (another sum order;
    # at this height the tcgen05 kernel, whose fp16 activation operand errs by ~2^-12 of each
    # row's |w| |x|: the three rows scaled x100 are compared through the argmax only)
    assert torch.equal(got, torch.argmax(y, dim=-1)) and torch.equal(got2, got)
    keep = torch.ones(out, dtype=torch.bool, device=DEV)
    if ties:
        keep[[123, 7000, 19999]] = False
    assert (y - logits)[:, keep].abs().max() <= 1e-3 * logits[:, keep].abs().max()
    assert torch.equal(got, torch.argmax(logits, dim=-1))
    if ties:
        assert (got == 123).all()


@pytest.mark.parametrize("swiglu", [False, True])
@pytest.mark.parametrize("n", [2048, 6144])
@pytest.mark.parametrize("M", [1, 2, 3, 8, 16])
def test_fused_staging_bitwise_equals_separate_transform(cbs, M, n, swiglu):
    """The fused transform gives the same bits as the standalone transform kernel followed by a
    GEMV on the pre-rotated rows: both compute the same fp32 values in the same order. M <= 3:
    the CUDA-core prologue's staging (rotation table in shared memory, coalesced row loads, one
    raw row per round for M tiles that do not fit). M >= 4: the tensor-core path's transform +
    hi/lo split in one launch against the transform followed by the split kernel."""
    from compressai_b200 import _lib
    out = 1000
    idx, scale = synth.random_matrix(7 + M, out, n, (16,))
    cbd = dev_cbs(cbs)
    mat = (torch.from_numpy(idx[0]).to(DEV), None, torch.from_numpy(scale).to(DEV, cbd["16"].dtype))
    rot = vq.get_rot("mlp_down" if n == 6144 else "dense_q", n, DEV)
    if swiglu:
        x = torch.randn(M, 2 * n, device=DEV)
        xr = kernels.swiglu_rht(x, rot)
        mode = _lib.VQ2_ACT_SWIGLU_RHT
    else:
        x = torch.randn(M, n, device=DEV).half()
        xr = rot.fwd_f32(x)
        mode = _lib.VQ2_ACT_RHT
    y_fused = kernels.gemv_multi(x, [mat], cbd["16"], None, rot=rot, mode=mode, out_dtype=torch.float32)[0]
    y_split = kernels.gemv_multi(xr, [mat], cbd["16"], None, mode=_lib.VQ2_ACT_ROTATED, out_dtype=torch.float32)[0]
    assert torch.equal(y_fused, y_split)
