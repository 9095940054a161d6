"""The tcgen05 / TMEM / TMA batched GEMV (csrc/vq_gemm_umma.cu) against the fp64 oracle.

It serves multi-matrix GEMVs of M >= 4 rows whose 128-row tiles give every SM work (tall
matrices such as lm_head); smaller ones keep the split-K mma.sync kernel. Every output row is
checked against a torch fp32 decode of the same weights; a spread of rows (first tile, tile
boundaries, the ragged last tile) against the fp64 oracle. Tolerances: fp16 codebooks take
the activations rounded once to fp16, max|y - ref| / max|ref| <= 1e-3;
bf16 codebooks run hi + lo activation halves (2 bpw: fp32-level); at 3 bpw the two codebook rows
are summed and rounded to bf16 once per weight, held to the 4e-3 bf16 bar of the other tests.
"""
import numpy as np
import pytest
import torch

from compressai_b200 import _lib, kernels, runtime, synth, vq
from oracle import vq2_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3
TOL_BF16 = 4e-3


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.fixture(scope="module")
def cbs():
    return synth.random_codebooks(1)


def sample_rows(out):
    rows = set(range(0, 160)) | set(range(out - 160, out))
    rows |= {t * 128 + d for t in range(1, out // 128) for d in (-1, 0)}
    return np.array(sorted(r for r in rows if 0 <= r < out))


def kernel_names(fn):
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


def torch_ref(x, i0, i1, cb0, cb1, scale):
    """fp32 decode of the whole matrix on the GPU, then x . W^T (a plain torch restatement)."""
    w = cb0.float()[i0.long() & 0xFFFF]
    if i1 is not None:
        w = w + cb1.float()[i1.long()]
    w = w.reshape(i0.shape[0], -1) * scale.float()[:, None]
    return x.float() @ w.t()


@pytest.mark.parametrize("M", [4, 16, 24, 64, 100, 200])
@pytest.mark.parametrize("bits", [(16,), (16, 8)])
@pytest.mark.parametrize("cbdt", [torch.float16, torch.bfloat16])
def test_umma_tall_matrix_vs_oracle(cbs, M, bits, cbdt):
    out, n = 20000, 2048  # 157 tiles, the last one ragged (32 rows)
    idx, scale = synth.random_matrix(M + 7 * len(bits), out, n, bits)
    cbd = {k: torch.from_numpy(v.astype(np.float32)).to(DEV, cbdt) for k, v in cbs.items()}
    cb_np = {k: v.float().cpu().numpy() for k, v in cbd.items()}
    sc = torch.from_numpy(scale).to(DEV, cbdt)
    x = np.random.default_rng(M).standard_normal((M, n)).astype(np.float32)
    xd = torch.from_numpy(x).to(DEV)
    i0 = torch.from_numpy(idx[0]).to(DEV)
    i1 = torch.from_numpy(idx[1]).to(DEV) if len(bits) > 1 else None
    cb1 = cbd["16_8"] if i1 is not None else None
    _lib.load().vq2_tc_status(1)
    run = lambda: kernels.vq_gemv(xd, i0, cbd["16"], sc, i1=i1, cb1=cb1, out_dtype=torch.float32)  # noqa: E731
    names = kernel_names(run)
    assert any("vq_umma_kernel" in k for k in names), names
    y = run()
    torch.cuda.synchronize()
    assert _lib.load().vq2_tc_status(1) == 0
    tol = TOL_BF16 if (cbdt == torch.bfloat16 and i1 is not None) else TOL
    ref_all = torch_ref(xd, i0, i1, cbd["16"], cb1, sc)
    assert rel_err(y.cpu().numpy(), ref_all.cpu().numpy()) < tol
    rows = sample_rows(out)
    sc_np = sc.float().cpu().numpy()
    ref = np.stack([O.vq_gemv_legacy(x[m], idx[0][rows], cb_np["16"], sc_np[rows], 1.0,
                                     idx[1][rows] if i1 is not None else None, cb_np.get("16_8"))
                    for m in range(M)])
    assert rel_err(y.cpu().numpy()[:, rows], ref) < tol


def test_umma_bf16_hilo_is_fp32_accurate(cbs):
    """bf16 codebooks: the hi + lo activation halves keep the result at fp32-level accuracy."""
    out, n, M = 19200, 2048, 32
    idx, scale = synth.random_matrix(11, out, n)
    cb = torch.from_numpy(cbs["16"].astype(np.float32)).to(DEV, torch.bfloat16)
    sc = torch.from_numpy(scale).to(DEV, torch.bfloat16)
    x = torch.randn(M, n, device=DEV)
    i0 = torch.from_numpy(idx[0]).to(DEV)
    y = kernels.vq_gemv(x, i0, cb, sc, out_dtype=torch.float32)
    ref = torch_ref(x, i0, None, cb, None, sc)
    assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) < 5e-5


@pytest.mark.parametrize("M", [8, 64])
def test_umma_packed_linear_fused_rotation(cbs, M):
    """PackedLinear at batch M on a tall matrix: the RHT writes the fp16 operand, the tcgen05 GEMV
    consumes it; against the oracle's dequantize-then-matmul on a spread of rows."""
    out, n = 19456, 2048
    idx, scale = synth.random_matrix(5 + M, out, n)
    cbd = {k: torch.from_numpy(v).to(DEV) for k, v in cbs.items()}
    lin = runtime.PackedLinear((out, n), (16,), "lm_head", [torch.from_numpy(idx[0])], torch.from_numpy(scale),
                               cbd, DEV)
    x = np.random.default_rng(3).standard_normal((M, n)).astype(np.float16)
    xd = torch.from_numpy(x).to(DEV)
    assert any("vq_umma_kernel" in k for k in kernel_names(lambda: lin(xd)))
    y = lin(xd).float().cpu().numpy()
    rows = sample_rows(out)
    perm, sign, hb = O.rot_params("lm_head", n)
    ref = O.gemv_ref(x.astype(np.float64), [idx[0][rows]], (16,), cbs, scale[rows], perm, sign, hb)
    assert rel_err(y[:, rows], ref) < TOL


def test_umma_multi_matrix_problems(cbs):
    """Three matrices sharing one input (rows 8000, 8192, 9000: 198 tiles, problem edges inside the
    item list) in one launch, each against the torch fp32 reference."""
    n, M = 2048, 48
    outs = [8000, 8192, 9000]
    cbd = {k: torch.from_numpy(v).to(DEV) for k, v in cbs.items()}
    mats, refs = [], []
    x = torch.randn(M, n, device=DEV)
    for j, o in enumerate(outs):
        idx, scale = synth.random_matrix(40 + j, o, n)
        i0 = torch.from_numpy(idx[0]).to(DEV)
        sc = torch.from_numpy(scale).to(DEV)
        mats.append((i0, None, sc))
        refs.append(torch_ref(x, i0, None, cbd["16"], None, sc))
    Y = torch.empty(len(outs), M, max(outs), device=DEV)
    ys = [Y[j, :, :o] for j, o in enumerate(outs)]
    kernels.gemv_multi(x, mats, cbd["16"], None, out_dtype=torch.float32, ys=ys, y_row_stride=max(outs))
    for y, r in zip(ys, refs):
        assert rel_err(y.cpu().numpy(), r.cpu().numpy()) < TOL


def test_umma_small_matrix_keeps_split_k_kernel(cbs):
    """A 2048-row matrix has 16 tiles, too few for the persistent tcgen05 grid: the split-K
    mma.sync kernel serves it (hi + lo, fp32-level accuracy)."""
    idx, scale = synth.random_matrix(9, 2048, 2048)
    cbd = {k: torch.from_numpy(v).to(DEV) for k, v in cbs.items()}
    x = torch.randn(16, 2048, device=DEV)
    i0 = torch.from_numpy(idx[0]).to(DEV)
    sc = torch.from_numpy(scale).to(DEV)
    names = kernel_names(lambda: kernels.vq_gemv(x, i0, cbd["16"], sc, out_dtype=torch.float32))
    assert not any("vq_umma_kernel" in k for k in names) and any("vq_gemm_tc_kernel" in k for k in names)
    y = kernels.vq_gemv(x, i0, cbd["16"], sc, out_dtype=torch.float32)
    assert rel_err(y.cpu().numpy(), torch_ref(x, i0, None, cbd["16"], None, sc).cpu().numpy()) < 3e-5
