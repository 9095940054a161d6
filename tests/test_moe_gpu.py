"""MoE path on the GPU vs the oracle and the reference's golden outputs: router, resident
experts, MoE block with shared expert, paged experts (all store modes) with bit-exact LRU."""
import numpy as np
import pytest
import torch

from compressai_b200 import container, moe, paged_runtime, synth
from oracle import vq2_oracle as O
from tests.conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3


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


def cb16_dev(cbs):
    return torch.from_numpy(cbs["16"]).to(DEV)


ROT2048 = O.rot_params("moe_expert_2048", 2048)
ROT512 = O.rot_params("moe_expert_512", 512)


@pytest.mark.parametrize("T,E,K", [(1, 256, 8), (32, 256, 8), (5, 64, 4), (3, 1000, 16)])
def test_router_matches_reference_math(T, E, K):
    logits = np.random.default_rng(T * E).standard_normal((T, E)).astype(np.float32)
    ids, w = moe.route(torch.from_numpy(logits).to(DEV), K)
    rid, rw = O.router_ref(logits, K)
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.abs(w.cpu().numpy() - rw).max() < 1e-6


def test_router_golden_and_shared_gate():
    d = golden("moe.npz")
    for nm in ("t1", "t4"):
        ids, w = moe.route(torch.from_numpy(d[f"{nm}_logits"]).to(DEV), 8)
        assert np.array_equal(ids.cpu().numpy(), d[f"{nm}_ids"])
        assert np.abs(w.cpu().numpy() - d[f"{nm}_w"]).max() < 1e-6
    h = np.random.default_rng(0).standard_normal((4, 2048)).astype(np.float16)
    g = (0.02 * np.random.default_rng(1).standard_normal(2048)).astype(np.float32)
    lg = torch.randn(4, 256, device=DEV)
    _, _, sw = moe.route(lg, 8, torch.from_numpy(h).to(DEV), torch.from_numpy(g).to(DEV))
    ref = 1 / (1 + np.exp(-(h.astype(np.float64) @ g.astype(np.float64))))
    assert np.abs(sw.cpu().numpy() - ref).max() < 1e-5


def resident_pool(seed, E, extra=None):
    pool = moe.ExpertRecordPool(E + (1 if extra is not None else 0), DEV)
    for e in range(E):
        pool.set_expert(e, *[torch.from_numpy(a) for a in synth.synth_expert(seed, e)])
    if extra is not None:
        pool.set_expert(E, *[torch.from_numpy(a) for a in extra])
    return pool


def test_resident_moe_matches_reference_golden(cbs):
    """PackedMoEExpertUniversal vs the reference's own CPU expert path (golden)."""
    d = golden("moe.npz")
    seed = int(d["t1_seed"])
    pool = resident_pool(seed, 256)
    ex = moe.PackedMoEExpertUniversal(pool, cb16_dev(cbs), DEV)
    for nm in ("t1", "t4"):
        h = torch.from_numpy(d[f"{nm}_h"]).to(DEV)
        y = ex(h, torch.from_numpy(d[f"{nm}_ids"]).to(DEV), torch.from_numpy(d[f"{nm}_w"]).to(DEV))
        assert y.dtype == torch.float16
        assert rel_err(y.float().cpu().numpy(), d[f"{nm}_y"]) < TOL, nm


@pytest.mark.parametrize("T", [1, 32])
def test_moe_block_with_shared_expert(cbs, T):
    seed = 11
    shared = synth.synth_expert(99, 0)
    pool = resident_pool(seed, 256, extra=shared)
    ex = moe.PackedMoEExpertUniversal(pool, cb16_dev(cbs), DEV, shared=True)
    g = (0.05 * np.random.default_rng(2).standard_normal(2048)).astype(np.float32)
    blk = moe.MoEBlock(ex, shared_gate=torch.from_numpy(g).to(DEV))
    logits = np.random.default_rng(3 + T).standard_normal((T, 256)).astype(np.float32)
    h = np.random.default_rng(4 + T).standard_normal((T, 2048)).astype(np.float16)
    y = blk(torch.from_numpy(h).to(DEV), torch.from_numpy(logits).to(DEV)).float().cpu().numpy()
    ids, w = O.router_ref(logits, 8)
    sw = 1 / (1 + np.exp(-(h.astype(np.float64) @ g.astype(np.float64))))
    ref = O.moe_layer_ref(h, ids, w, lambda e: synth.synth_expert(seed, e), cbs["16"], ROT2048, ROT512,
                          shared=shared, shared_w=sw)
    assert rel_err(y, ref) < TOL


def test_moe_layer_matches_reference_golden(cbs):
    """vq2_moe_layer (router + experts in one call) on the golden logits reproduces the reference's
    own routed-expert outputs (no shared expert)."""
    d = golden("moe.npz")
    pool = resident_pool(int(d["t1_seed"]), 256)
    ex = moe.PackedMoEExpertUniversal(pool, cb16_dev(cbs), DEV)
    for nm in ("t1", "t4"):
        y = moe.moe_layer(torch.from_numpy(d[f"{nm}_h"]).to(DEV), torch.from_numpy(d[f"{nm}_logits"]).to(DEV),
                          pool, ex.cb16, ex.rot_2048, ex.rot_512, 8)
        assert rel_err(y.float().cpu().numpy(), d[f"{nm}_y"]) < TOL, nm


@pytest.mark.parametrize("T", [1, 7, 32])
def test_moe_layer_equals_route_plus_expert_ffn(cbs, T):
    """The one-call layer (RHT in the router kernel, combine in the down GEMV's epilogue) agrees
    with route + expert_ffn (RHT in the gate_up prologue, separate combine kernel) to fp32
    rounding, with and without the shared expert."""
    shared = synth.synth_expert(98, 0)
    pool = resident_pool(12, 256, extra=shared)
    ex = moe.PackedMoEExpertUniversal(pool, cb16_dev(cbs), DEV, shared=True)
    g = torch.from_numpy((0.05 * np.random.default_rng(5).standard_normal(2048)).astype(np.float32)).to(DEV)
    h = torch.from_numpy(np.random.default_rng(6 + T).standard_normal((T, 2048)).astype(np.float16)).to(DEV)
    lg = torch.randn(T, 256, device=DEV)
    for gate in (None, g):
        y = moe.moe_layer(h, lg, pool, ex.cb16, ex.rot_2048, ex.rot_512, 8, shared_gate=gate, hi=256,
                          out_dtype=torch.float32)
        if gate is None:
            ids, w = moe.route(lg, 8)
            k = 8
        else:
            ids, w, sw = moe.route(lg, 8, h, gate)
            ids = torch.cat([ids, torch.full((T, 1), 256, dtype=torch.int32, device=DEV)], 1)
            w = torch.cat([w, sw[:, None]], 1)
            k = 9
        ref = moe.expert_ffn(h, ids.reshape(-1).contiguous(), w, pool, ex.cb16, ex.rot_2048, ex.rot_512, k,
                             out_dtype=torch.float32)
        assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("K,shared", [(8, True), (8, False), (4, True)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_moe_layer_one_token_path_bitwise(cbs, monkeypatch, K, shared, out_dtype):
    """A one-token layer runs in two launches that each route the token themselves
    (moe_decode.cu); routing keys, weights, shared gate, staging, FMA, shuffle and combine order
    are those of the router kernel + GEMVs, so the outputs are bit-identical to that path
    (VQ2_MOE_T1=0), for the whole layer and for a rank's expert slice."""
    sh = synth.synth_expert(96, 0)
    full = resident_pool(14, 256, extra=sh)
    ex = moe.PackedMoEExpertUniversal(full, cb16_dev(cbs), DEV, shared=True)
    g = torch.from_numpy((0.05 * np.random.default_rng(11).standard_normal(2048)).astype(np.float32)).to(DEV)
    h = torch.from_numpy(np.random.default_rng(12).standard_normal((1, 2048)).astype(np.float16)).to(DEV)
    slice_pool = moe.ExpertRecordPool(64 + 1, DEV)
    slice_pool.raw[:64].copy_(full.raw[64:128])
    slice_pool.raw[64].copy_(full.raw[256])
    for trial in range(3):
        lg = torch.randn(1, 256, device=DEV)
        lg[0, 64:128] += 1.5 * trial  # from a few of the slice's experts to most of them
        cases = [dict(pool=full, hi=256), dict(pool=slice_pool, lo=64, hi=128, rank=1, world=4)]
        for kw in cases:
            pool = kw.pop("pool")
            outs = []
            for env in ("1", "0"):
                monkeypatch.setenv("VQ2_MOE_T1", env)
                outs.append(moe.moe_layer(h, lg, pool, ex.cb16, ex.rot_2048, ex.rot_512, K,
                                          shared_gate=g if shared else None, out_dtype=out_dtype, **kw))
            assert torch.equal(outs[0], outs[1]), (trial, kw)
            assert torch.isfinite(outs[0].float()).all()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("T", [1, 5, 32])
def test_moe_layer_rank_partials_sum_to_full_layer(cbs, world, T):
    """Expert parallelism emulated on one GPU: each rank's layer over its expert slice (+ its
    share of the shared expert's tokens) gives an fp32 partial; tokens with nothing local get zero
    rows; the partials sum to the single-GPU layer and to the fp64 oracle."""
    shared = synth.synth_expert(97, 0)
    full = resident_pool(13, 256, extra=shared)
    ex = moe.PackedMoEExpertUniversal(full, cb16_dev(cbs), DEV, shared=True)
    g_np = (0.05 * np.random.default_rng(7).standard_normal(2048)).astype(np.float32)
    g = torch.from_numpy(g_np).to(DEV)
    h_np = np.random.default_rng(8 + T).standard_normal((T, 2048)).astype(np.float16)
    lg_np = np.random.default_rng(9 + T).standard_normal((T, 256)).astype(np.float32)
    h, lg = torch.from_numpy(h_np).to(DEV), torch.from_numpy(lg_np).to(DEV)
    whole = moe.moe_layer(h, lg, full, ex.cb16, ex.rot_2048, ex.rot_512, 8, shared_gate=g, hi=256,
                          out_dtype=torch.float32)
    parts = []
    for rank in range(world):
        lo, hi = rank * 256 // world, (rank + 1) * 256 // world
        pool = moe.ExpertRecordPool(hi - lo + 1, DEV)
        pool.raw[: hi - lo].copy_(full.raw[lo:hi])
        pool.raw[hi - lo].copy_(full.raw[256])
        parts.append(moe.moe_layer(h, lg, pool, ex.cb16, ex.rot_2048, ex.rot_512, 8, shared_gate=g, lo=lo, hi=hi,
                                   rank=rank, world=world, out_dtype=torch.float32))
    total = torch.stack(parts).sum(0)
    assert rel_err(total.cpu().numpy(), whole.cpu().numpy()) < 1e-5
    ids, w = O.router_ref(lg_np, 8)
    if T == 1:  # a rank holding none of the token's experts and not its shared problem returns zeros
        for rank in range(world):
            lo, hi = rank * 256 // world, (rank + 1) * 256 // world
            if rank != 0 and not any(lo <= e < hi for e in ids[0]):
                assert not parts[rank].abs().any()
    sw = 1 / (1 + np.exp(-(h_np.astype(np.float64) @ g_np.astype(np.float64))))
    ref = O.moe_layer_ref(h_np, ids, w, lambda e: synth.synth_expert(13, e), cbs["16"], ROT2048, ROT512,
                          shared=shared, shared_w=sw)
    assert rel_err(total.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("mode", ["image_pinned", "offset", "mmap"])
@pytest.mark.parametrize("T,cap", [(1, 12), (3, 10), (4, 8)])
def test_paged_experts_outputs_and_lru(cbs, tmp_path, mode, T, cap):
    layers, E, seed = 2, 24, 5
    if mode == "image_pinned":
        img, _ = container.synthetic_vq2m_image(layers, E, seed=seed)
        store = paged_runtime.PagedModelStore.from_image(torch.from_numpy(img).pin_memory(), device=DEV)
    else:
        path = str(tmp_path / "p.vq2m")
        container.write_synthetic_vq2m(path, layers, E, seed=seed)
        store = paged_runtime.PagedModelStore(path, use_mmap=(mode == "mmap"), device=DEV)
    cb = cb16_dev(cbs)
    mods = [paged_runtime.PagedMoEExpert(ln, store, cb, capacity=cap, device=DEV) for ln in range(layers)]
    oracles = [O.LRUSlotOracle(cap) for _ in range(layers)]
    rng = np.random.default_rng(T * 10 + cap)
    for step in range(6):
        h = rng.standard_normal((T, 2048)).astype(np.float16)
        for ln in range(layers):
            ids = np.stack([rng.choice(E, 8, replace=False) for _ in range(T)])
            w = rng.random((T, 8)).astype(np.float32)
            w /= w.sum(1, keepdims=True)
            y = mods[ln](torch.from_numpy(h).to(DEV), torch.from_numpy(ids), torch.from_numpy(w))
            for e in ids.reshape(-1):
                oracles[ln].get_slot(int(e))
            assert (mods[ln].hits, mods[ln].misses) == (oracles[ln].hits, oracles[ln].misses)
            assert mods[ln].expert_to_slot == oracles[ln].expert_to_slot
            expert = lambda e, ln=ln: tuple(t.numpy() for t in store.get_expert_weights(ln, e))
            ref = O.moe_layer_ref(h, ids, w, expert, cbs["16"], ROT2048, ROT512)
            assert rel_err(y.float().cpu().numpy(), ref) < TOL, (mode, step, ln)
            h = y.cpu().numpy().astype(np.float16)
    assert store.bytes_paged == sum(m.misses for m in mods) * store.expert_bytes
    store.close()


@pytest.mark.parametrize("T", [1, 3, 9])
def test_native_paged_step_matches_python_path_bitwise(cbs, tmp_path, T):
    """A pinned-image store runs the native step (vq2_paged_moe_step: one call per step; for
    T * 8 <= 64 the single-launch fused FFN kernel), an offset store the Python copy path with the
    four-kernel FFN; per token both do the same arithmetic, so outputs, slot contents and LRU
    sequences agree bit for bit (T = 9 exercises the native step's id upload path)."""
    layers, E, cap = 2, 40, 12
    path = str(tmp_path / "p.vq2m")
    container.write_synthetic_vq2m(path, layers, E, seed=9)
    native = paged_runtime.PagedModelStore.from_image(torch.from_numpy(np.fromfile(path, np.uint8)).pin_memory(),
                                                      device=DEV)
    python = paged_runtime.PagedModelStore(path, device=DEV)
    cb = cb16_dev(cbs)
    mods = {nm: [paged_runtime.PagedMoEExpert(ln, st, cb, capacity=cap, device=DEV) for ln in range(layers)]
            for nm, st in (("native", native), ("python", python))}
    assert all(m.native for m in mods["native"]) and not any(m.native for m in mods["python"])
    rng = np.random.default_rng(T)
    for step in range(4):
        h = torch.from_numpy(rng.standard_normal((T, 2048)).astype(np.float16)).to(DEV)
        for ln in range(layers):
            ids = torch.from_numpy(np.stack([rng.choice(E, 8, replace=False) for _ in range(T)]))
            w = torch.from_numpy(rng.random((T, 8)).astype(np.float32)).to(DEV)
            y = {nm: ms[ln](h, ids, w) for nm, ms in mods.items()}
            assert torch.equal(y["native"], y["python"]), (T, step, ln)
            a, b = mods["native"][ln], mods["python"][ln]
            assert (a.hits, a.misses, a.expert_to_slot) == (b.hits, b.misses, b.expert_to_slot)
            for slot in a.expert_to_slot.values():
                assert torch.equal(a.pool.raw[slot], b.pool.raw[slot])
            h = y["native"]
    assert native.bytes_paged == python.bytes_paged
    native.close()
    python.close()


def test_expert_ffn_abi_workspace_and_errors(cbs):
    """vq2_moe_expert_ffn through the C-ABI: workspace sizing, too-small workspace refused,
    out-of-range ids contribute zero."""
    from compressai_b200 import _lib, vq
    lib = _lib.load()
    # 1 KB of fused-kernel counters + fp32 gate_up and down outputs + the compaction lists
    assert lib.vq2_moe_expert_ffn_workspace(1, 8, 1024, 2048) == 1024 + 8 * 1024 * 4 + 8 * 2048 * 4 + 256
    assert lib.vq2_moe_expert_ffn_workspace(0, 8, 1024, 2048) == -1
    seed, E = 21, 6
    pool = resident_pool(seed, E)
    cb = cb16_dev(cbs)
    r_in, r_mid = vq.get_rot("moe_expert_2048", 2048, DEV), vq.get_rot("moe_expert_512", 512, DEV)
    T, K = 2, 3
    h = torch.randn(T, 2048, device=DEV).half()
    ids = torch.tensor([0, 5, 99, 2, -1, 3], dtype=torch.int32, device=DEV)
    w = torch.rand(T, K, device=DEV)
    out = torch.empty(T, 2048, device=DEV, dtype=torch.float32)
    ws = torch.empty(lib.vq2_moe_expert_ffn_workspace(T, K, 1024, 2048), dtype=torch.uint8, device=DEV)
    args = lambda nbytes: (_lib.ptr(h), _lib.VQ2_F16, T, K, _lib.ptr(ids), _lib.ptr(w), _lib.ptr(pool.raw), E, 1024,
                           256, 2048, 64, _lib.ptr(cb), _lib.VQ2_F16, _lib.ptr(r_in.perm), _lib.ptr(r_in.sign), 2048,
                           float(r_in.scale), _lib.ptr(r_mid.perm), _lib.ptr(r_mid.sign), 512, float(r_mid.scale),
                           _lib.ptr(ws), nbytes, _lib.ptr(out), _lib.VQ2_F32, _lib.stream_ptr(DEV))
    assert lib.vq2_moe_expert_ffn(*args(ws.numel() - 1)) == _lib.VQ2_ERR_ARG
    _lib.call("vq2_moe_expert_ffn", *args(ws.numel()))
    ids_np = ids.cpu().numpy().reshape(T, K)
    wn = w.cpu().numpy()
    zero = tuple(np.zeros_like(a) for a in synth.synth_expert(seed, 0))
    expert = lambda e: synth.synth_expert(seed, e) if 0 <= e < E else zero
    ref = O.moe_layer_ref(h.cpu().numpy(), ids_np, wn, expert, cbs["16"], ROT2048, ROT512)
    assert rel_err(out.cpu().numpy(), ref) < 2e-5
