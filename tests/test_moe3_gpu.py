"""Promoted 3 bpw experts (expert_modes == 3) on the GPU: the residual-codebook expert FFN against
the fp64 oracle, and PagedMoEExpert over a mixed container (native and Python paths) against
the oracle, with the LRU seeing only the paged (2 bpw) experts as in the reference
(vq2/paged_runtime.py:446-460)."""
import numpy as np
import pytest
import torch

from compressai_b200 import container, moe, paged_runtime, synth, vq
from oracle import vq2_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3
ROT2048 = O.rot_params("moe_expert_2048", 2048)
ROT512 = O.rot_params("moe_expert_512", 512)


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.fixture(scope="module")
def cbs():
    return synth.random_codebooks(1)


def test_expert_ffn_res_matches_oracle_with_add(cbs):
    E = 5
    pool3 = moe.Expert3Pool(E, DEV)
    ex = [synth.synth_expert_3bit(4, e) for e in range(E)]
    for e in range(E):
        pool3.set_record(e, torch.from_numpy(np.concatenate([np.ascontiguousarray(a).view(np.uint8).reshape(-1)
                                                             for a in ex[e]])))
    cb16 = torch.from_numpy(cbs["16"]).to(DEV)
    cb8 = torch.from_numpy(cbs["16_8"]).to(DEV)
    r_in, r_mid = vq.get_rot("moe_expert_2048", 2048, DEV), vq.get_rot("moe_expert_512", 512, DEV)
    rng = np.random.default_rng(1)
    T, K = 2, 3
    h = rng.standard_normal((T, 2048)).astype(np.float16)
    ids = np.array([[4, -1, 1], [0, 2, -1]], dtype=np.int32)
    w = rng.random((T, K)).astype(np.float32)
    add = rng.standard_normal((T, 2048)).astype(np.float32) * 0.1
    out = moe.expert_ffn_res(torch.from_numpy(h).to(DEV), torch.from_numpy(ids.reshape(-1)).to(DEV),
                             torch.from_numpy(w).to(DEV), pool3, cb16, cb8, r_in, r_mid, K,
                             add=torch.from_numpy(add).to(DEV), out_dtype=torch.float32).cpu().numpy()
    skip = ids < 0
    ref = O.moe_layer_ref(h, np.where(skip, 0, ids), np.where(skip, 0.0, w), lambda e: ex[e], cbs["16"], ROT2048,
                          ROT512, cb8=cbs["16_8"]) + add
    assert rel_err(out, ref) < 2e-5


@pytest.mark.parametrize("mode", ["image_pinned", "offset"])
@pytest.mark.parametrize("T", [1, 3])
def test_paged_moe_with_promoted_experts(cbs, tmp_path, mode, T):
    layers, E, cap = 2, 20, 10
    promoted = {(0, 1), (0, 7), (1, 3), (1, 12), (1, 19)}
    fn = lambda ln, e: (synth.synth_expert_3bit(ln, e) if (ln, e) in promoted else synth.synth_expert(ln, e))
    path = str(tmp_path / "m.vq2m")
    container.write_vq2m(path, layers, E, fn)
    if mode == "image_pinned":
        store = paged_runtime.PagedModelStore.from_image(torch.from_numpy(np.fromfile(path, np.uint8)).pin_memory(),
                                                         device=DEV)
    else:
        store = paged_runtime.PagedModelStore(path, device=DEV)
    cb16 = torch.from_numpy(cbs["16"]).to(DEV)
    cb8 = torch.from_numpy(cbs["16_8"]).to(DEV)
    mods = [paged_runtime.PagedMoEExpert(ln, store, cb16, capacity=cap, device=DEV, cb8=cb8) for ln in range(layers)]
    assert all(m.native == (mode == "image_pinned") for m in mods)
    oracles = [O.LRUSlotOracle(cap) for _ in range(layers)]
    rng = np.random.default_rng(T)
    for step in range(5):
        for ln in range(layers):
            h = rng.standard_normal((T, 2048)).astype(np.float16)
            ids = np.stack([rng.choice(E, 8, replace=False) for _ in range(T)])
            if step == 0:
                ids[0, :2] = [e for (l_, e) in sorted(promoted) if l_ == ln][:2]   # promoted experts appear
            w = rng.random((T, 8)).astype(np.float32)
            y = mods[ln](torch.from_numpy(h).to(DEV), torch.from_numpy(ids), torch.from_numpy(w).to(DEV))
            for e in ids.reshape(-1):
                if (ln, int(e)) not in promoted:
                    oracles[ln].get_slot(int(e))
            m, o = mods[ln], oracles[ln]
            assert (m.hits, m.misses, m.expert_to_slot) == (o.hits, o.misses, o.expert_to_slot)
            ref = O.moe_layer_ref(h, ids, w, lambda e, ln=ln: fn(ln, e), cbs["16"], ROT2048, ROT512, cb8=cbs["16_8"])
            assert rel_err(y.float().cpu().numpy(), ref) < TOL, (mode, step, ln)
    store.close()
