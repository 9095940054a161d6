"""Pin the CPU oracle (oracle/vq2_oracle.py) to golden vectors produced by running the
reference implementation itself (tests/golden/make_golden.py). CPU only."""
import numpy as np

from compressai_b200 import synth
from oracle import vq2_oracle as O
from tests.conftest import golden


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def cbs():
    d = golden("codebooks.npz")
    return {"16": d["cb16"], "16_8": d["cb16_8"]}


def test_codebook_shapes():
    c = cbs()
    assert c["16"].shape == (65536, 8) and c["16"].dtype == np.float16
    assert c["16_8"].shape == (256, 8)


def test_rotation_matches_reference():
    d = golden("rot.npz")
    keys = sorted(k[5:] for k in d.files if k.startswith("perm_"))
    assert len(keys) >= 6
    for key in keys:
        tag, n = key.rsplit("_", 1)
        n = int(n)
        assert O.tag_seed(tag) == int(d[f"seed_{key}"])
        perm, sign, hb = O.rot_params(tag, n)
        assert np.array_equal(perm, d[f"perm_{key}"]), key
        assert np.array_equal(sign.astype(np.int8), d[f"sign_{key}"]), key
        assert hb == int(d[f"hb_{key}"])
        x = d[f"x_{key}"]
        assert rel(O.rht_fwd(x, perm, sign, hb), d[f"fwd_{key}"]) < 1e-5, key
        assert rel(O.rht_inv(x, perm, sign, hb), d[f"inv_{key}"]) < 1e-5, key
        # orthogonality
        assert rel(O.rht_inv(O.rht_fwd(x, perm, sign, hb), perm, sign, hb), x) < 1e-12


def test_gemv_oracle_matches_reference_dequant_matmul():
    d = golden("gemv.npz")
    c = cbs()
    names = sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_meta")})
    assert {"cfg1", "b3_m4", "n6144", "ragged"} <= set(names)
    for nm in names:
        out, n, nst, M = d[f"{nm}_meta"]
        cfg = (16,) if nst == 1 else (16, 8)
        idx = [d[f"{nm}_idx0"]] + ([d[f"{nm}_idx1"]] if nst > 1 else [])
        assert idx[0].shape == (out, n // 8) and idx[0].dtype == np.int16
        perm, sign, hb = O.rot_params(str(d[f"{nm}_tag"]), int(n))
        x = d[f"{nm}_x"].astype(np.float64)
        y = O.gemv_ref(x, idx, cfg, c, d[f"{nm}_scale"], perm, sign, hb)
        assert rel(y, d[f"{nm}_y"]) < 1e-5, nm
        if out * n <= 256 * 2048:   # literal dequantize-then-matmul on the small cases
            W = O.dequant(idx, cfg, c, d[f"{nm}_scale"], perm, sign, hb)
            assert rel(x @ W.T, d[f"{nm}_y"]) < 1e-5, nm


def test_moe_oracle_matches_reference_cpu_path():
    d = golden("moe.npz")
    c = cbs()
    rot2048 = O.rot_params("moe_expert_2048", 2048)
    rot512 = O.rot_params("moe_expert_512", 512)
    for nm in ("t1", "t4"):
        ids, w = O.router_ref(d[f"{nm}_logits"], 8)
        assert np.array_equal(ids, d[f"{nm}_ids"])
        assert np.array_equal(w, d[f"{nm}_w"])
        seed = int(d[f"{nm}_seed"])
        y = O.moe_layer_ref(d[f"{nm}_h"], ids, w, lambda e: synth.synth_expert(seed, e), c["16"], rot2048, rot512)
        assert rel(y, d[f"{nm}_y"]) < 1e-5, nm


def test_lru_oracle_matches_reference_get_slot():
    d = golden("lru.npz")
    for nm in ("cap39", "cap4", "cap8"):
        steps, layers, cap, seed = d[f"{nm}_meta"]
        trace = synth.zipf_trace(int(steps), int(layers), seed=int(seed))
        assert np.array_equal(trace, d[f"{nm}_trace"])
        ref_slots, ref_hits, ref_cnt = d[f"{nm}_slots"], d[f"{nm}_hits"], d[f"{nm}_counters"]
        for ln in range(layers):
            o = O.LRUSlotOracle(int(cap))
            got = [o.get_slot(int(e)) for e in trace[:, ln, :].reshape(-1)]
            slots = np.array([g[0] for g in got]).reshape(int(steps), -1)
            hits = np.array([g[1] for g in got]).reshape(int(steps), -1)
            assert np.array_equal(slots, ref_slots[:, ln, :]), (nm, ln)
            assert np.array_equal(hits, ref_hits[:, ln, :].astype(bool)), (nm, ln)
            assert (o.hits, o.misses, len(o.activated)) == tuple(ref_cnt[ln])
