"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

This script is test infrastructure. It is run by hand in a container that has the reference
checkout (read-only) mounted; the GPU box never runs it. It copies the reference's ``vq2``
package into a temporary directory (``vq2/common.py:18`` creates a directory next to the
package at import time, which fails on a read-only mount), imports it on the CPU, and
records the reference's own outputs on seeded inputs:

* ``codebooks.npz``  -- universal codebooks fit by ``vq.train_codebooks`` (``vq2/vq.py:170-191``)
  on N(0,1) samples (seed 1), keys "16" [65536,8] and "16_8" [256,8], stored fp16.
* ``rot.npz``        -- perm/sign of ``vq.Rot`` (``vq2/vq.py:47-57``) for every tag used, plus
  ``Rot.fwd`` outputs in fp32 on seeded inputs.
* ``gemv.npz``       -- matrices quantized by ``quantize_35b.fast_quantize_matrix``
  (``vq2/quantize_35b.py:30-104``) and the reference dequantize-then-matmul output
  (``QMat.dequant``, ``vq2/vq.py:283-292``) computed in fp64.
* ``moe.npz``        -- one MoE layer through the reference's CPU expert path
  (``vq2/paged_runtime.py:19-41`` gate_up/down, ``Rot.fwd`` for 2048 and 512) with routing by
  the installed transformers ``Qwen3_5MoeTopKRouter`` math; expert weights are regenerated
  from seeds by ``compressai_b200.synth.synth_expert`` so only outputs are stored.
* ``lru.npz``        -- hit/slot sequences of the reference ``PagedMoEExpert._get_slot``
  (``vq2/paged_runtime.py:415-437``) replayed on a seeded Zipf routing trace.
* ``vq2m.npz``       -- hashes of the tensors that the reference ``PagedModelStore``
  (``vq2/paged_runtime.py:49-173``) parses out of a small ``.vq2m`` written by this repo's writer.
* ``lru_cache.npz``  -- hit flags, store loads and final recency order of the reference
  ``LRUExpertCache`` (``vq2/paged_runtime.py:287-313``) on seeded (layer, expert) sequences.
* ``fixed.npz``      -- the reference ``pack_fixed`` / ``unpack_fixed`` (``vq2/export.py:39-70``)
  on seeded symbols (4/8/12/16 bits, odd and even counts), and a small fixed-width ``.vq2``
  container (``vq2_small.pt``, built in the reference's stream layout) decoded by the reference
  ``read_container`` (``vq2/runtime.py:155-193``).

Usage:  python tests/golden/make_golden.py [stage ...]
"""
import hashlib
import os
import shutil
import sys
import tempfile
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_SRC = os.environ.get("VQ2_REFERENCE_DIR", "/root/reference")
sys.path.insert(0, REPO)

from oracle import vq2_oracle as O  # noqa: E402,F401
from compressai_b200 import synth  # noqa: E402

_REF = None


def ref():
    """Import the reference vq2 package from a writable temporary copy (CPU only)."""
    global _REF
    if _REF is None:
        tmp = tempfile.mkdtemp(prefix="vq2ref_")
        shutil.copytree(os.path.join(REF_SRC, "vq2"), os.path.join(tmp, "vq2"))
        sys.path.insert(0, tmp)
        import vq2.vq as vq
        import vq2.quantize_35b as q35
        import vq2.paged_runtime as pr
        import vq2.export as ex
        _REF = dict(vq=vq, q35=q35, pr=pr, ex=ex, tmp=tmp)
    return _REF


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def stage_codebooks():
    out = os.path.join(HERE, "codebooks.npz")
    if os.path.exists(out):
        print("codebooks.npz exists; skipping")
        return
    vq = ref()["vq"]
    g = torch.Generator().manual_seed(1)
    S = torch.randn(1 << 18, 8, generator=g)
    t0 = time.time()
    cbs = vq.train_codebooks(S, [(16,), (16, 8)], iters=15)
    print(f"train_codebooks: {time.time() - t0:.0f}s")
    c16 = cbs.cb["16"].float().numpy()
    c168 = cbs.cb["16_8"].float().numpy()
    # Only the fp16 rounding is kept: containers store fp16 codebooks (vq2/export.py:118) and the
    # reference pipeline quantizes and dequantizes with fp16-rounded values
    # (pipeline.load_codebooks, vq2/pipeline.py:75-77).
    np.savez(out, cb16=c16.astype(np.float16), cb16_8=c168.astype(np.float16))


def load_cbs():
    d = np.load(os.path.join(HERE, "codebooks.npz"))
    return {"16": d["cb16"], "16_8": d["cb16_8"]}


def ref_codebooks():
    """Reference ``Codebooks`` object holding fp16-rounded values as fp32, as
    ``pipeline.load_codebooks`` (vq2/pipeline.py:75-77) returns them."""
    vq = ref()["vq"]
    d = np.load(os.path.join(HERE, "codebooks.npz"))
    cb = {"16": torch.from_numpy(d["cb16"].astype(np.float32)),
          "16_8": torch.from_numpy(d["cb16_8"].astype(np.float32))}
    return vq.Codebooks(cb)


ROT_TAGS = [("dense_q", 2048), ("attn", 2048), ("mlp_down", 6144), ("mlp_up", 2048),
            ("moe_expert_2048", 2048), ("moe_expert_512", 512), ("lm_head", 2048),
            ("small_1024", 1024)]


def stage_rot():
    vq = ref()["vq"]
    res = {}
    for tag, n in ROT_TAGS:
        r = vq.Rot(n, vq.tag_seed(tag), "cpu")
        key = f"{tag}_{n}"
        res[f"perm_{key}"] = r.perm.numpy().astype(np.int32)
        res[f"sign_{key}"] = r.sign.float().numpy().astype(np.int8)
        res[f"hb_{key}"] = np.int32(r.hb)
        g = torch.Generator().manual_seed(11)
        x = torch.randn(3, n, generator=g)
        res[f"x_{key}"] = x.numpy()
        res[f"fwd_{key}"] = r.fwd(x).numpy()
        res[f"inv_{key}"] = r.inv(x).numpy()
        res[f"seed_{key}"] = np.int64(vq.tag_seed(tag))
    np.savez(os.path.join(HERE, "rot.npz"), **res)


def _quantize(W, tag, cfg):
    R = ref()
    R["q35"].init_cb_cache(ref_codebooks())
    return R["q35"].fast_quantize_matrix(W, tag=tag, cfg=cfg, dev="cpu")


def _ref_dequant_y(q, x):
    """y = x . W^T with W from the reference QMat.dequant (fp32), accumulated in fp64."""
    vq = ref()["vq"]
    qm = vq.QMat(tuple(q["shape"]), tuple(q["cfg"]), q["tag"], q["idx"], q["scale"])
    W = qm.dequant(ref_codebooks(), "cpu", torch.float32).double()
    return (x.double() @ W.T).numpy()


GEMV_CASES = [
    # name, out, n, cfg, tag, M, seed_w, seed_x
    ("cfg1", 2048, 2048, (16,), "dense_q", 1, 0, 2),
    ("b3_m4", 256, 2048, (16, 8), "attn", 4, 5, 6),
    ("n6144", 128, 6144, (16,), "mlp_down", 2, 7, 8),
    ("b3_n6144", 64, 6144, (16, 8), "mlp_down", 3, 9, 10),
    ("n512", 192, 512, (16,), "moe_expert_512", 5, 12, 13),
    ("ragged", 77, 1024, (16,), "small_1024", 1, 14, 15),
]


def stage_gemv():
    res = {}
    for name, out, n, cfg, tag, M, sw, sx in GEMV_CASES:
        t0 = time.time()
        W = 0.02 * torch.randn(out, n, generator=torch.Generator().manual_seed(sw))
        q = _quantize(W, tag, cfg)
        x = torch.randn(M, n, generator=torch.Generator().manual_seed(sx)).half()
        y = _ref_dequant_y(q, x.float())
        res[f"{name}_idx0"] = q["idx"][0].numpy()
        if len(cfg) > 1:
            res[f"{name}_idx1"] = q["idx"][1].numpy()
        res[f"{name}_scale"] = q["scale"].numpy()
        res[f"{name}_x"] = x.numpy()
        res[f"{name}_y"] = y
        res[f"{name}_meta"] = np.array([out, n, len(cfg), M], dtype=np.int64)
        res[f"{name}_tag"] = np.array(tag)
        print(f"gemv case {name}: {time.time() - t0:.1f}s")
    np.savez_compressed(os.path.join(HERE, "gemv.npz"), **res)


MOE_CASES = [
    # name, T, logits seed, hidden seed, expert-data seed
    ("t1", 1, 3, 4, 100),
    ("t4", 4, 31, 41, 100),
]


def stage_moe():
    R = ref()
    vq, pr = R["vq"], R["pr"]
    cb16 = torch.from_numpy(load_cbs()["16"].astype(np.float32))
    rot2048 = vq.Rot(2048, vq.tag_seed("moe_expert_2048"), "cpu")
    rot512 = vq.Rot(512, vq.tag_seed("moe_expert_512"), "cpu")
    res = {}
    for name, T, sl, sh, se in MOE_CASES:
        logits = torch.randn(T, 256, generator=torch.Generator().manual_seed(sl))
        h = torch.randn(T, 2048, generator=torch.Generator().manual_seed(sh)).half()
        # routing: installed transformers Qwen3_5MoeTopKRouter.forward math on given logits
        probs = torch.nn.functional.softmax(logits, dtype=torch.float, dim=-1)
        top_v, top_i = torch.topk(probs, 8, dim=-1)
        top_v /= top_v.sum(dim=-1, keepdim=True)
        y = torch.zeros(T, 2048, dtype=torch.float64)
        for t in range(T):
            ids = top_i[t].tolist()
            gu_idx = torch.stack([torch.from_numpy(synth.synth_expert(se, e)[0]) for e in ids])
            gu_sc = torch.stack([torch.from_numpy(synth.synth_expert(se, e)[1].astype(np.float32)) for e in ids])
            dn_idx = torch.stack([torch.from_numpy(synth.synth_expert(se, e)[2]) for e in ids])
            dn_sc = torch.stack([torch.from_numpy(synth.synth_expert(se, e)[3].astype(np.float32)) for e in ids])
            slots = torch.arange(8, dtype=torch.int32)
            xr = rot2048.fwd(h[t].float())
            y_gu = torch.empty(8, 1024, dtype=torch.float32)
            pr.vq_moe_parallel_gate_up_cpu(xr, slots, gu_idx, cb16, gu_sc, y_gu, OUT=1024, NG=256, rs=1.0)
            act = torch.nn.functional.silu(y_gu[:, :512]) * y_gu[:, 512:]
            act_r = rot512.fwd(act)
            y_dn = torch.empty(8, 2048, dtype=torch.float32)
            pr.vq_moe_parallel_down_cpu(act_r, slots, dn_idx, cb16, dn_sc, y_dn, OUT=2048, NG=64, rs=1.0)
            y[t] = (y_dn.double() * top_v[t].double()[:, None]).sum(0)
        res[f"{name}_logits"] = logits.numpy()
        res[f"{name}_h"] = h.numpy()
        res[f"{name}_ids"] = top_i.numpy().astype(np.int64)
        res[f"{name}_w"] = top_v.numpy()
        res[f"{name}_y"] = y.numpy()
        res[f"{name}_seed"] = np.int64(se)
        print(f"moe case {name} done")
    np.savez_compressed(os.path.join(HERE, "moe.npz"), **res)


class _StubStore:
    """Stands in for PagedModelStore: records loads instead of copying bytes."""

    def __init__(self):
        self.meta = {}
        self.num_experts = 256
        self.loads = []

    def load_expert_into_slot(self, layer_idx, expert_id, slot, *a, **k):
        self.loads.append((layer_idx, expert_id, slot))


LRU_CASES = [
    # name, steps, layers, capacity, trace seed
    ("cap39", 512, 40, 39, 0),
    ("cap4", 64, 3, 4, 1),
    ("cap8", 128, 2, 8, 2),
]


def stage_lru():
    pr = ref()["pr"]
    cb16 = torch.zeros(65536, 8)
    res = {}
    for name, steps, layers, cap, seed in LRU_CASES:
        trace = synth.zipf_trace(steps, layers, seed=seed)
        slots = np.zeros(trace.shape, dtype=np.int16)
        hits = np.zeros(trace.shape, dtype=np.uint8)
        counters = np.zeros((layers, 3), dtype=np.int64)
        for ln in range(layers):
            st = _StubStore()
            m = pr.PagedMoEExpert(ln, st, cb16, capacity=cap, device="cpu")
            for s in range(steps):
                for k in range(trace.shape[2]):
                    h0 = m.hits
                    slots[s, ln, k] = m._get_slot(int(trace[s, ln, k]))
                    hits[s, ln, k] = m.hits - h0
            counters[ln] = (m.hits, m.misses, len(m.activated_experts_set))
            del m
        res[f"{name}_trace"] = trace
        res[f"{name}_slots"] = slots
        res[f"{name}_hits"] = hits
        res[f"{name}_counters"] = counters
        res[f"{name}_meta"] = np.array([steps, layers, cap, seed], dtype=np.int64)
        print(f"lru case {name}: hit rate {hits.mean():.4f}")
    np.savez_compressed(os.path.join(HERE, "lru.npz"), **res)


def stage_vq2m():
    """Write a small .vq2m with this repo's writer and parse it with the reference reader."""
    from compressai_b200 import container
    pr = ref()["pr"]
    d = tempfile.mkdtemp(prefix="vq2m_")
    path = os.path.join(d, "small.vq2m")
    dims = dict(gu_rows=16, gu_cols=8, dn_rows=32, dn_cols=2)
    container.write_synthetic_vq2m(path, num_layers=2, num_experts=5, seed=7, **dims)
    res = {"file_sha": np.array(hashlib.sha256(open(path, "rb").read()).hexdigest())}
    for use_mmap in (False, True):
        st = pr.PagedModelStore(path, use_mmap=use_mmap, device="cpu")
        for ln in range(2):
            for e in range(5):
                gui, gus, dni, dns = st.get_expert_weights(ln, e, device="cpu")
                key = f"m{int(use_mmap)}_{ln}_{e}"
                res[key] = np.array([sha(gui.numpy()), sha(gus.numpy()), sha(dni.numpy()), sha(dns.numpy())])
        res[f"m{int(use_mmap)}_entries"] = np.array(st.moe_offsets, dtype=np.int64)
        res[f"m{int(use_mmap)}_hdr"] = np.array([st.num_layers, st.num_experts, st.payload_start,
                                                 st.gu_rows, st.gu_cols, st.dn_rows, st.dn_cols])
        try:
            st.close()
        except AttributeError:
            # with >= 11 GB free RAM the reference reads the whole file into `bytes`
            # (vq2/paged_runtime.py:70-74) and its close() then fails on bytes.close()
            st.file.close()
    np.savez(os.path.join(HERE, "vq2m.npz"), **res)
    shutil.rmtree(d)


LRU_CACHE_CASES = [("c3", 3, 300, 0), ("c16", 16, 600, 1), ("c0", 0, 20, 2)]


class _RecordingStore:
    """Stand-in store: records every expert load and returns small tagged tensors."""

    def __init__(self):
        self.loads = []

    def get_expert_weights(self, layer_idx, expert_id, device="cpu"):
        self.loads.append((layer_idx, expert_id))
        t = torch.tensor([layer_idx, expert_id])
        return t, t + 1, t + 2, t + 3


def stage_lru_cache():
    pr = ref()["pr"]
    res = {}
    for name, cap, n, seed in LRU_CACHE_CASES:
        rng = np.random.default_rng(seed)
        keys = np.stack([rng.integers(0, 3, n), np.minimum(rng.zipf(1.3, n), 40)], 1).astype(np.int64)
        st = _RecordingStore()
        c = pr.LRUExpertCache(capacity=cap, device="cpu")
        hits = []
        for ln, e in keys:
            h0 = c.hits
            c.get(st, int(ln), int(e))
            hits.append(c.hits - h0)
        res[f"{name}_keys"] = keys
        res[f"{name}_hits"] = np.array(hits, dtype=np.uint8)
        res[f"{name}_loads"] = np.array(st.loads, dtype=np.int64).reshape(-1, 2)
        res[f"{name}_final"] = np.array(list(c.cache.keys()), dtype=np.int64).reshape(-1, 2)
        res[f"{name}_counters"] = np.array([c.hits, c.misses, cap], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "lru_cache.npz"), **res)


SMALL_VQ2 = [("model.layers.0.self_attn.q_proj", (16,), (24, 64), "attn"),
             ("model.layers.0.mlp.down_proj", (16, 8), (16, 128), "mlp_down"),
             ("model.layers.1.self_attn.q_proj", (16,), (8, 64), "attn"),
             ("model.embed_tokens", (16,), (32, 64), "embed")]


def stage_fixed():
    R = ref()
    ex = R["ex"]
    res = {}
    rng = np.random.default_rng(17)
    for bits in (4, 8, 12, 16):
        for n in (1, 2, 7, 1000, 1001):
            sym = rng.integers(0, 1 << bits, n).astype(np.int64)
            buf = ex.pack_fixed(sym, bits)
            res[f"b{bits}_n{n}_sym"] = sym
            res[f"b{bits}_n{n}_buf"] = np.asarray(buf, dtype=np.uint8)
            res[f"b{bits}_n{n}_out"] = np.asarray(ex.unpack_fixed(np.asarray(buf), bits, n), dtype=np.int64)
    # a small fixed-width container in the reference's stream layout: one stream per codebook
    # key, the owners' index arrays concatenated in name order (vq2/export.py:93-131)
    names = [nm for nm, _, _, _ in SMALL_VQ2]
    meta, idx, scales = {}, {}, {}
    for nm, cfg, shape, tag in SMALL_VQ2:
        meta[nm] = {"shape": list(shape), "cfg": list(cfg), "tag": tag}
        ng = shape[1] // 8
        idx[nm] = [rng.integers(0, 1 << 16, (shape[0], ng)).astype(np.int64)]
        if len(cfg) > 1:
            idx[nm].append(rng.integers(0, 256, (shape[0], ng)).astype(np.int64))
        scales[nm] = torch.from_numpy((0.02 * np.exp(0.1 * rng.standard_normal(shape[0]))).astype(np.float16))
    streams = {}
    for key, stage, bits in (("16", 0, 16), ("16_8", 1, 8)):
        owners = [nm for nm in names if len(meta[nm]["cfg"]) > stage]
        sym = np.concatenate([idx[nm][stage].reshape(-1) for nm in owners])
        streams[key] = {"bits": bits, "sizes": [int(idx[nm][stage].size) for nm in owners], "mode": "fixed",
                        "fixed": torch.from_numpy(np.asarray(ex.pack_fixed(sym, bits)))}
    # placeholder codebooks (index decoding never reads them; full-size ones would bloat the file)
    cbs = {"16": torch.zeros(4, 8), "16_8": torch.zeros(4, 8)}
    C = {"names": names, "meta": meta, "streams": streams, "scales": scales, "codebooks": cbs,
         "codebooks_embed": cbs, "dense": {}}
    path = os.path.join(HERE, "vq2_small.pt")
    torch.save(C, path)
    import vq2.runtime as rt
    D = rt.read_container(path)
    for nm in names:
        for i, t in enumerate(D["idx"][nm]):
            res[f"ctr_{nm}_{i}"] = t.numpy()
    np.savez_compressed(os.path.join(HERE, "fixed.npz"), **res)


STAGES = dict(codebooks=stage_codebooks, rot=stage_rot, gemv=stage_gemv, moe=stage_moe,
              lru=stage_lru, vq2m=stage_vq2m, lru_cache=stage_lru_cache, fixed=stage_fixed)

if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count())
    names = sys.argv[1:] or list(STAGES)
    for nm in names:
        t0 = time.time()
        STAGES[nm]()
        print(f"[stage {nm}] {time.time() - t0:.1f}s", flush=True)
