"""Seeded synthetic inputs for the decode path (the reference's trained weights, codebooks and
containers are not available, so every workload is drawn from fixed seeds).

Pure numpy; imported by tests, ``bench.py`` and the fixture generator. Nothing here runs on
the product's compute path.
"""
import numpy as np

# Dimensions of one routed expert of the 35B-A3B-shaped MoE (vq2/paged_runtime.py:331-355,
# vq2/pack_35b_to_vq2m.py:209-212): gate_up [1024, 2048] and down [2048, 512] at 2 bpw.
GU_ROWS, GU_COLS = 1024, 256
DN_ROWS, DN_COLS = 2048, 64
EXPERT_BYTES = GU_ROWS * GU_COLS * 2 + GU_ROWS * 2 + DN_ROWS * DN_COLS * 2 + DN_ROWS * 2  # 792,576


def synth_expert(seed, e, gu_rows=GU_ROWS, gu_cols=GU_COLS, dn_rows=DN_ROWS, dn_cols=DN_COLS):
    """Deterministic expert ``e`` of data set ``seed``: (gu_idx int16 [gu_rows, gu_cols],
    gu_scale fp16 [gu_rows], dn_idx int16 [dn_rows, dn_cols], dn_scale fp16 [dn_rows]).

    Indices are uniform over the 2^16 codebook rows; scales are positive around 0.02, the
    row RMS of a ~N(0, 0.02) weight after rotation (vq2/quantize_35b.py:47)."""
    rng = np.random.default_rng([int(seed), int(e)])
    gu_idx = rng.integers(0, 1 << 16, size=(gu_rows, gu_cols), dtype=np.uint16).view(np.int16)
    gu_sc = (0.02 * np.exp(0.1 * rng.standard_normal(gu_rows))).astype(np.float16)
    dn_idx = rng.integers(0, 1 << 16, size=(dn_rows, dn_cols), dtype=np.uint16).view(np.int16)
    dn_sc = (0.02 * np.exp(0.1 * rng.standard_normal(dn_rows))).astype(np.float16)
    return gu_idx, gu_sc, dn_idx, dn_sc


def synth_expert_3bit(seed, e, gu_rows=GU_ROWS, gu_cols=GU_COLS, dn_rows=DN_ROWS, dn_cols=DN_COLS):
    """A promoted 3 bpw expert (reference tools/build_mixed_b2_container.py:50-80): (gu_idx0 int16,
    gu_idx1 uint8, gu_scale fp16, dn_idx0 int16, dn_idx1 uint8, dn_scale fp16), seeded."""
    gi, gs, di, ds = synth_expert(seed, e, gu_rows, gu_cols, dn_rows, dn_cols)
    rng = np.random.default_rng([int(seed), int(e), 0x3B])
    return (gi, rng.integers(0, 256, size=gi.shape, dtype=np.uint8), gs, di,
            rng.integers(0, 256, size=di.shape, dtype=np.uint8), ds)


def synth_expert_skewed(seed, e, gu_rows=GU_ROWS, gu_cols=GU_COLS, dn_rows=DN_ROWS, dn_cols=DN_COLS,
                        sigma=3000.0):
    """As synth_expert, but indices |N(0, sigma)| (clipped to 65535): a codebook whose rows are
    ordered by usage, the case where ANS coding of the index bytes pays (about 0.82 of the
    stored size at sigma 3000)."""
    gu_idx, gu_sc, dn_idx, dn_sc = synth_expert(seed, e, gu_rows, gu_cols, dn_rows, dn_cols)
    rng = np.random.default_rng([int(seed), int(e), 0x5EED])
    skew = lambda shape: np.minimum(np.abs(rng.normal(0.0, sigma, shape)), 65535).astype(np.uint16).view(np.int16)
    return skew(gu_idx.shape), gu_sc, skew(dn_idx.shape), dn_sc


def zipf_trace(steps, layers, seed=0, num_experts=256, top_k=8, s=1.1):
    """Routing trace [steps, layers, top_k] (int16) with a Zipf(s) expert popularity per layer.

    Layer l ranks its experts by a permutation pi_l = rng.permutation(E) (all layers first);
    rank r has probability proportional to (r+1)^-s. Each (step, layer), in that order, draws
    top_k distinct ranks without replacement and maps them through pi_l."""
    rng = np.random.default_rng(seed)
    perms = [rng.permutation(num_experts) for _ in range(layers)]
    p = (np.arange(num_experts) + 1.0) ** -s
    p /= p.sum()
    out = np.empty((steps, layers, top_k), dtype=np.int16)
    for st in range(steps):
        for ln in range(layers):
            out[st, ln] = perms[ln][rng.choice(num_experts, top_k, replace=False, p=p)]
    return out


def random_codebooks(seed=1):
    """Codebook stand-ins for throughput runs: "16" [65536, 8] and "16_8" [256, 8] fp16 drawn
    N(0, 1) and N(0, 0.3) (values only affect numerics, not speed)."""
    rng = np.random.default_rng(seed)
    return {"16": rng.standard_normal((1 << 16, 8)).astype(np.float16),
            "16_8": (0.3 * rng.standard_normal((256, 8))).astype(np.float16)}


def random_matrix(seed, out, n, bits=(16,)):
    """Seeded random VQ matrix: list of index arrays per stage + fp16 row scales."""
    rng = np.random.default_rng(seed)
    ng = n // 8
    idx = [rng.integers(0, 1 << 16, size=(out, ng), dtype=np.uint16).view(np.int16)]
    if len(bits) > 1:
        idx.append(rng.integers(0, 256, size=(out, ng), dtype=np.uint8))
    scale = (0.02 * np.exp(0.1 * rng.standard_normal(out))).astype(np.float16)
    return idx, scale
