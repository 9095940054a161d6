"""Host-side paging logic (CPU): the .vq2m container against the reference reader's output,
corrupt-file handling, and the product LRU against the reference _get_slot sequences."""
import hashlib
import os

import numpy as np
import pytest
import torch

from compressai_b200 import container, paged_runtime, synth
from tests.conftest import golden

DIMS = dict(gu_rows=16, gu_cols=8, dn_rows=32, dn_cols=2)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture()
def small_vq2m(tmp_path):
    path = str(tmp_path / "small.vq2m")
    container.write_synthetic_vq2m(path, num_layers=2, num_experts=5, seed=7, **DIMS)
    return path


def test_writer_matches_golden_file(small_vq2m):
    d = golden("vq2m.npz")
    assert hashlib.sha256(open(small_vq2m, "rb").read()).hexdigest() == str(d["file_sha"])


@pytest.mark.parametrize("mode", ["offset", "mmap", "image"])
def test_reader_matches_reference_reader(small_vq2m, mode):
    d = golden("vq2m.npz")
    if mode == "image":
        st = paged_runtime.PagedModelStore.from_image(np.fromfile(small_vq2m, dtype=np.uint8), device="cpu")
    else:
        st = paged_runtime.PagedModelStore(small_vq2m, use_mmap=(mode == "mmap"), device="cpu")
    hdr = d["m0_hdr"]
    assert (st.num_layers, st.num_experts, st.payload_start, st.gu_rows, st.gu_cols, st.dn_rows,
            st.dn_cols) == tuple(int(v) for v in hdr)
    assert np.array_equal(np.array(st.moe_offsets, dtype=np.int64), d["m0_entries"])
    for ln in range(2):
        for e in range(5):
            got = [sha(t.numpy()) for t in st.get_expert_weights(ln, e, device="cpu")]
            assert got == list(d[f"m0_{ln}_{e}"]), (ln, e)
            assert got == list(d[f"m1_{ln}_{e}"]), (ln, e)
            # and the content is the seeded expert
            ref = synth.synth_expert(7 * 1_000_003 + ln, e, **DIMS)
            for a, b in zip(st.get_expert_weights(ln, e), ref):
                assert np.array_equal(a.numpy(), b)
    st.close()


def test_corrupt_containers(tmp_path, small_vq2m):
    with pytest.raises(FileNotFoundError):
        paged_runtime.PagedModelStore(str(tmp_path / "missing.vq2m"))
    raw = bytearray(open(small_vq2m, "rb").read())
    bad = tmp_path / "bad_magic.vq2m"
    bad.write_bytes(b"XXXX" + bytes(raw[4:]))
    with pytest.raises(ValueError):
        paged_runtime.PagedModelStore(str(bad))
    trunc = tmp_path / "trunc.vq2m"
    trunc.write_bytes(bytes(raw[: len(raw) - 100]))
    with pytest.raises(ValueError):
        paged_runtime.PagedModelStore(str(trunc))
    short = tmp_path / "short.vq2m"
    short.write_bytes(bytes(raw[:40]))
    with pytest.raises(ValueError):
        paged_runtime.PagedModelStore(str(short))


def test_synthetic_image_layout():
    img, end = container.synthetic_vq2m_image(2, 3, seed=1, **DIMS)
    st = paged_runtime.PagedModelStore.from_image(img, device="cpu")
    rec = container.record_bytes(**DIMS)
    assert end == container.RESERVED_HEADER_BYTES + 6 * rec
    off, nb = st.layout.record(1, 2)
    assert nb == rec and off == container.RESERVED_HEADER_BYTES + 5 * rec
    gi, gs, di, ds = st.get_expert_weights(1, 2)
    assert gs.dtype == torch.float16 and np.all(gs.float().numpy() > 0)


def _lru_module(cap):
    img, _ = container.synthetic_vq2m_image(1, 256, seed=0, **DIMS)
    st = paged_runtime.PagedModelStore.from_image(img, device="cpu")
    return paged_runtime.PagedMoEExpert(0, st, cb16=None, capacity=cap, device="cpu")


@pytest.mark.parametrize("case", ["cap39", "cap4", "cap8"])
def test_product_lru_matches_reference_sequence(case):
    d = golden("lru.npz")
    steps, layers, cap, seed = (int(v) for v in d[f"{case}_meta"])
    trace = d[f"{case}_trace"]
    ref_slots, ref_hits, ref_cnt = d[f"{case}_slots"], d[f"{case}_hits"], d[f"{case}_counters"]
    for ln in range(min(layers, 6)):
        m = _lru_module(cap)
        got = [m._assign_slot(int(e)) for e in trace[:, ln, :].reshape(-1)]
        assert np.array_equal(np.array([g[0] for g in got]).reshape(steps, -1), ref_slots[:, ln, :])
        assert np.array_equal(np.array([g[1] for g in got]).reshape(steps, -1), ref_hits[:, ln, :].astype(bool))
        assert (m.hits, m.misses, len(m.activated_experts_set)) == tuple(ref_cnt[ln])


def test_cpu_forward_is_refused():
    m = _lru_module(4)
    with pytest.raises(ValueError, match="CUDA"):
        m(torch.zeros(1, 64), torch.zeros(1, 8, dtype=torch.long), torch.zeros(1, 8))


def test_promoted_3bit_experts_in_container(tmp_path):
    """Promoted 3 bpw experts (6-tuples) are written as idx0 || idx1 entries with
    expert_modes["L:E"] = 3 and 1,185,792-byte records at the 35B shape; the LRU of a CPU-side
    PagedMoEExpert never sees them (reference vq2/paged_runtime.py:446-460)."""
    promoted = {(0, 3), (1, 0), (1, 4)}
    fn = lambda ln, e: (synth.synth_expert_3bit(ln, e, **DIMS) if (ln, e) in promoted
                        else synth.synth_expert(ln, e, **DIMS))
    path = str(tmp_path / "m.vq2m")
    container.write_vq2m(path, 2, 6, fn, dims=DIMS)
    st = paged_runtime.PagedModelStore(path, device="cpu")
    lay = st.layout
    assert lay.meta["expert_modes"] == {f"{ln}:{e}": 3 for ln, e in promoted}
    for ln in range(2):
        for e in range(6):
            bits = 3 if (ln, e) in promoted else 2
            assert lay.expert_mode(ln, e) == bits
            assert lay.record(ln, e)[1] == container.record_bytes(bits=bits, **DIMS)
            rec = st.read_record(ln, e)
            parts = fn(ln, e)
            want = np.concatenate([np.ascontiguousarray(a).view(np.uint8).reshape(-1) for a in parts]) if bits == 2 \
                else np.concatenate([np.ascontiguousarray(a).view(np.uint8).reshape(-1) for a in
                                     (parts[0], parts[1], parts[2], parts[3], parts[4], parts[5])])
            assert np.array_equal(rec, want)
    assert container.record_bytes(bits=3) == 1185792
    m = paged_runtime.PagedMoEExpert(1, st, torch.zeros(65536, 8, dtype=torch.float16), capacity=3, device="cpu",
                                     cb8=torch.zeros(256, 8, dtype=torch.float16))
    assert m.promoted == [0, 4] and m.pool3.record_bytes == container.record_bytes(bits=3, **DIMS)
    with pytest.raises(ValueError):   # promoted experts need the residual codebook
        paged_runtime.PagedMoEExpert(1, st, torch.zeros(65536, 8, dtype=torch.float16), capacity=3, device="cpu")
    st.close()


# ---------------------------------------------------------------- fixed-width streams, .vq2 read
@pytest.mark.parametrize("bits", [4, 8, 12, 16])
@pytest.mark.parametrize("n", [1, 2, 7, 1000, 1001])
def test_unpack_fixed_matches_reference(bits, n):
    """runtime.unpack_fixed on the reference's own pack_fixed output equals the reference's
    unpack_fixed (vq2/export.py:39-70), odd counts included."""
    from compressai_b200 import runtime
    d = golden("fixed.npz")
    out = runtime.unpack_fixed(d[f"b{bits}_n{n}_buf"], bits, n)
    assert np.array_equal(out, d[f"b{bits}_n{n}_out"])
    assert np.array_equal(out, d[f"b{bits}_n{n}_sym"])


def test_read_container_matches_reference():
    """read_container / decode_indices on a fixed-width .vq2 built in the reference's stream layout
    give the reference read_container's index tensors (dtype and bits)."""
    from compressai_b200 import runtime
    from tests.conftest import GOLDEN
    d = golden("fixed.npz")
    C = runtime.read_container(os.path.join(GOLDEN, "vq2_small.pt"))
    assert C["format"] == "vq2r"
    for nm in C["names"]:
        for i, t in enumerate(C["idx"][nm]):
            ref = d[f"ctr_{nm}_{i}"]
            assert t.dtype == (torch.int16 if i == 0 else torch.uint8)
            assert t.shape == ref.shape and np.array_equal(t.numpy(), ref), (nm, i)


# ---------------------------------------------------------------- LRUExpertCache (older API)
class _RecordingStore:
    def __init__(self):
        self.loads = []

    def get_expert_weights(self, layer_idx, expert_id, device="cpu"):
        self.loads.append((layer_idx, expert_id))
        t = torch.tensor([layer_idx, expert_id])
        return t, t + 1, t + 2, t + 3


@pytest.mark.parametrize("case", ["c3", "c16", "c0"])
def test_lru_expert_cache_matches_reference(case):
    """Hit flags, store loads, counters and the final recency order equal those of the reference
    LRUExpertCache (vq2/paged_runtime.py:287-313) on the same (layer, expert) sequence."""
    d = golden("lru_cache.npz")
    hits_ref, loads_ref = d[f"{case}_hits"], d[f"{case}_loads"]
    c_hits, c_misses, cap = (int(v) for v in d[f"{case}_counters"])
    st = _RecordingStore()
    c = paged_runtime.LRUExpertCache(capacity=cap, device="cpu")
    hits = []
    for ln, e in d[f"{case}_keys"]:
        h0 = c.hits
        w = c.get(st, int(ln), int(e))
        assert int(w[0][0]) == ln and int(w[0][1]) == e
        hits.append(c.hits - h0)
    assert np.array_equal(np.array(hits, dtype=np.uint8), hits_ref)
    assert np.array_equal(np.array(st.loads, dtype=np.int64).reshape(-1, 2), loads_ref)
    assert (c.hits, c.misses) == (c_hits, c_misses)
    assert np.array_equal(np.array(list(c.cache.keys()), dtype=np.int64).reshape(-1, 2), d[f"{case}_final"])
    assert len(c) == len(d[f"{case}_final"]) <= cap
