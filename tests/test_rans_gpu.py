"""VQ2A rANS decode on the GPU through the C-ABI: bit-exact against the encoder's input and the C
oracle (golden streams, edge sizes, a full-size expert record), malformed streams flagged in the
status word with every write kept inside the output, and the ANS-coded paged MoE path giving the
same pool contents, LRU sequence and outputs as the raw container."""
import numpy as np
import pytest
import torch

from compressai_b200 import _lib, ans, container, paged_runtime, synth
from oracle import rans as R
from tests.conftest import golden
from tests.test_rans_cpu import CASES, corruptions

pytestmark = pytest.mark.gpu
DEV = "cuda"
GUARD = 4096


def gpu_decode(enc, n, stream_bytes=None):
    """Decode through vq2_rans_decode into an output with guard bytes on both sides; returns
    (status, decoded, guards intact)."""
    src = torch.from_numpy(np.ascontiguousarray(enc)).to(DEV)
    buf = torch.full((n + 2 * GUARD,), 0xA5, dtype=torch.uint8, device=DEV)
    out = buf[GUARD:GUARD + n]
    status = ans.new_status(DEV)
    nb = src.numel() if stream_bytes is None else stream_bytes
    _lib.check(_lib.load().vq2_rans_decode(_lib.ptr(src), nb, n, _lib.ptr(out) if n else _lib.ptr(buf), n,
                                          _lib.ptr(status), _lib.stream_ptr(DEV)), "vq2_rans_decode")
    torch.cuda.synchronize()
    b = buf.cpu().numpy()
    intact = (b[:GUARD] == 0xA5).all() and (b[GUARD + n:] == 0xA5).all()
    return int(status.item()), b[GUARD:GUARD + n], intact


@pytest.mark.parametrize("case", CASES)
def test_decode_golden_streams(case):
    d = golden("rans.npz")
    x, enc = d[f"in_{case}"], d[f"enc_{case}"]
    st, dec, intact = gpu_decode(enc, x.size)
    assert st == 0 and intact and np.array_equal(dec, x)


@pytest.mark.parametrize("n", [1, 33, 8191, 8192, 8193, 4 * 8192 + 1, 1 << 20, (1 << 24) + 77])
@pytest.mark.parametrize("dist", ["uniform", "skew", "const"])
def test_decode_bit_exact(n, dist):
    rng = np.random.default_rng(n % 1000 + len(dist))
    if dist == "uniform":
        x = rng.integers(0, 256, n).astype(np.uint8)
    elif dist == "skew":
        x = np.minimum(rng.geometric(0.02, n), 255).astype(np.uint8)
    else:
        x = np.full(n, 3, np.uint8)
    enc = ans.encode(x)
    st, dec, intact = gpu_decode(enc, n)
    assert st == 0 and intact and np.array_equal(dec, x)


def test_decode_through_python_api_and_multiple_chunks_per_cta():
    x = np.minimum(np.abs(np.random.default_rng(2).normal(0, 3000, 300_000)), 65535).astype(np.uint16)
    enc = torch.from_numpy(ans.encode(x)).to(DEV)
    out, status = ans.decode(enc, x.nbytes)
    ans.check_status(status)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), x)


def test_malformed_streams_flagged_and_writes_bounded():
    x = np.minimum(np.random.default_rng(4).geometric(0.05, 20000), 255).astype(np.uint8)
    enc = R.encode(x)
    for name, s, code in corruptions(enc, x.size):
        st_o, dec_o = R.decode(s, x.size)
        st, dec, intact = gpu_decode(s, x.size)
        assert intact, name
        assert (st != 0) == (st_o != 0), (name, st, st_o)
        if code is not None:
            assert st == code, (name, st)
    # truncated streams: refused on the host when shorter than the header, else flagged
    for cut in (1040, enc.size - 16, enc.size - 300):
        if cut < 1040 + 4 * 4:
            src = torch.from_numpy(enc[:cut].copy()).to(DEV)
            out = torch.empty(x.size, dtype=torch.uint8, device=DEV)
            status = ans.new_status(DEV)
            assert _lib.load().vq2_rans_decode(_lib.ptr(src), cut, x.size, _lib.ptr(out), x.size, _lib.ptr(status),
                                               _lib.stream_ptr(DEV)) == _lib.VQ2_ERR_SHAPE
        else:
            st, _, intact = gpu_decode(enc[:cut], x.size)
            assert st != 0 and intact, cut
    with pytest.raises(ans.ANSDecodeError):
        s = enc.copy()
        s[0] ^= 1
        _, status = ans.decode(torch.from_numpy(s).to(DEV), x.size)
        ans.check_status(status)


def test_output_capacity_refused():
    enc = torch.from_numpy(R.encode(np.zeros(100, np.uint8))).to(DEV)
    out = torch.empty(99, dtype=torch.uint8, device=DEV)
    status = ans.new_status(DEV)
    assert _lib.load().vq2_rans_decode(_lib.ptr(enc), enc.numel(), 100, _lib.ptr(out), 99, _lib.ptr(status),
                                       _lib.stream_ptr(DEV)) == _lib.VQ2_ERR_SHAPE


def test_decode_segments_expands_full_size_expert_record(tmp_path):
    path = str(tmp_path / "a.vq2m")
    container.write_vq2m(path, 1, 2, lambda ln, e: synth.synth_expert_skewed(ln, e), index_coding="vq2a")
    img = np.fromfile(path, dtype=np.uint8)
    lay = container.parse_header(memoryview(img[:container.RESERVED_HEADER_BYTES]))
    status = ans.new_status(DEV)
    for e in range(2):
        off, nb = lay.record(0, e)
        src = torch.from_numpy(img[off:off + nb].copy()).to(DEV)
        dst = torch.zeros(lay.expert_bytes, dtype=torch.uint8, device=DEV)
        ans.decode_segments(src, lay.segments(0, e), dst, status)
        ans.check_status(status)
        want = np.concatenate([a.view(np.uint8).reshape(-1) for a in synth.synth_expert_skewed(0, e)])
        assert np.array_equal(dst.cpu().numpy(), want)
        assert nb < 0.85 * lay.expert_bytes


def test_decode_segments_refuses_out_of_range_plans():
    src = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    dst = torch.zeros(1024, dtype=torch.uint8, device=DEV)
    status = ans.new_status(DEV)
    for segs in ([(0, 100, 1000, 100, 1)],          # destination overflow
                 [(4000, 200, 0, 200, 1)],          # source overflow
                 [(0, 100, 0, 50, 1)],              # stored size mismatch
                 [(0, 16, 0, 100, 0)],              # ANS segment shorter than its header
                 [(0, 16, 0, 16, 2)]):              # unknown kind
        with pytest.raises(ValueError):
            ans.decode_segments(src, segs, dst, status)
    with pytest.raises(ValueError):
        ans.decode_segments(src, [(0, 16, 0, 16, 1)] * 33, dst, status)   # at most 32 segments


@pytest.mark.parametrize("mode", ["image_pinned", "offset"])
def test_paged_moe_over_ans_container_matches_raw(tmp_path, mode):
    layers, E, cap, T = 2, 20, 8, 3
    fn = lambda ln, e: synth.synth_expert_skewed(ln, e)
    paths = {c: str(tmp_path / f"{c}.vq2m") for c in ("raw", "vq2a")}
    for c, p in paths.items():
        container.write_vq2m(p, layers, E, fn, index_coding=c)

    def open_store(p):
        if mode == "image_pinned":
            return paged_runtime.PagedModelStore.from_image(torch.from_numpy(np.fromfile(p, np.uint8)).pin_memory(),
                                                            device=DEV)
        return paged_runtime.PagedModelStore(p, device=DEV)

    stores = {c: open_store(p) for c, p in paths.items()}
    assert stores["vq2a"].ans_coded and not stores["raw"].ans_coded
    cb = torch.from_numpy(synth.random_codebooks(1)["16"]).to(DEV)
    mods = {c: [paged_runtime.PagedMoEExpert(ln, st, cb, capacity=cap, device=DEV) for ln in range(layers)]
            for c, st in stores.items()}
    rng = np.random.default_rng(8)
    for step in range(5):
        h = torch.from_numpy(rng.standard_normal((T, 2048)).astype(np.float16)).to(DEV)
        for ln in range(layers):
            ids = torch.from_numpy(np.stack([rng.choice(E, 8, replace=False) for _ in range(T)]))
            w = torch.from_numpy(rng.random((T, 8)).astype(np.float32))
            y = {c: m[ln](h, ids, w) for c, m in mods.items()}
            assert torch.equal(y["raw"], y["vq2a"]), (step, ln)
            a, b = mods["raw"][ln], mods["vq2a"][ln]
            assert (a.hits, a.misses, a.expert_to_slot) == (b.hits, b.misses, b.expert_to_slot)
            for slot in a.expert_to_slot.values():   # every filled slot holds identical bytes
                assert torch.equal(a.pool.raw[slot], b.pool.raw[slot])
            h = y["raw"]
    stores["vq2a"].check_decode_status()
    assert stores["vq2a"].bytes_paged < 0.85 * stores["raw"].bytes_paged
    # the reference accessor decodes on the GPU too
    gi, gs, di, ds = stores["vq2a"].get_expert_weights(1, 7)
    want = fn(1, 7)
    assert all(np.array_equal(t.numpy(), w) for t, w in zip((gi, gs, di, ds), want))
    for st in stores.values():
        st.close()
