"""VQ2A rANS coding on the CPU: the C oracle against the golden streams and an independent
pure-Python decoder, the product host encoder (C-ABI) against the oracle byte for byte, malformed
streams rejected by the oracle, and the ANS-coded .vq2m container variant."""
import struct

import numpy as np
import pytest

from compressai_b200 import ans, container, synth
from oracle import rans as R
from tests.conftest import golden

CASES = ["empty", "one", "const", "two_symbols", "uniform_8191", "geom_8192", "nib_8193", "skew_u16"]


def py_decode(stream, n):
    """Straight restatement of the format for small streams (pure Python)."""
    b = bytes(stream)
    u32 = lambda o: struct.unpack_from("<I", b, o)[0]
    u16 = lambda o: struct.unpack_from("<H", b, o)[0]
    assert u32(0) == 0x41325156 and u32(4) == n
    nc = u32(8)
    freq = [[u16(16 + 2 * (k * 256 + s)) for s in range(256)] for k in range(2)]
    start = [np.concatenate([[0], np.cumsum(f)]).tolist() for f in freq]
    out = bytearray(n)
    for c in range(nc):
        o0 = u32(1040 + 4 * c)
        pos = o0 + 384
        cnt = min(8192, n - 8192 * c)
        for w in range(64):
            k = w & 1
            x = u32(o0 + 4 * w)
            nw = u16(o0 + 256 + 2 * w)
            words = [u16(pos + 2 * q) for q in range(nw)]
            pos += 2 * nw
            wi = 0
            for i in range(w, cnt, 64):
                slot = x & 4095
                s = next(t for t in range(256) if start[k][t] <= slot < start[k][t + 1])
                x = freq[k][s] * (x >> 12) + slot - start[k][s]
                if x < 65536:
                    x = (x << 16) | words[wi]
                    wi += 1
                out[8192 * c + i] = s
            assert x == 65536 and wi == nw
    return np.frombuffer(bytes(out), np.uint8)


def product_encode(v):
    return ans.encode(v)


@pytest.mark.parametrize("case", CASES)
def test_oracle_reproduces_golden_streams(case):
    d = golden("rans.npz")
    x, enc = d[f"in_{case}"], d[f"enc_{case}"]
    assert np.array_equal(R.encode(x), enc)
    st, dec = R.decode(enc, x.size)
    assert st == 0 and np.array_equal(dec, x)


@pytest.mark.parametrize("case", ["one", "two_symbols", "nib_8193"])
def test_python_decoder_agrees_with_golden(case):
    d = golden("rans.npz")
    x, enc = d[f"in_{case}"], d[f"enc_{case}"]
    assert np.array_equal(py_decode(enc, x.size), x)


def test_frequency_quantization_known_answers():
    d = golden("rans.npz")
    assert np.array_equal(R.quantize(d["q_counts"]), d["q_freq"])
    assert (R.quantize(np.zeros(256)) == 16).all()                       # empty context
    assert (R.quantize(np.full(256, 5)) == 16).all()                     # uniform: 1 + 15 each
    one = np.zeros(256)
    one[9] = 1000
    f = R.quantize(one)
    assert f[9] == 3841 and (np.delete(f, 9) == 1).all()
    # remainders: counts (1, 1, 1, 0...) -> 1 + 1280 each, leftover 4096 - 3843 - 253 = 0
    three = np.zeros(256)
    three[:3] = 1
    f = R.quantize(three)
    assert f[:3].tolist() == [1281, 1281, 1281] and f.sum() == 4096
    # ties broken towards the smaller symbol: counts 1 at 0..6 -> 3840/7 = 548 r 4
    seven = np.zeros(256)
    seven[:7] = 1
    f = R.quantize(seven)
    assert f.sum() == 4096 and f[:4].tolist() == [550, 550, 550, 550] and f[4:7].tolist() == [549] * 3


def numpy_quantize(counts):
    counts = np.asarray(counts, dtype=np.uint64)
    tot = int(counts.sum())
    if tot == 0:
        return np.full(256, 16, np.uint16)
    q = counts * np.uint64(3840)
    f = (1 + q // np.uint64(tot)).astype(np.int64)
    rem = (q % np.uint64(tot)).astype(np.int64)
    order = sorted(range(256), key=lambda s: (-rem[s], s))
    for s in order[:4096 - f.sum()]:
        f[s] += 1
    return f.astype(np.uint16)


def test_frequency_quantization_matches_numpy_restatement():
    rng = np.random.default_rng(11)
    for t in range(50):
        c = rng.integers(0, 10 ** rng.integers(1, 7), 256)
        c[rng.random(256) < 0.3] = 0
        assert np.array_equal(R.quantize(c), numpy_quantize(c)), t


@pytest.mark.parametrize("n", [0, 1, 31, 32, 33, 8191, 8192, 8193, 16384 + 5, 100_003])
@pytest.mark.parametrize("dist", ["uniform", "skew", "const"])
def test_product_encoder_matches_oracle_bytes(n, dist):
    rng = np.random.default_rng(n + len(dist))
    if dist == "uniform":
        x = rng.integers(0, 256, n).astype(np.uint8)
    elif dist == "skew":
        x = np.minimum(rng.geometric(0.03, n), 255).astype(np.uint8)
    else:
        x = np.full(n, 200, np.uint8)
    enc = product_encode(x)
    assert np.array_equal(enc, R.encode(x))
    assert enc.size <= ans.bound(n) and enc.size % 16 == 0
    st, dec = R.decode(enc, n)
    assert st == 0 and np.array_equal(dec, x)


def test_product_encoder_views_any_dtype_as_bytes():
    idx = np.random.default_rng(1).integers(0, 65536, (64, 32), dtype=np.uint16).view(np.int16)
    assert np.array_equal(ans.encode(idx), R.encode(idx.view(np.uint8).reshape(-1)))


def test_product_encoder_rejects_small_capacity():
    import ctypes
    from compressai_b200 import _lib
    lib = _lib.load()
    x = np.arange(1000, dtype=np.uint8)
    out = np.zeros(64, np.uint8)
    got = ctypes.c_int64(0)
    assert lib.vq2_rans_encode(x.ctypes.data, x.size, out.ctypes.data, out.size, ctypes.byref(got)) == _lib.VQ2_ERR_ARG
    assert lib.vq2_rans_encode(x.ctypes.data, -1, out.ctypes.data, out.size, ctypes.byref(got)) == _lib.VQ2_ERR_SHAPE
    assert lib.vq2_rans_bound(-5) == -1


def corruptions(enc, n):
    """(name, stream, expected oracle status) for single planted faults in a valid stream."""
    out = []

    def mut(name, fn, code):
        s = enc.copy()
        fn(s)
        out.append((name, s, code))

    mut("magic", lambda s: s.__setitem__(0, s[0] ^ 1), 1)
    mut("count", lambda s: s[8:12].view(np.uint32).__setitem__(0, 99), 2)
    mut("freq_zero", lambda s: s[16:18].view(np.uint16).__setitem__(0, 0), 3)
    mut("freq_sum", lambda s: s[20:22].view(np.uint16).__setitem__(0, s[20:22].view(np.uint16)[0] + 1), 3)
    mut("chunk_off", lambda s: s[1040 + 4:1044 + 4].view(np.uint32).__setitem__(0, 1 << 30), 4)
    o0 = int(enc[1040:1044].view(np.uint32)[0])
    mut("word_count", lambda s: s[o0 + 256:o0 + 258].view(np.uint16).__setitem__(0, 0xFFFF), 5)
    mut("word_total", lambda s: s[o0 + 258:o0 + 260].view(np.uint16).__setitem__(0, 120), 5)
    mut("chunk_in_header", lambda s: s[1040:1044].view(np.uint32).__setitem__(0, 16), 4)
    mut("state", lambda s: s[o0:o0 + 4].view(np.uint32).__setitem__(0, 12345), None)
    mut("word_flip", lambda s: s.__setitem__(o0 + 384 + 40, s[o0 + 384 + 40] ^ 0x5A), None)
    return out


def test_oracle_rejects_malformed_streams():
    x = np.minimum(np.random.default_rng(4).geometric(0.05, 20000), 255).astype(np.uint8)
    enc = R.encode(x)
    for name, s, code in corruptions(enc, x.size):
        st, _ = R.decode(s, x.size)
        if code is None:
            assert st != 0, name   # state / word damage ends at a wrong final state
        else:
            assert st == code, (name, st)
    # truncated streams
    for cut in (8, 1040, enc.size - 16):
        assert R.decode(enc[:cut], x.size)[0] != 0


DIMS = dict(gu_rows=32, gu_cols=16, dn_rows=64, dn_cols=4)


def test_ans_coded_container_layout(tmp_path):
    path = str(tmp_path / "a.vq2m")
    fn = lambda ln, e: synth.synth_expert_skewed(ln, e, sigma=300.0, **DIMS)
    size = container.write_vq2m(path, 2, 3, fn, dims=DIMS, index_coding="vq2a")
    img = np.fromfile(path, dtype=np.uint8)
    assert img.size == size
    lay = container.parse_header(memoryview(img[:container.RESERVED_HEADER_BYTES]), file_size=img.size)
    assert lay.ans_coded and lay.expert_bytes == container.record_bytes(**DIMS)
    for ln in range(2):
        for e in range(3):
            gi, gs, di, ds = fn(ln, e)
            off, nb = lay.record(ln, e)
            rec = img[off:off + nb]
            dec = np.zeros(lay.expert_bytes, np.uint8)
            for so, sb, do, n, kind in lay.segments(ln, e):
                if kind == 0:
                    st, d = R.decode(rec[so:so + sb], n)
                    assert st == 0
                else:
                    assert sb == n
                    d = rec[so:so + sb]
                dec[do:do + n] = d
            want = np.concatenate([a.view(np.uint8).reshape(-1) for a in (gi, gs, di, ds)])
            assert np.array_equal(dec, want)
    # a raw container of the same experts has the same decoded records and plain segments
    raw = str(tmp_path / "r.vq2m")
    container.write_vq2m(raw, 2, 3, fn, dims=DIMS)
    rl = container.parse_header(open(raw, "rb").read(container.RESERVED_HEADER_BYTES))
    assert not rl.ans_coded and all(k == 1 for *_, k in rl.segments(1, 2))


def test_ans_coded_container_rejects_bad_scale_sizes(tmp_path):
    path = str(tmp_path / "a.vq2m")
    container.write_vq2m(path, 1, 2, lambda ln, e: synth.synth_expert(ln, e, **DIMS), dims=DIMS,
                         index_coding="vq2a")
    img = bytearray(open(path, "rb").read())
    toff = struct.unpack_from("<Q", img, 12)[0]             # header: 4s H H H H, then moe_table_off
    struct.pack_into("<I", img, toff + 20, 7)                # entry <QIQI...>: gate_up scale size
    with pytest.raises(ValueError):
        container.parse_header(memoryview(bytes(img[:container.RESERVED_HEADER_BYTES])))
