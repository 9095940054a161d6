"""The paged ``.vq2m`` expert container: layout, parsing and writing.

Layout (identical to the reference so files interchange; reference vq2/pack_35b_to_vq2m.py:
22-35, 58, 138-152, 200-247 and the reader vq2/paged_runtime.py:89-123):

* 64-byte header ``<4sHHHH QQQQQ 12s>``: magic ``VQ2M``, version 1, num_layers, num_experts,
  pad, moe_table_off (64), moe_table_len, meta_json_off, meta_json_len, payload_start
  (2 MiB), 12 pad bytes;
* expert table of num_layers x num_experts entries ``<QIQIQIQI>`` (48 B):
  (offset, size) of gate_up indices (int16), gate_up scales (fp16), down indices (int16),
  down scales (fp16);
* UTF-8 JSON meta (dims ``gu_rows``/``gu_cols``/``dn_rows``/``dn_cols``, optional
  ``other_tensors`` and ``expert_modes``);
* payload from 2 MiB: per layer, per expert, the four tensors back to back, so one expert is a
  single contiguous record of ``expert_bytes`` bytes (792,576 B at the 35B-A3B shape).

ANS-coded variant (this repository's extension; meta ``"index_coding": "vq2a"``): the two index
entries of each expert point at VQ2A rANS streams of the index bytes (compressai_b200.ans) and
their sizes are the stream sizes; scales stay stored. A record is still contiguous, of variable
size, and a paged miss copies it compressed and expands it into the slot on the GPU. Readers that
do not know the key see the header unchanged and reject the mismatched sizes.
"""
import json
import os
import struct

import numpy as np

from . import synth

MAGIC = b"VQ2M"
VERSION = 1
HEADER_FMT = "<4sHHHH QQQQQ 12s"
ENTRY_FMT = "<QIQIQIQI"
HEADER_SIZE = struct.calcsize(HEADER_FMT)       # 64
ENTRY_SIZE = struct.calcsize(ENTRY_FMT)         # 48
RESERVED_HEADER_BYTES = 2 * 1024 * 1024
DEFAULT_DIMS = dict(gu_rows=1024, gu_cols=256, dn_rows=2048, dn_cols=64)


def record_bytes(gu_rows=1024, gu_cols=256, dn_rows=2048, dn_cols=64, bits=2):
    """Bytes of one expert record: 792,576 at 2 bpw, 1,185,792 for a promoted 3 bpw expert
    (each index entry is idx0 int16 followed by idx1 uint8)."""
    w = 3 if bits == 3 else 2
    return gu_rows * gu_cols * w + gu_rows * 2 + dn_rows * dn_cols * w + dn_rows * 2


class Vq2mLayout:
    """Parsed header, table and meta of a .vq2m image (bytes-like or file head)."""

    def __init__(self, num_layers, num_experts, payload_start, table, meta):
        self.num_layers = num_layers
        self.num_experts = num_experts
        self.payload_start = payload_start
        self.table = table          # [layer][expert] -> 8-tuple
        self.meta = meta
        self.gu_rows = meta.get("gu_rows", 1024)
        self.gu_cols = meta.get("gu_cols", 256)
        self.dn_rows = meta.get("dn_rows", 2048)
        self.dn_cols = meta.get("dn_cols", 64)

        self.index_coding = meta.get("index_coding", "raw")
        if self.index_coding not in ("raw", "vq2a"):
            raise ValueError(f"unknown index_coding {self.index_coding!r}")

    @property
    def expert_bytes(self):
        """Bytes of one decoded expert record (the pool slot size)."""
        return record_bytes(self.gu_rows, self.gu_cols, self.dn_rows, self.dn_cols)

    @property
    def ans_coded(self):
        return self.index_coding == "vq2a"

    @property
    def max_record_bytes(self):
        """Largest stored record (== expert_bytes for raw containers)."""
        m = 0
        for row in self.table:
            for (og, sg, os_, ss, od, sd, ods, sds) in row:
                if sg:
                    m = max(m, sg + ss + sd + sds)
        return m

    def segments(self, layer, expert):
        """Decode plan of one record, relative to the record start: [(src_off, src_bytes,
        dst_off, n, kind)] for gate_up indices, gate_up scales, down indices, down scales
        (kind 0 = VQ2A stream, 1 = stored); dst offsets follow the decoded record layout."""
        og, sg, os_, ss, od, sd, ods, sds = self.table[layer][expert]
        n_gi, n_gs = self.gu_rows * self.gu_cols * 2, self.gu_rows * 2
        n_di, n_ds = self.dn_rows * self.dn_cols * 2, self.dn_rows * 2
        k = 0 if self.ans_coded else 1
        return [(0, sg, 0, n_gi, k), (os_ - og, ss, n_gi, n_gs, 1), (od - og, sd, n_gi + n_gs, n_di, k),
                (ods - og, sds, n_gi + n_gs + n_di, n_ds, 1)]

    def expert_mode(self, layer, expert):
        """3 for a promoted 3 bpw expert (meta expert_modes["L:E"] == 3), else 2."""
        return 3 if self.meta.get("expert_modes", {}).get(f"{layer}:{expert}") == 3 else 2

    def record(self, layer, expert):
        """(offset, nbytes) of the contiguous record of one expert; raises if the four tensors
        are not back to back (a file the paging fast path cannot serve with one copy)."""
        og, sg, os_, ss, od, sd, ods, sds = self.table[layer][expert]
        if sg == 0:
            raise ValueError(f"expert ({layer}, {expert}) missing from the container")
        if not (os_ == og + sg and od == os_ + ss and ods == od + sd):
            raise ValueError(f"expert ({layer}, {expert}) is not stored contiguously")
        return og, sg + ss + sd + sds


def parse_header(head, file_size=None):
    """Parse header + table + meta from the first bytes of a .vq2m (at least payload_start
    bytes, or the whole image). Raises ValueError on a bad magic/version or out-of-range
    offsets."""
    head = memoryview(head)
    if len(head) < HEADER_SIZE:
        raise ValueError("truncated .vq2m header")
    (magic, version, nl, ne, _, toff, tlen, moff, mlen, pstart, _) = struct.unpack(HEADER_FMT, head[:HEADER_SIZE])
    if magic != MAGIC or version != VERSION:
        raise ValueError("invalid .vq2m file or incompatible version")
    if tlen != nl * ne * ENTRY_SIZE or toff + tlen > len(head) or moff + mlen > len(head):
        raise ValueError("corrupt .vq2m header: table/meta outside the header region")
    ents = list(struct.iter_unpack(ENTRY_FMT, head[toff:toff + tlen]))
    table = [ents[ln * ne:(ln + 1) * ne] for ln in range(nl)]
    meta = json.loads(bytes(head[moff:moff + mlen]).decode("utf-8"))
    lay = Vq2mLayout(nl, ne, pstart, table, meta)
    if lay.ans_coded:  # stored scales must have the dimensions' sizes
        for row in table:
            for (og, sg, os_, ss, od, sd, ods, sds) in row:
                if sg and (ss, sds) != (lay.gu_rows * 2, lay.dn_rows * 2):
                    raise ValueError("corrupt .vq2m: expert scale sizes disagree with the dimensions")
    if file_size is not None:
        for row in table:
            for (og, sg, os_, ss, od, sd, ods, sds) in row:
                if sg and max(og + sg, os_ + ss, od + sd, ods + sds) > file_size:
                    raise ValueError("corrupt .vq2m: expert record beyond end of file")
    return lay


def _header_bytes(num_layers, num_experts, table, meta):
    meta_b = json.dumps(meta).encode("utf-8")
    tbl = bytearray()
    for ln in range(num_layers):
        for e in range(num_experts):
            tbl += struct.pack(ENTRY_FMT, *table[ln][e])
    toff = HEADER_SIZE
    moff = toff + len(tbl)
    if moff + len(meta_b) > RESERVED_HEADER_BYTES:
        raise RuntimeError("header exceeds the reserved 2 MiB")
    hdr = struct.pack(HEADER_FMT, MAGIC, VERSION, num_layers, num_experts, 0, toff, len(tbl), moff, len(meta_b),
                      RESERVED_HEADER_BYTES, b"\x00" * 12)
    out = bytearray(RESERVED_HEADER_BYTES)
    out[:HEADER_SIZE] = hdr
    out[toff:moff] = tbl
    out[moff:moff + len(meta_b)] = meta_b
    return bytes(out)


def _table_and_meta(num_layers, num_experts, dims, meta_extra):
    gr, gc, dr, dc = dims["gu_rows"], dims["gu_cols"], dims["dn_rows"], dims["dn_cols"]
    sz = (gr * gc * 2, gr * 2, dr * dc * 2, dr * 2)
    rec = sum(sz)
    table = []
    off = RESERVED_HEADER_BYTES
    for ln in range(num_layers):
        row = []
        for e in range(num_experts):
            o1 = off
            o2 = o1 + sz[0]
            o3 = o2 + sz[1]
            o4 = o3 + sz[2]
            row.append((o1, sz[0], o2, sz[1], o3, sz[2], o4, sz[3]))
            off += rec
        table.append(row)
    meta = dict(num_layers=num_layers, num_experts=num_experts, hidden_dim=gc * 8, intermediate_dim=gr // 2,
                other_tensors={}, **dims)
    if meta_extra:
        meta.update(meta_extra)
    return table, meta, off


def write_vq2m(path, num_layers, num_experts, expert_fn, dims=None, meta_extra=None, index_coding="raw"):
    """Write a .vq2m whose expert (layer, e) is ``expert_fn(layer, e)`` = (gu_idx int16,
    gu_scale fp16, dn_idx int16, dn_scale fp16). index_coding "vq2a" stores the index tensors
    as VQ2A rANS streams (host encoder of the C-ABI library). Returns the file size."""
    dims = dict(DEFAULT_DIMS, **(dims or {}))
    if index_coding == "raw":
        # experts returned as 6-tuples (idx0, idx1, scale per matrix) are promoted 3 bpw experts:
        # index entries idx0 || idx1 and meta expert_modes["L:E"] = 3
        _, meta, _ = _table_and_meta(num_layers, num_experts, dims, meta_extra)
        table = [[None] * num_experts for _ in range(num_layers)]
        modes = {}
        off = RESERVED_HEADER_BYTES
        with open(path, "wb") as f:
            f.write(b"\x00" * RESERVED_HEADER_BYTES)
            for ln in range(num_layers):
                for e in range(num_experts):
                    parts = expert_fn(ln, e)
                    if len(parts) == 6:
                        gi0, gi1, gs, di0, di1, ds = parts
                        ent = [np.concatenate([np.ascontiguousarray(gi0, np.int16).view(np.uint8).reshape(-1),
                                               np.ascontiguousarray(gi1, np.uint8).reshape(-1)]),
                               np.ascontiguousarray(gs, np.float16).view(np.uint8).reshape(-1),
                               np.concatenate([np.ascontiguousarray(di0, np.int16).view(np.uint8).reshape(-1),
                                               np.ascontiguousarray(di1, np.uint8).reshape(-1)]),
                               np.ascontiguousarray(ds, np.float16).view(np.uint8).reshape(-1)]
                        modes[f"{ln}:{e}"] = 3
                    else:
                        ent = [a.view(np.uint8).reshape(-1) for a in _typed(parts)]
                    row = []
                    for a in ent:
                        row += [off, a.size]
                        f.write(a.tobytes())
                        off += a.size
                    table[ln][e] = tuple(row)
            if modes:
                meta = dict(meta, expert_modes=modes)
            f.seek(0)
            f.write(_header_bytes(num_layers, num_experts, table, meta))
        return off
    if index_coding != "vq2a":
        raise ValueError(f"unknown index_coding {index_coding!r}")
    from . import ans
    _, meta, _ = _table_and_meta(num_layers, num_experts, dims, dict(meta_extra or {}, index_coding="vq2a"))
    table = [[None] * num_experts for _ in range(num_layers)]
    off = RESERVED_HEADER_BYTES
    with open(path, "wb") as f:
        f.write(b"\x00" * RESERVED_HEADER_BYTES)
        for ln in range(num_layers):
            for e in range(num_experts):
                gi, gs, di, ds = _typed(expert_fn(ln, e))
                parts = [ans.encode(gi), gs.view(np.uint8), ans.encode(di), ds.view(np.uint8)]
                ent = []
                for p in parts:
                    ent += [off, p.size]
                    f.write(p.tobytes())
                    off += p.size
                table[ln][e] = tuple(ent)
        f.seek(0)
        f.write(_header_bytes(num_layers, num_experts, table, meta))
    return off


def _typed(parts):
    gi, gs, di, ds = parts
    return (np.ascontiguousarray(gi, dtype=np.int16), np.ascontiguousarray(gs, dtype=np.float16),
            np.ascontiguousarray(di, dtype=np.int16), np.ascontiguousarray(ds, dtype=np.float16))


def write_synthetic_vq2m(path, num_layers, num_experts, seed=0, **dims):
    """Container of seeded synthetic experts (compressai_b200.synth.synth_expert, data seed
    seed * 1_000_003 + layer)."""
    d = dict(DEFAULT_DIMS, **dims)
    return write_vq2m(path, num_layers, num_experts,
                      lambda ln, e: synth.synth_expert(seed * 1_000_003 + ln, e, d["gu_rows"], d["gu_cols"],
                                                       d["dn_rows"], d["dn_cols"]), dims=d)


def synthetic_vq2m_image(num_layers, num_experts, seed=0, out=None, **dims):
    """Whole .vq2m image in memory (numpy uint8, or written into ``out``, e.g. a pinned buffer)
    for large paging benchmarks: expert payloads are tiled from a 64 MiB seeded random block
    (uniform 16-bit indices) with fp16 scales ~0.02 patched in, which writes GBs in seconds."""
    d = dict(DEFAULT_DIMS, **dims)
    table, meta, end = _table_and_meta(num_layers, num_experts, d, None)
    img = np.empty(end, dtype=np.uint8) if out is None else out
    if img.nbytes < end:
        raise ValueError("output buffer too small")
    img[:RESERVED_HEADER_BYTES] = np.frombuffer(_header_bytes(num_layers, num_experts, table, meta), np.uint8)
    rng = np.random.default_rng(seed)
    block = rng.integers(0, 256, size=64 << 20, dtype=np.uint8)
    scale_gu = (0.02 * np.exp(0.1 * rng.standard_normal(d["gu_rows"]))).astype(np.float16).view(np.uint8)
    scale_dn = (0.02 * np.exp(0.1 * rng.standard_normal(d["dn_rows"]))).astype(np.float16).view(np.uint8)
    pos = RESERVED_HEADER_BYTES
    rec = record_bytes(d["gu_rows"], d["gu_cols"], d["dn_rows"], d["dn_cols"])
    boff = 0
    for ln in range(num_layers):
        for e in range(num_experts):
            n = rec
            if boff + n > block.size:
                boff = (boff * 7 + 4099) % (block.size - n)
            img[pos:pos + n] = block[boff:boff + n]
            og, sg, os_, ss, od, sd, ods, sds = table[ln][e]
            img[os_:os_ + ss] = scale_gu
            img[ods:ods + sds] = scale_dn
            boff += n + 4096
            pos += n
    return img[:end], end


def synthetic_ans_vq2m_image(num_layers, num_experts, seed=0, distinct=64, out=None, **dims):
    """ANS-coded (index_coding "vq2a") .vq2m image in memory for paging benchmarks: ``distinct``
    skewed-index experts (synth.synth_expert_skewed) are encoded once and their records tiled
    over the (layer, expert) grid, expert (l, e) taking record (l * num_experts + e) % distinct.
    Returns (image, size); ``out`` (e.g. a pinned buffer of at least ``size`` bytes) may be
    given, else use ``ans_image_size`` first to size it."""
    from . import ans
    d = dict(DEFAULT_DIMS, **dims)
    recs = []
    for i in range(distinct):
        gi, gs, di, ds = _typed(synth.synth_expert_skewed(seed, i, d["gu_rows"], d["gu_cols"], d["dn_rows"],
                                                          d["dn_cols"]))
        recs.append([ans.encode(gi), gs.view(np.uint8), ans.encode(di), ds.view(np.uint8)])
    _, meta, _ = _table_and_meta(num_layers, num_experts, d, {"index_coding": "vq2a"})
    table = [[None] * num_experts for _ in range(num_layers)]
    off = RESERVED_HEADER_BYTES
    for ln in range(num_layers):
        for e in range(num_experts):
            ent = []
            for p in recs[(ln * num_experts + e) % distinct]:
                ent += [off, p.size]
                off += p.size
            table[ln][e] = tuple(ent)
    img = np.empty(off, dtype=np.uint8) if out is None else out
    if img.nbytes < off:
        raise ValueError(f"output buffer too small: {img.nbytes} < {off}")
    img[:RESERVED_HEADER_BYTES] = np.frombuffer(_header_bytes(num_layers, num_experts, table, meta), np.uint8)
    flat = [np.concatenate(r) for r in recs]
    for ln in range(num_layers):
        for e in range(num_experts):
            r = flat[(ln * num_experts + e) % distinct]
            o = table[ln][e][0]
            img[o:o + r.size] = r
    return img[:off], off


def ans_image_size(num_layers, num_experts, seed=0, distinct=64, **dims):
    """Size in bytes of synthetic_ans_vq2m_image with the same arguments."""
    from . import ans
    d = dict(DEFAULT_DIMS, **dims)
    sizes = []
    for i in range(distinct):
        gi, gs, di, ds = _typed(synth.synth_expert_skewed(seed, i, d["gu_rows"], d["gu_cols"], d["dn_rows"],
                                                          d["dn_cols"]))
        sizes.append(ans.encode(gi).size + gs.nbytes + ans.encode(di).size + ds.nbytes)
    total = RESERVED_HEADER_BYTES
    for k in range(num_layers * num_experts):
        total += sizes[k % distinct]
    return total
