"""Paged MoE runtime over a ``.vq2m`` container, mirroring reference ``vq2/paged_runtime.py``.

* ``PagedModelStore`` reads the container (offset mode: pread into pinned staging; mmap mode;
  or an in-memory image, e.g. a pinned host tensor, which is DMA'd with no staging copy).
* ``PagedMoEExpert`` keeps a static pool of C expert slots in HBM and decides hits, misses and
  evictions on the host with exactly the reference's LRU (``_get_slot``,
  vq2/paged_runtime.py:415-437: hit -> move_to_end; miss -> free_slots.pop(), else evict the
  least recently used), so hit/miss/slot sequences match it bit for bit.
* Differences from the reference: a miss is ONE copy of the contiguous 792,576-byte expert
  record into a record-layout slot (the reference issues four), on a side CUDA stream; the
  experts that hit are computed while the misses are in flight, the misses right after their
  copy lands; scales stay fp16 (the reference converts them to bf16 on the host); the whole
  (hits, misses, combine) step is three to five launches for any T instead of a Python loop
  over tokens. There is no CPU compute path: CPU devices may hold the bookkeeping (for tests)
  but forward() on them raises.
"""
import ctypes
import mmap
import os
import threading
from collections import OrderedDict

import numpy as np
import torch
import torch.nn as nn

from . import _lib, ans, container, moe, vq

DEVICE = "cuda" if torch.cuda.is_available() else "cpu"


class PagedModelStore:
    """Reader of a .vq2m container (reference vq2/paged_runtime.py:49-284).

    use_mmap=False: offset mode, each expert record is read with pread into a pinned staging
    ring and copied to the device asynchronously. use_mmap=True: the file is memory-mapped and
    records are copied from the mapping into the staging ring. ``PagedModelStore.from_image``
    wraps an in-memory image (a pinned uint8 tensor is copied to the device directly)."""

    STAGING_BUFFERS = 8

    def __init__(self, file_path, use_mmap=False, device=None, _image=None):
        self.device = device if device is not None else DEVICE
        self.use_mmap = use_mmap
        self.lock = threading.Lock()
        self.mm = None
        self.file = None
        self.image = None
        if _image is not None:
            self.file_path = None
            self.image = _image
            head = _image[:container.RESERVED_HEADER_BYTES]
            head = head.numpy() if isinstance(head, torch.Tensor) else head
            self.layout = container.parse_header(memoryview(np.ascontiguousarray(head)), file_size=len(_image))
        else:
            self.file_path = os.fspath(file_path)
            if not os.path.exists(self.file_path):
                raise FileNotFoundError(f".vq2m container not found: {self.file_path}")
            size = os.path.getsize(self.file_path)
            self.file = open(self.file_path, "rb")
            head = self.file.read(min(size, container.RESERVED_HEADER_BYTES))
            self.layout = container.parse_header(head, file_size=size)
            if use_mmap:
                self.mm = mmap.mmap(self.file.fileno(), 0, access=mmap.ACCESS_READ)
        lay = self.layout
        self.num_layers, self.num_experts = lay.num_layers, lay.num_experts
        self.payload_start = lay.payload_start
        self.moe_offsets = lay.table
        self.meta = lay.meta
        self.other_tensors = self.meta.get("other_tensors", {})
        self.gu_rows, self.gu_cols = lay.gu_rows, lay.gu_cols
        self.dn_rows, self.dn_cols = lay.dn_rows, lay.dn_cols
        self.expert_bytes = lay.expert_bytes
        self.ans_coded = lay.ans_coded
        self.max_record_bytes = lay.max_record_bytes if lay.ans_coded else lay.expert_bytes
        self._dev_stage = {}     # (device, stream) -> staging ring / buffer for compressed records
        self._rec_cache = {}     # (layer, expert) -> (offset, bytes, segment plan)
        self._ans_status = {}    # device -> int32 decode status word
        self._staging = None
        self._staging_next = 0
        self.bytes_paged = 0

    @classmethod
    def from_image(cls, image, device=None):
        """Container held in host memory (numpy uint8 array or uint8 tensor, pinned for DMA)."""
        return cls(None, device=device, _image=image)

    # ---- raw record access -------------------------------------------------------------------
    def _host_record(self, layer_idx, expert_id):
        """Host bytes of one expert record: a tensor view (image / mmap) or None (offset mode)."""
        off, nb = self.layout.record(layer_idx, expert_id)
        if self.image is not None:
            img = self.image
            return img[off:off + nb] if isinstance(img, torch.Tensor) else torch.from_numpy(img[off:off + nb])
        if self.mm is not None:
            return np.frombuffer(self.mm, dtype=np.uint8, count=nb, offset=off)
        return None

    def read_record(self, layer_idx, expert_id, out=None):
        """Copy one stored expert record (compressed in an ANS-coded container) into a host
        buffer (numpy/tensor uint8) and return it."""
        off, nb = self.layout.record(layer_idx, expert_id)
        if out is None:
            out = np.empty(nb, dtype=np.uint8)
        view = out.numpy() if isinstance(out, torch.Tensor) else out
        src = self._host_record(layer_idx, expert_id)
        if src is not None:
            view[:nb] = src.numpy() if isinstance(src, torch.Tensor) else src
        else:
            with self.lock:
                got = os.preadv(self.file.fileno(), [memoryview(view[:nb])], off)
            if got != nb:
                raise IOError(f"short read of expert ({layer_idx}, {expert_id}): {got} of {nb} bytes")
        return out

    def _staging_ring(self):
        if self._staging is None:
            pin = torch.cuda.is_available()
            self._staging = [(torch.empty(self.max_record_bytes, dtype=torch.uint8, pin_memory=pin),
                              torch.cuda.Event() if pin else None) for _ in range(self.STAGING_BUFFERS)]
        return self._staging

    def load_record_async(self, layer_idx, expert_id, dst, stream=None):
        """Copy one expert record into device memory ``dst`` (uint8 [expert_bytes]) on
        ``stream`` without blocking the host on the copy: pinned images go straight to the
        device; other sources pass through a ring of pinned staging buffers, each reused only
        after its previous copy has completed.

        ANS-coded containers: the compressed record lands in one of a ring of device staging
        buffers owned by ``stream``, and a decode stream paired with it expands the record into
        ``dst`` (one launch), so the copy of the next miss overlaps this decode. Consumers wait
        on ``load_streams(stream)``; decode errors raise the status word read by
        check_decode_status."""
        src = self._host_record(layer_idx, expert_id)
        stream = stream or torch.cuda.current_stream(dst.device)
        _, nb = self.layout.record(layer_idx, expert_id)
        if self.ans_coded:
            ring = self._ans_ring(dst.device, stream)
            land, ready, free = ring["bufs"][ring["next"]]
            ring["next"] = (ring["next"] + 1) % len(ring["bufs"])
            stream.wait_event(free)  # the decode that last read this staging buffer is done
            land = land[:nb]
        else:
            land = dst
        if isinstance(src, torch.Tensor) and src.is_pinned():
            with torch.cuda.stream(stream):
                land.copy_(src, non_blocking=True)
        else:
            hring = self._staging_ring()
            buf, ev = hring[self._staging_next]
            self._staging_next = (self._staging_next + 1) % len(hring)
            ev.synchronize()  # the previous copy out of this buffer is done
            self.read_record(layer_idx, expert_id, out=buf)
            with torch.cuda.stream(stream):
                land.copy_(buf[:nb], non_blocking=True)
                ev.record(stream)
        if self.ans_coded:
            dec = ring["decode_stream"]
            ready.record(stream)
            dec.wait_event(ready)
            ans.decode_segments(land, self.layout.segments(layer_idx, expert_id), dst,
                                self.decode_status(dst.device), dec)
            free.record(dec)
        self.bytes_paged += nb

    ANS_STAGES = 4

    def _ans_ring(self, device, stream):
        key = (str(device), stream.cuda_stream)
        ring = self._dev_stage.get(key)
        if ring is None:
            ring = {"decode_stream": torch.cuda.Stream(device), "next": 0,
                    "bufs": [(torch.empty(self.max_record_bytes, dtype=torch.uint8, device=device),
                              torch.cuda.Event(), torch.cuda.Event()) for _ in range(self.ANS_STAGES)]}
            self._dev_stage[key] = ring
        return ring

    def load_streams(self, stream):
        """Streams whose work a consumer of records loaded on ``stream`` must wait for."""
        ring = self._dev_stage.get((str(stream.device), stream.cuda_stream))
        return [stream] if ring is None else [stream, ring["decode_stream"]]

    # ---- native paged step support ------------------------------------------------------------
    def pinned_image(self):
        """True when records are read from a pinned host image (the native step's source)."""
        return isinstance(self.image, torch.Tensor) and self.image.is_pinned()

    def miss_arrays(self, layer_idx, misses):
        """Host arrays describing the records of ``misses`` [(expert, slot)] for
        vq2_paged_moe_step: (src pointers uint64, bytes int64, slots int32, segment plans
        int64 [n, 20] or None, total bytes)."""
        n = len(misses)
        src = np.empty(n, dtype=np.uint64)
        nbytes = np.empty(n, dtype=np.int64)
        slots = np.empty(n, dtype=np.int32)
        segs = np.empty((n, 20), dtype=np.int64) if self.ans_coded else None
        base = self.image.data_ptr()
        cache = self._rec_cache
        for i, (e, slot) in enumerate(misses):
            key = (layer_idx, e)
            ent = cache.get(key)
            if ent is None:
                off, nb = self.layout.record(layer_idx, e)
                plan = np.asarray(self.layout.segments(layer_idx, e), dtype=np.int64).reshape(-1) \
                    if self.ans_coded else None
                ent = cache[key] = (off, nb, plan)
            src[i] = base + ent[0]
            nbytes[i] = ent[1]
            slots[i] = slot
            if segs is not None:
                segs[i] = ent[2]
        return src, nbytes, slots, segs, int(nbytes.sum())

    def pager_stage(self, device, copy_stream):
        """Staging of coded records for the native step, one per copy stream and shared by the
        layers that page through it: a device buffer of two halves of 8 records, a decode
        stream, the events ordering them and the host turn counter."""
        key = ("pager", str(device), copy_stream.cuda_stream)
        st = self._dev_stage.get(key)
        if st is None:
            half = 8 * ((self.max_record_bytes + 255) // 256 * 256)
            evs = [torch.cuda.Event() for _ in range(3)]
            for ev in evs:  # the C side waits on them before their first record
                ev.record(copy_stream)
            st = {"buf": torch.empty(2 * half, dtype=torch.uint8, device=device),
                  "decode_stream": torch.cuda.Stream(device), "ready": evs[0], "free0": evs[1], "free1": evs[2],
                  "turn": np.zeros(1, dtype=np.int64)}
            self._dev_stage[key] = st
        return st

    def decode_status(self, device):
        """The device status word shared by every ANS decode of this store on ``device``."""
        key = str(torch.device(device))
        st = self._ans_status.get(key)
        if st is None:
            st = ans.new_status(device)
            self._ans_status[key] = st
        return st

    def check_decode_status(self):
        """Synchronize and raise ans.ANSDecodeError if any decode met a malformed stream."""
        for key, st in self._ans_status.items():
            torch.cuda.synchronize(torch.device(key))
            ans.check_status(st)

    def read_expert_record(self, layer_idx, expert_id):
        """Decoded record of one expert (host uint8 [expert_bytes]); ANS-coded records are
        decoded on the GPU."""
        if not self.ans_coded:
            return self.read_record(layer_idx, expert_id)
        if not torch.cuda.is_available():
            raise RuntimeError("ANS-coded containers are decoded on the GPU; no CUDA device is available")
        dev = torch.device("cuda", torch.cuda.current_device())
        out = torch.empty(self.expert_bytes, dtype=torch.uint8, device=dev)
        self.load_record_async(layer_idx, expert_id, out, torch.cuda.current_stream(dev))
        self.check_decode_status()  # synchronizes the device, decode streams included
        return out.cpu().numpy()

    # ---- reference-compatible accessors -----------------------------------------------------
    def _split(self, rec):
        rec = torch.as_tensor(rec)
        gr, gc, dr, dc = self.gu_rows, self.gu_cols, self.dn_rows, self.dn_cols
        w = rec.view(torch.int16)
        o1 = gr * gc
        o2 = o1 + gr
        o3 = o2 + dr * dc
        return (w[:o1].view(gr, gc), w[o1:o2].view(torch.float16), w[o2:o3].view(dr, dc),
                w[o3:o3 + dr].view(torch.float16))

    def get_expert_weights(self, layer_idx, expert_id, device="cpu"):
        """(gu_idx int16, gu_scale fp16, dn_idx int16, dn_scale fp16) of one expert
        (vq2/paged_runtime.py:175-207; scales stay fp16 on every device)."""
        parts = self._split(torch.from_numpy(self.read_expert_record(layer_idx, expert_id)))
        return tuple(p.clone() if str(device) == "cpu" else p.to(device) for p in parts)

    def load_expert_into_slot(self, layer_idx, expert_id, slot, pool_gu_idx, pool_gu_scale, pool_dn_idx,
                              pool_dn_scale, device=None):
        """Copy one expert into slot `slot` of four separate pool tensors (reference signature,
        vq2/paged_runtime.py:125-173); scales are converted to the pool's dtype."""
        gi, gs, di, ds = self._split(torch.from_numpy(self.read_expert_record(layer_idx, expert_id)))
        nb = pool_gu_idx.is_cuda
        pool_gu_idx[slot].copy_(gi, non_blocking=False)
        pool_gu_scale[slot].copy_(gs.to(pool_gu_scale.dtype), non_blocking=nb)
        pool_dn_idx[slot].copy_(di, non_blocking=False)
        pool_dn_scale[slot].copy_(ds.to(pool_dn_scale.dtype), non_blocking=nb)
        self.bytes_paged += self.expert_bytes

    def get_dense_tensor(self, name, device="cpu"):
        """Dense bf16 tensor listed in meta["other_tensors"] (vq2/paged_runtime.py:209-226)."""
        info = self.other_tensors.get(name)
        if not info or info.get("type") != "dense":
            return None
        raw = self._read_span(info["offset"], info["size"])
        return torch.from_numpy(raw).view(torch.bfloat16).view(*info["shape"]).to(device)

    def get_quant_linear(self, name, cbs_data=None, device="cpu"):
        """Quantized linear listed in meta["other_tensors"]: a dict of indices and fp32 scales
        (vq2/paged_runtime.py:228-279 without cbs_data); with cbs_data, the dequantized bf16
        weight (inverse rotation on the device)."""
        info = self.other_tensors.get(name)
        if not info or info.get("type") != "quant_linear":
            return None
        idx = []
        for im in info["idx_meta"]:
            dt = np.int16 if im.get("dtype", "int16") == "int16" else np.uint8
            idx.append(torch.from_numpy(self._read_span(im["offset"], im["size"]).view(dt).copy()).to(device))
        sm = info["scale_meta"]
        scale = torch.from_numpy(self._read_span(sm["offset"], sm["size"]).view(np.float16).copy()).to(device).float()
        if cbs_data is None:
            return {"shape": info["shape"], "cfg": info["cfg"], "tag": info["tag"], "idx": idx, "scale": scale}
        rows, n = info["shape"]
        rec = 0
        for i, cfg_bits in enumerate(info["cfg"]):
            cb = torch.as_tensor(cbs_data[vq.cfg_key(info["cfg"], i)]).to(device=device, dtype=torch.float32)
            ix = idx[i].to(torch.int64) & (0xFFFF if cfg_bits > 8 else 0xFF)
            rec = rec + cb[ix]
        Q = rec.reshape(rows, n) * scale[:, None]
        return vq.get_rot(info["tag"], n, device).inv_f32(Q).to(torch.bfloat16)

    def _read_span(self, off, size):
        out = np.empty(size, dtype=np.uint8)
        if self.image is not None:
            img = self.image
            out[:] = (img[off:off + size].numpy() if isinstance(img, torch.Tensor) else img[off:off + size])
        elif self.mm is not None:
            out[:] = np.frombuffer(self.mm, dtype=np.uint8, count=size, offset=off)
        else:
            with self.lock:
                got = os.preadv(self.file.fileno(), [memoryview(out)], off)
            if got != size:
                raise IOError("short read")
        return out

    def close(self):
        if self.mm is not None:
            self.mm.close()
            self.mm = None
        if self.file is not None:
            self.file.close()
            self.file = None


class LRUExpertCache:
    """Whole-expert cache keyed by (layer, expert) with least-recently-used eviction and hit /
    miss counters: the older cache API of reference vq2/paged_runtime.py:287-313, kept for its
    callers (the streaming benchmark, the LEGION engine's imports). Recency is the insertion
    order of a plain dict: a hit moves its key to the end; a miss loads the expert through
    ``store.get_expert_weights(layer, expert, device=...)``, appends it, and drops keys from the
    front while more than ``capacity`` experts are held. ``cache`` exposes the entries in
    recency order (oldest first), as the reference's OrderedDict does."""

    def __init__(self, capacity=128, device=DEVICE):
        if capacity < 0:
            raise ValueError("capacity must be >= 0")
        self.capacity = int(capacity)
        self.device = device
        self.cache = {}
        self.hits = 0
        self.misses = 0

    def __len__(self):
        return len(self.cache)

    def __contains__(self, key):
        return tuple(key) in self.cache

    def get(self, store, layer_idx, expert_id):
        key = (layer_idx, expert_id)
        entry = self.cache.pop(key, None)
        if entry is None:
            self.misses += 1
            entry = tuple(store.get_expert_weights(layer_idx, expert_id, device=self.device))
        else:
            self.hits += 1
        self.cache[key] = entry
        while len(self.cache) > self.capacity:
            self.cache.pop(next(iter(self.cache)))
        return entry


class PagedMoEExpert(nn.Module):
    """Routed experts of one MoE layer served from a static HBM pool of `capacity` slots
    (vq2/paged_runtime.py:316-568). forward(hidden_states [T, H], topk_idx [T, k],
    topk_weights [T, k]) -> [T, H] in the hidden dtype. topk_idx on the host avoids the
    device-to-host read of the ids (the reference always reads them back, :443)."""

    def __init__(self, layer_idx, store, cb16, capacity=96, device=DEVICE, copy_stream=None, cb8=None):
        super().__init__()
        self.layer_idx = layer_idx
        self.store = store
        self.cb16 = cb16
        self.capacity = capacity
        self.device = torch.device(device)
        self.hidden_dim = store.gu_cols * 8
        self.intermediate_dim = store.gu_rows // 2
        # Promoted 3 bpw experts (expert_modes == 3) stay resident and bypass the LRU, as in the
        # reference (vq2/paged_runtime.py:357-389, 446-460); here they stay in VQ form (no dense
        # bf16 weights) and run through the residual-codebook expert FFN.
        self.promoted = [e for e in range(store.num_experts) if store.layout.expert_mode(layer_idx, e) == 3]
        self._promoted_row = {e: i for i, e in enumerate(self.promoted)}
        self.pool3, self.cb8 = None, cb8
        if self.promoted:
            if cb8 is None:
                raise ValueError(f"layer {layer_idx} has promoted 3-bit experts: pass cb8 (the '16_8' codebook)")
            self.pool3 = moe.Expert3Pool(len(self.promoted), self.device, store.gu_rows, store.gu_cols,
                                         store.dn_rows, store.dn_cols)
            for e, row in self._promoted_row.items():
                rec = store.read_record(layer_idx, e)
                if rec.size != self.pool3.record_bytes:
                    raise ValueError(f"promoted expert ({layer_idx}, {e}) record has {rec.size} bytes, "
                                     f"expected {self.pool3.record_bytes}")
                self.pool3.set_record(row, torch.from_numpy(rec))
        self.pool = moe.ExpertRecordPool(capacity, self.device, store.gu_rows, store.gu_cols, store.dn_rows,
                                         store.dn_cols)
        # reference attribute names, as views into the record pool
        self.pool_gu_idx, self.pool_gu_scale = self.pool.gu_idx, self.pool.gu_scale
        self.pool_dn_idx, self.pool_dn_scale = self.pool.dn_idx, self.pool.dn_scale
        self.expert_to_slot = {}
        self.free_slots = list(range(capacity))
        self.access_order = OrderedDict()
        self.hits = 0
        self.misses = 0
        self.activated_experts_set = set()
        if self.device.type == "cuda":
            self.rot_2048 = vq.get_rot("moe_expert_2048", self.hidden_dim, self.device)
            self.rot_512 = vq.get_rot("moe_expert_512", self.intermediate_dim, self.device)
            self.copy_stream = copy_stream or torch.cuda.Stream(self.device)
            self._compute_done = torch.cuda.Event()
            self._compute_done.record(torch.cuda.current_stream(self.device))
            # Native step (vq2_paged_moe_step) when records come from a pinned host image: the
            # copies, decode, id upload and expert FFN of a step are one C-ABI call.
            self.native = store.pinned_image()
            if self.native:
                self._copy_done, self._ids_done = torch.cuda.Event(), torch.cuda.Event()
                cur = torch.cuda.current_stream(self.device)
                self._copy_done.record(cur)
                self._ids_done.record(cur)
                self._ids_cap = 0
                self._ws = torch.empty(0, dtype=torch.uint8, device=self.device)
                self._layer = None
        self._pending_loads = []

    # ---- host LRU (reference semantics) -----------------------------------------------------
    def _assign_slot(self, e_id):
        """Bookkeeping of _get_slot (vq2/paged_runtime.py:415-437) without the copy:
        returns (slot, hit). The counters are updated through the instance dict: nn.Module's
        __setattr__ costs microseconds per call on this per-expert path."""
        d = self.__dict__
        self.activated_experts_set.add(e_id)
        if e_id in self.expert_to_slot:
            d["hits"] += 1
            self.access_order.move_to_end(e_id)
            return self.expert_to_slot[e_id], True
        d["misses"] += 1
        if self.free_slots:
            slot = self.free_slots.pop()
        else:
            evict_id, _ = self.access_order.popitem(last=False)
            slot = self.expert_to_slot.pop(evict_id)
        self.expert_to_slot[e_id] = slot
        self.access_order[e_id] = None
        return slot, False

    def _get_slot(self, e_id):
        """Reference-compatible: assign a slot and start paging the expert in on a miss."""
        slot, hit = self._assign_slot(e_id)
        if not hit:
            self._load(e_id, slot)
        return slot

    def _load(self, e_id, slot):
        if self.device.type != "cuda":
            self.store.load_expert_into_slot(self.layer_idx, e_id, slot, self.pool_gu_idx, self.pool_gu_scale,
                                             self.pool_dn_idx, self.pool_dn_scale)
            return
        # the slot may still be read by compute already enqueued: order the copy after it
        self.copy_stream.wait_event(self._compute_done)
        self.store.load_record_async(self.layer_idx, e_id, self.pool.raw[slot], self.copy_stream)

    # ---- native step ------------------------------------------------------------------------
    def _native_layer(self, P):
        """The vq2_paged_layer of this module, with id buffers for at least P problems."""
        if self._layer is not None and P <= self._ids_cap:
            return self._layer
        if self._layer is not None:
            self._ids_done.synchronize()  # the old pinned buffer is no longer being copied from
        cap = max(P, 64)
        self._ids_host = torch.empty(cap, dtype=torch.int32, pin_memory=True)
        self._ids_dev = torch.empty(cap, dtype=torch.int32, device=self.device)
        self._ids_cap = cap
        st = self.store
        coded = st.ans_coded
        stage = st.pager_stage(self.device, self.copy_stream) if coded else None
        status = st.decode_status(self.device) if coded else None
        self._stage = stage  # keeps the shared staging alive with this layer
        r_in, r_mid = self.rot_2048, self.rot_512
        self._layer = _lib.PagedLayer(
            pool=self.pool.raw.data_ptr(), capacity=self.capacity, gu_rows=st.gu_rows, gu_cols=st.gu_cols,
            dn_rows=st.dn_rows, dn_cols=st.dn_cols, cb0=self.cb16.data_ptr(), val_dtype=_lib.dtype_code(self.cb16),
            index_coding=1 if coded else 0, perm_in=r_in.perm.data_ptr(), sign_in=r_in.sign.data_ptr(),
            hb_in=r_in.hb, perm_mid=r_mid.perm.data_ptr(), sign_mid=r_mid.sign.data_ptr(), hb_mid=r_mid.hb,
            scale_in=float(r_in.scale), scale_mid=float(r_mid.scale),
            stage=stage["buf"].data_ptr() if coded else None, stage_bytes=stage["buf"].numel() if coded else 0,
            status=status.data_ptr() if coded else None,
            stage_turn=stage["turn"].ctypes.data if coded else None,
            decode_stream=stage["decode_stream"].cuda_stream if coded else None,
            stage_ready=stage["ready"].cuda_event if coded else None,
            stage_free0=stage["free0"].cuda_event if coded else None,
            stage_free1=stage["free1"].cuda_event if coded else None, ids_host=self._ids_host.data_ptr(),
            ids_dev=self._ids_dev.data_ptr(), ids_cap=cap, copy_stream=self.copy_stream.cuda_stream,
            copy_done=self._copy_done.cuda_event, compute_done=self._compute_done.cuda_event,
            ids_done=self._ids_done.cuda_event)
        return self._layer

    def _promoted(self, h, rows3, w, partial, out):
        """Add the promoted experts (pool3 rows ``rows3``, -1 elsewhere) to the fp32 partial of
        the paged experts, writing ``out``."""
        ids3 = torch.as_tensor(rows3, dtype=torch.int32).reshape(-1).pin_memory().to(self.device, non_blocking=True)
        moe.expert_ffn_res(h, ids3, w, self.pool3, self.cb16, self.cb8, self.rot_2048, self.rot_512, w.shape[1],
                           add=partial, out=out)

    def _step(self, h, slot_rows, w, out, misses, stream, rows3=None):
        """Load ``misses`` and run the experts of tokens h on ``slot_rows`` in one native call
        (plus the promoted experts of ``rows3``)."""
        if rows3 is not None and any(r >= 0 for row in rows3 for r in row):
            partial = torch.empty(out.shape, dtype=torch.float32, device=self.device)
            self._step(h, slot_rows, w, partial, misses, stream)
            self._promoted(h, rows3, w, partial, out)
            return
        T, K = len(slot_rows), len(slot_rows[0])
        layer = self._native_layer(T * K)
        need = _lib.load().vq2_moe_expert_ffn_workspace(T, K, self.store.gu_rows, self.store.dn_rows)
        if self._ws.numel() < need:  # zeroed: the fused FFN keeps its counters in the first 1 KB
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        slots = np.asarray(slot_rows, dtype=np.int32).reshape(-1)
        n = len(misses)
        if n:
            src, nbytes, mslots, segs, total = self.store.miss_arrays(self.layer_idx, misses)
            args = (n, src.ctypes.data, nbytes.ctypes.data, mslots.ctypes.data,
                    segs.ctypes.data if segs is not None else None)
            self.store.bytes_paged += total
        else:
            args = (0, None, None, None, None)
        _lib.call("vq2_paged_moe_step", ctypes.byref(layer), h.data_ptr(), _lib.dtype_code(h), T, K,
                  slots.ctypes.data, w.data_ptr(), *args, self._ws.data_ptr(), self._ws.numel(), out.data_ptr(),
                  _lib.dtype_code(out), stream.cuda_stream)

    def _forward_native(self, h, ids_list, w, out, stream):
        T = h.shape[0]
        seg_start, seg_slots, slot_rows, rows3, misses = 0, set(), [], [], []
        promoted = self._promoted_row
        for t in range(T):
            row, row3 = [], []
            for e in ids_list[t]:
                e = int(e)
                if e in promoted:  # resident 3 bpw expert: not paged, not counted by the LRU
                    row.append(-1)
                    row3.append(promoted[e])
                    continue
                row3.append(-1)
                slot, hit = self._assign_slot(e)
                if not hit and slot in seg_slots:
                    # the slot is still to be read by earlier tokens of this batch: run them first
                    self._step(h[seg_start:t], slot_rows, w[seg_start:t], out[seg_start:t], misses, stream, rows3)
                    seg_start, seg_slots, slot_rows, rows3, misses = t, set(), [], [], []
                if not hit:
                    misses.append((e, slot))
                row.append(slot)
            slot_rows.append(row)
            rows3.append(row3)
            seg_slots.update(row)
        self._step(h[seg_start:T], slot_rows, w[seg_start:T], out[seg_start:T], misses, stream, rows3)
        return out

    def _join_loads(self, stream):
        for s in self.store.load_streams(self.copy_stream):
            stream.wait_stream(s)

    # ---- compute ----------------------------------------------------------------------------
    def _run(self, h, slots, w, out, rows3=None):
        """Expert FFN of tokens h [t, H] on pool slots [t, k] with weights [t, k] into out (plus
        the promoted experts of ``rows3``)."""
        stream = torch.cuda.current_stream(self.device)
        ids = torch.as_tensor(slots, dtype=torch.int32).reshape(-1).pin_memory().to(self.device, non_blocking=True)
        if rows3 is not None and any(r >= 0 for row in rows3 for r in row):
            partial = moe.expert_ffn(h, ids, w, self.pool, self.cb16, self.rot_2048, self.rot_512, w.shape[1],
                                     out_dtype=torch.float32)
            self._promoted(h, rows3, w, partial, out)
        else:
            moe.expert_ffn(h, ids, w, self.pool, self.cb16, self.rot_2048, self.rot_512, w.shape[1], out=out)
        self._compute_done.record(stream)

    def forward(self, hidden_states, topk_idx, topk_weights):
        if self.device.type != "cuda" or not hidden_states.is_cuda:
            raise ValueError("PagedMoEExpert computes on CUDA only (no CPU fallback)")
        T = hidden_states.shape[0]
        K = topk_idx.shape[-1]
        ids = topk_idx.reshape(T, K)
        ids_list = ids.tolist() if not ids.is_cuda else ids.cpu().tolist()  # reference: .tolist() sync
        w = topk_weights.reshape(T, K)
        if w.is_cuda:
            w = w.to(self.device, torch.float32).contiguous()
        else:  # a pinned bounce keeps the upload asynchronous
            w = w.to(torch.float32).contiguous().pin_memory().to(self.device, non_blocking=True)
        h = hidden_states.reshape(T, -1).contiguous()
        out = torch.empty(T, self.hidden_dim, dtype=hidden_states.dtype, device=self.device)
        stream = torch.cuda.current_stream(self.device)
        if self.native:
            return self._forward_native(h, ids_list, w, out, stream)

        seg_start, seg_slots, slot_rows, rows3 = 0, set(), [], []
        loads_in_seg = False
        promoted = self._promoted_row
        for t in range(T):
            row, row3 = [], []
            for e in ids_list[t]:
                e = int(e)
                if e in promoted:  # resident 3 bpw expert: not paged, not counted by the LRU
                    row.append(-1)
                    row3.append(promoted[e])
                    continue
                row3.append(-1)
                slot, hit = self._assign_slot(e)
                if not hit and slot in seg_slots:
                    # the slot is still to be read by earlier tokens of this batch: run them first
                    if loads_in_seg:
                        self._join_loads(stream)
                    self._run(h[seg_start:t], slot_rows, w[seg_start:t], out[seg_start:t], rows3)
                    seg_start, seg_slots, slot_rows, rows3, loads_in_seg = t, set(), [], [], False
                if not hit:
                    self._load(e, slot)
                    loads_in_seg = True
                row.append(slot)
            slot_rows.append(row)
            rows3.append(row3)
            seg_slots.update(row)
        if loads_in_seg:
            self._join_loads(stream)
        self._run(h[seg_start:T], slot_rows, w[seg_start:T], out[seg_start:T], rows3)
        return out


class DeviceResidentPagedMoE:
    """Device-resident paged MoE decode (T = 1) over a pinned ``.vq2m`` image: per layer step,
    ``vq2_lru_step`` (the reference ``_get_slot`` LRU, vq2/paged_runtime.py:415-437, as a GPU
    kernel), then the routed-expert FFN on the slots with the missed records read by its kernels
    from the pinned image (zero-copy) and written into their slots on the way
    (``vq2_paged_moe_t1``; ``vq2_fetch_records`` + ``vq2_moe_expert_ffn`` for other shapes or with
    VQ2_PAGED_FUSED=0) -- no host synchronisation, so the steps of
    all layers (with the router) can be captured in one CUDA graph. This removes the per-layer
    ``.tolist()`` read-back of reference ``PagedMoEExpert.forward`` (:443). Hit/miss/slot
    sequences are bit-exact with the reference LRU; capacity must be at least top_k."""

    def __init__(self, store, cb16, capacity=39, device=DEVICE, top_k=8):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DeviceResidentPagedMoE runs on CUDA only")
        if not store.pinned_image() or store.ans_coded:
            raise ValueError("device-resident paging needs a raw .vq2m held in a pinned host image")
        if capacity < top_k:
            raise ValueError("capacity must be >= top_k (a step must not evict its own experts)")
        if store.meta.get("expert_modes"):
            raise ValueError("device-resident paging does not serve promoted 3-bit experts; use PagedMoEExpert")
        lib = _lib.load()
        dptr = ctypes.c_void_p()
        _lib.check(lib.vq2_host_device_pointer(store.image.data_ptr(), ctypes.byref(dptr)), "vq2_host_device_pointer")
        self.image_dev = dptr.value
        self.store, self.cb16, self.capacity, self.top_k = store, cb16, capacity, top_k
        L, E = store.num_layers, store.num_experts
        self.num_layers, self.num_experts = L, E
        self.pools = [moe.ExpertRecordPool(capacity, self.device, store.gu_rows, store.gu_cols, store.dn_rows,
                                           store.dn_cols) for _ in range(L)]
        self.state = torch.from_numpy(np.stack([self.initial_lru_state(E, capacity)] * L)).to(self.device)
        base = store.layout
        self.rec_off = torch.tensor([[base.record(ln, e)[0] for e in range(E)] for ln in range(L)], dtype=torch.int64,
                                    device=self.device)
        self.slots = torch.empty(L, top_k, dtype=torch.int32, device=self.device)
        self.miss = torch.zeros(L, 1 + 2 * top_k, dtype=torch.int32, device=self.device)
        self.rot_in = vq.get_rot("moe_expert_2048", store.gu_cols * 8, self.device)
        self.rot_mid = vq.get_rot("moe_expert_512", store.gu_rows // 2, self.device)
        # the fetch fused into the FFN (vq2_paged_moe_t1) where the shapes are its specialisation;
        # VQ2_PAGED_FUSED=0 keeps the separate fetch + FFN (the same outputs)
        self.fused = (os.environ.get("VQ2_PAGED_FUSED", "1") != "0" and lib.vq2_paged_moe_t1_workspace(top_k) > 0
                      and store.gu_cols * 8 == 2048 and store.gu_rows == 1024 and store.dn_rows == 2048
                      and store.dn_cols * 8 == 512 and self.rot_in.hb == 2048 and self.rot_mid.hb == 512
                      and cb16.dtype in (torch.float16, torch.bfloat16))
        self.ws_bytes = max(lib.vq2_moe_expert_ffn_workspace(1, top_k, store.gu_rows, store.dn_rows),
                            lib.vq2_paged_moe_t1_workspace(top_k) if self.fused else 0)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=self.device)

    @staticmethod
    def initial_lru_state(num_experts, capacity):
        """The int32 LRU state of vq2_lru_step for an empty pool: no experts, list(range(cap))
        as the free-slot stack (reference PagedMoEExpert.__init__, vq2/paged_runtime.py:344-348)."""
        nst = _lib.load().vq2_lru_state_ints(num_experts, capacity)
        st = np.full(nst, -1, dtype=np.int32)
        st[2] = capacity
        st[3:5] = 0
        st[5] = capacity
        st[6] = num_experts
        st[7] = 0
        st[8 + 3 * num_experts:] = np.arange(capacity, dtype=np.int32)
        return st

    def layer(self, ln, hidden, ids, weights, out=None):
        """One layer for one token: hidden [1, H], ids int32 [top_k] and weights fp32 [1, top_k]
        on the device (router output). Returns [1, H] in hidden's dtype (or fills ``out``)."""
        lib = _lib.load()
        st = _lib.stream_ptr(self.device)
        K = self.top_k
        if ids.dtype != torch.int32 or ids.numel() != K or not ids.is_cuda:
            raise ValueError("ids must be an int32 CUDA tensor of top_k entries")
        h = hidden.reshape(1, -1)
        if out is None:
            out = torch.empty_like(h)
        pool = self.pools[ln]
        _lib.check(lib.vq2_lru_step(_lib.ptr(self.state[ln]), _lib.ptr(ids), K, _lib.ptr(self.slots[ln]),
                                    _lib.ptr(self.miss[ln]), st), "vq2_lru_step")
        ri, rm = self.rot_in, self.rot_mid
        w = weights.reshape(-1).float().contiguous()
        if self.fused:  # missed records read from the image by the FFN kernels, written into their slots
            _lib.call("vq2_paged_moe_t1", _lib.ptr(h), _lib.dtype_code(h), K, _lib.ptr(ids), _lib.ptr(self.slots[ln]),
                      _lib.ptr(self.miss[ln]), _lib.ptr(w), _lib.ptr(pool.raw), self.capacity, self.store.gu_rows,
                      self.store.gu_cols, self.store.dn_rows, self.store.dn_cols, _lib.ptr(self.cb16),
                      _lib.dtype_code(self.cb16), _lib.ptr(ri.perm), _lib.ptr(ri.sign), ri.hb, float(ri.scale),
                      _lib.ptr(rm.perm), _lib.ptr(rm.sign), rm.hb, float(rm.scale), self.image_dev,
                      _lib.ptr(self.rec_off[ln]), self.num_experts, _lib.ptr(self.ws), self.ws_bytes, _lib.ptr(out),
                      _lib.dtype_code(out), st)
            return out
        _lib.check(lib.vq2_fetch_records(self.image_dev, _lib.ptr(self.rec_off[ln]), pool.record_bytes,
                                         _lib.ptr(pool.raw), self.capacity, _lib.ptr(self.miss[ln]), K,
                                         self.num_experts, st), "vq2_fetch_records")
        _lib.call("vq2_moe_expert_ffn", _lib.ptr(h), _lib.dtype_code(h), 1, K, _lib.ptr(self.slots[ln]),
                  _lib.ptr(weights), _lib.ptr(pool.raw), self.capacity, self.store.gu_rows, self.store.gu_cols,
                  self.store.dn_rows, self.store.dn_cols, _lib.ptr(self.cb16), _lib.dtype_code(self.cb16),
                  _lib.ptr(ri.perm), _lib.ptr(ri.sign), ri.hb, float(ri.scale), _lib.ptr(rm.perm),
                  _lib.ptr(rm.sign), rm.hb, float(rm.scale), _lib.ptr(self.ws), self.ws_bytes, _lib.ptr(out),
                  _lib.dtype_code(out), st)
        return out

    def lru_view(self, ln):
        """Host copy of one layer's LRU: (hits, misses, expert_to_slot dict, access order list,
        error flag) -- for checking against the reference sequence."""
        s = self.state[ln].cpu().numpy()
        E = self.num_experts
        e2s = s[8:8 + E]
        nxt = s[8 + 2 * E:8 + 3 * E]
        order, x = [], int(s[0])
        while x >= 0 and len(order) <= E:
            order.append(x)
            x = int(nxt[x])
        return int(s[3]), int(s[4]), {int(e): int(e2s[e]) for e in np.nonzero(e2s >= 0)[0]}, order, int(s[7])
