"""Device-resident paging (T = 1 decode, no host round trip): the GPU LRU against the reference
_get_slot sequence (oracle), outputs bit-equal to the host-driven PagedMoEExpert on the same
trace, the golden reference LRU traces, and a whole multi-layer step captured in a CUDA graph."""
import numpy as np
import pytest
import torch

from compressai_b200 import container, paged_runtime, synth
from oracle import vq2_oracle as O
from tests.conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def pinned_store(tmp_path, layers, E, seed=3):
    path = str(tmp_path / "d.vq2m")
    container.write_synthetic_vq2m(path, layers, E, seed=seed)
    img = torch.from_numpy(np.fromfile(path, np.uint8)).pin_memory()
    return paged_runtime.PagedModelStore.from_image(img, device=DEV)


def cb16():
    return torch.from_numpy(synth.random_codebooks(1)["16"]).to(DEV)


def zipf_ids(rng, E, K=8, s=1.1):
    p = 1.0 / np.arange(1, E + 1) ** s
    return rng.choice(E, K, replace=False, p=p / p.sum())


@pytest.mark.parametrize("cap", [8, 12, 30])
def test_device_lru_matches_reference_sequence(tmp_path, cap):
    layers, E = 2, 40
    store = pinned_store(tmp_path, layers, E)
    dr = paged_runtime.DeviceResidentPagedMoE(store, cb16(), capacity=cap, device=DEV)
    oracles = [O.LRUSlotOracle(cap) for _ in range(layers)]
    rng = np.random.default_rng(cap)
    h = torch.randn(1, 2048, device=DEV).half()
    w = torch.full((1, 8), 0.125, device=DEV)
    for step in range(25):
        for ln in range(layers):
            ids = zipf_ids(rng, E)
            dr.layer(ln, h, torch.from_numpy(ids.astype(np.int32)).to(DEV), w)
            want = [oracles[ln].get_slot(int(e))[0] for e in ids]
            assert dr.slots[ln].cpu().tolist() == want, (step, ln)
            hits, misses, e2s, order, err = dr.lru_view(ln)
            o = oracles[ln]
            assert (hits, misses, e2s, order, err) == (o.hits, o.misses, o.expert_to_slot, list(o.access_order), 0)
    store.close()


def test_device_lru_golden_reference_traces():
    """vq2_lru_step against the slot sequences recorded from the live reference _get_slot (Zipf
    trace, capacities 39 and 8; the capacity-4 trace is below top-k, which the device LRU
    refuses), every layer and step."""
    from compressai_b200 import _lib
    lib = _lib.load()
    d = golden("lru.npz")
    for name in ("cap39", "cap8"):
        steps, layers, cap, _ = (int(v) for v in d[f"{name}_meta"])
        trace = torch.from_numpy(d[f"{name}_trace"].astype(np.int32)).to(DEV)
        init = paged_runtime.DeviceResidentPagedMoE.initial_lru_state(256, cap)
        state = torch.from_numpy(np.stack([init] * layers)).to(DEV)
        slots = torch.empty(steps, layers, 8, dtype=torch.int32, device=DEV)
        miss = torch.zeros(layers, 17, dtype=torch.int32, device=DEV)
        st = _lib.stream_ptr(DEV)
        for s_ in range(steps):
            for ln in range(layers):
                assert lib.vq2_lru_step(_lib.ptr(state[ln]), _lib.ptr(trace[s_, ln]), 8, _lib.ptr(slots[s_, ln]),
                                        _lib.ptr(miss[ln]), st) == 0
        assert np.array_equal(slots.cpu().numpy(), d[f"{name}_slots"].astype(np.int32)), name
        stt = state.cpu().numpy()
        assert np.array_equal(stt[:, 3:5], d[f"{name}_counters"][:, :2]), name   # hits, misses
        assert (stt[:, 7] == 0).all()


def test_device_paging_outputs_equal_host_paging(tmp_path):
    layers, E, cap = 3, 48, 10
    store = pinned_store(tmp_path, layers, E, seed=11)
    cb = cb16()
    dr = paged_runtime.DeviceResidentPagedMoE(store, cb, capacity=cap, device=DEV)
    host = [paged_runtime.PagedMoEExpert(ln, store, cb, capacity=cap, device=DEV) for ln in range(layers)]
    rng = np.random.default_rng(5)
    h_d = h_h = torch.from_numpy(rng.standard_normal((1, 2048)).astype(np.float16)).to(DEV)
    for step in range(12):
        for ln in range(layers):
            ids = zipf_ids(rng, E)
            w = torch.from_numpy(rng.random((1, 8)).astype(np.float32)).to(DEV)
            h_d = dr.layer(ln, h_d, torch.from_numpy(ids.astype(np.int32)).to(DEV), w)
            h_h = host[ln](h_h, torch.from_numpy(ids[None].astype(np.int64)), w)
            assert torch.equal(h_d, h_h), (step, ln)
            hits, misses, e2s, _, _ = dr.lru_view(ln)
            assert (hits, misses, e2s) == (host[ln].hits, host[ln].misses, host[ln].expert_to_slot)
    # the fused path wrote every missed record into its slot while computing with it: each
    # resident expert's slot holds exactly its record of the image
    assert dr.fused
    for ln in range(layers):
        _, _, e2s, _, _ = dr.lru_view(ln)
        for e, slot in e2s.items():
            off = int(dr.rec_off[ln, e])
            rec = store.image[off:off + dr.pools[ln].record_bytes].to(DEV)
            assert torch.equal(dr.pools[ln].raw[slot], rec), (ln, e, slot)
    store.close()


def test_device_paging_step_in_one_cuda_graph(tmp_path):
    """All layers of a step (LRU, fetch, FFN) captured once; replays with new ids give the eager
    results and LRU states."""
    layers, E, cap = 3, 40, 9
    store = pinned_store(tmp_path, layers, E, seed=2)
    cb = cb16()
    eager = paged_runtime.DeviceResidentPagedMoE(store, cb, capacity=cap, device=DEV)
    graphed = paged_runtime.DeviceResidentPagedMoE(store, cb, capacity=cap, device=DEV)
    ids_buf = torch.zeros(layers, 8, dtype=torch.int32, device=DEV)
    w = torch.full((1, 8), 0.125, device=DEV)
    h_in = torch.randn(1, 2048, device=DEV).half()
    h_out = torch.empty_like(h_in)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            h = h_in
            for ln in range(layers):
                h = graphed.layer(ln, h, ids_buf[ln], w)
            h_out.copy_(h)
    torch.cuda.synchronize()
    # capture records without running: the graphed LRU is still in its initial state
    rng = np.random.default_rng(9)
    for step in range(10):
        ids = np.stack([zipf_ids(rng, E) for _ in range(layers)]).astype(np.int32)
        ids_buf.copy_(torch.from_numpy(ids))
        g.replay()
        h = h_in
        for ln in range(layers):
            h = eager.layer(ln, h, torch.from_numpy(ids[ln]).to(DEV), w)
        torch.cuda.synchronize()
        assert torch.equal(h_out, h), step
        for ln in range(layers):
            assert eager.lru_view(ln) == graphed.lru_view(ln)
    store.close()


def test_device_paging_refuses_unsuitable_stores(tmp_path):
    path = str(tmp_path / "o.vq2m")
    container.write_synthetic_vq2m(path, 1, 16, seed=1)
    offset = paged_runtime.PagedModelStore(path, device=DEV)
    with pytest.raises(ValueError):
        paged_runtime.DeviceResidentPagedMoE(offset, cb16(), capacity=8, device=DEV)
    pinned = paged_runtime.PagedModelStore.from_image(torch.from_numpy(np.fromfile(path, np.uint8)).pin_memory(),
                                                      device=DEV)
    with pytest.raises(ValueError):
        paged_runtime.DeviceResidentPagedMoE(pinned, cb16(), capacity=4, device=DEV)   # below top-k
    offset.close()
    pinned.close()
