"""Row-sharded greedy lm_head (compressai_b200.shard) on one GPU: the per-rank shard GEMVs with
their keys rebased to global rows and maximised over ranks give exactly the full matrix's greedy
ids (ranks emulated one after another: only the arithmetic, no cross-rank waits); and the
exchange kernel's bounded wait gives up with its status word when the "peer" never answers.
The cross-GPU exchange itself runs in tests/test_ep_gpu.py when the box has 2+ GPUs."""
import numpy as np
import pytest
import torch

from compressai_b200 import _lib, kernels, runtime, shard, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rebase(keys, lo):
    local = 0xFFFFFFFF - (keys & 0xFFFFFFFF)
    return (keys & ~0xFFFFFFFF) | (0xFFFFFFFF - (local + lo))


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("M", [1, 4])
def test_shard_keys_max_equals_full_greedy(world, M):
    V, n = 20000, 2048
    idx, scale = synth.random_matrix(V + world, V, n)
    cbd = {k: torch.from_numpy(v).to(DEV) for k, v in synth.random_codebooks(1).items()}
    full = runtime.PackedLinear((V, n), (16,), "lm_head", [torch.from_numpy(idx[0])], torch.from_numpy(scale), cbd, DEV)
    x = torch.randn(world * M, n, device=DEV).half()
    want = full.greedy(x)
    best = None
    for r in range(world):
        lo, hi = shard.shard_rows(V, world, r)
        sh = runtime.PackedLinear((hi - lo, n), (16,), "lm_head", [torch.from_numpy(idx[0][lo:hi])],
                                  torch.from_numpy(scale[lo:hi]), cbd, DEV)
        cb0, cb1 = sh.codebooks()
        k = rebase(kernels.gemv_argmax(x, sh.mat(), cb0, cb1, rot=sh.rot, keys=True), lo)
        best = k if best is None else torch.maximum(best, k)
    got = 0xFFFFFFFF - (best & 0xFFFFFFFF)
    assert torch.equal(got, want)


class _LoneRank:
    """PeerExchange fields backed by two local buffers: rank 0 of 2, the peer never writes."""

    def __init__(self, max_bytes, max_polls):
        lib = _lib.load()
        nbytes = lib.vq2_peer_exchange_buffer_bytes(max_bytes, 2)
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(2)]
        self.ptrs = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device=DEV)
        self.peers_dev = self.ptrs.data_ptr()
        self.world, self.rank, self.max_bytes, self.max_polls = 2, 0, max_bytes, max_polls
        self.state = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.err = torch.zeros(1, dtype=torch.int32, device=DEV)


def test_exchange_wait_gives_up_with_status():
    ex = _LoneRank(1 << 16, max_polls=4096)
    h = torch.randn(3, 2048, device=DEV).half()
    got = shard.PeerExchange._call(ex, h, 0, 0, torch.full((2, 3, 2048), 7.0, dtype=torch.float16, device=DEV))
    torch.cuda.synchronize()
    assert int(ex.err.item()) == 0x400
    assert torch.equal(got[0], h) and not got[1].float().abs().any()   # its own rows; the silent peer's are zero
    ex.err.zero_()
    keys = torch.tensor([(5 << 32) | (0xFFFFFFFF - 7), 0], dtype=torch.int64, device=DEV)
    m = shard.PeerExchange._call(ex, keys, 1, 100, torch.empty_like(keys))
    torch.cuda.synchronize()
    assert int(ex.err.item()) == 0x400
    assert int(0xFFFFFFFF - (int(m[0].item()) & 0xFFFFFFFF)) == 107 and int(m[1].item()) == 0
