"""Failure detection without a GPU fault: the expert-parallel rank sum's bounded wait for a peer.

One GPU, one process: the layer is called as rank 0 of a world of 2 whose "peer" buffer is a
second local buffer that no other rank ever writes, so the wait for rank 1's flags cannot be
satisfied. With a short poll limit the kernel gives up, records the timeout in the status word
(0x200), finishes with the data it has (rank 0's own partial), and the context stays usable:
a normal single-GPU layer right after runs and matches the oracle path."""
import numpy as np
import pytest
import torch

from compressai_b200 import _lib, moe, synth, vq

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _LoneRankPeers:
    """The fields moe.moe_layer reads from ep.PeerReduceContext, backed by local memory only."""

    def __init__(self, max_tokens, hidden, max_polls):
        lib = _lib.load()
        nbytes = lib.vq2_moe_peer_buffer_bytes(max_tokens, hidden, 2)
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(2)]
        self.ptrs = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device=DEV)
        self.peers_dev = self.ptrs.data_ptr()
        self.rank, self.world, self.max_tokens, self.max_polls = 0, 2, max_tokens, max_polls
        self.epochs = torch.zeros(4, dtype=torch.int32, device=DEV)
        self.err = torch.zeros(1, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("T", [1, 2])
def test_peer_wait_gives_up_and_reports_timeout(T):
    """T = 1 exercises the exchange fused into the one-token down kernel, T = 2 the peer combine
    kernel; both use the same flags and sequence number."""
    E = 16
    pool = moe.ExpertRecordPool(E // 2 + 1, DEV)
    for e in range(E // 2 + 1):
        pool.set_expert(e, *[torch.from_numpy(a) for a in synth.synth_expert(41, e)])
    cb = torch.from_numpy(synth.random_codebooks(2)["16"]).to(DEV)
    r_in, r_mid = vq.get_rot("moe_expert_2048", 2048, DEV), vq.get_rot("moe_expert_512", 512, DEV)
    gate = torch.from_numpy((0.05 * np.random.default_rng(1).standard_normal(2048)).astype(np.float32)).to(DEV)
    h = torch.randn(T, 2048, device=DEV).half()
    lg = torch.randn(T, E, device=DEV)
    peers = _LoneRankPeers(T, 2048, max_polls=4096)
    for call in range(2):  # the sequence number advances; the second wait gives up the same way
        peers.err.zero_()
        out = moe.moe_layer(h, lg, pool, cb, r_in, r_mid, 4, shared_gate=gate, lo=0, hi=E // 2, rank=0, world=2,
                            peer=peers, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert int(peers.err.item()) == 0x200, call
        # what it has: rank 0's own partial (the missing rank's slot is still zero)
        part = moe.moe_layer(h, lg, pool, cb, r_in, r_mid, 4, shared_gate=gate, lo=0, hi=E // 2, rank=0, world=2,
                             out_dtype=torch.float32)
        assert torch.allclose(out, part, rtol=1e-5, atol=1e-6), call
    # the context is intact: a complete single-GPU layer afterwards is finite and deterministic
    full = moe.ExpertRecordPool(E, DEV)
    for e in range(E):
        full.set_expert(e, *[torch.from_numpy(a) for a in synth.synth_expert(42, e)])
    y1 = moe.moe_layer(h, lg, full, cb, r_in, r_mid, 4)
    y2 = moe.moe_layer(h, lg, full, cb, r_in, r_mid, 4)
    assert torch.isfinite(y1.float()).all() and torch.equal(y1, y2)
