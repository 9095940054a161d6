"""Row-sharded lm_head for greedy decode across the ranks of one node.

Rank r of N holds rows [r*V/N, (r+1)*V/N) of the (tied) lm_head as its own PackedLinear. One
greedy step for the N ranks' tokens (each rank holds its own M hidden rows, as data-parallel
decode replicas do):

1. all-gather of the N*M hidden rows over NVLink peer memory (vq2_peer_exchange, mode gather);
2. the fused-argmax GEMV over this rank's rows for all N*M tokens (vq2_gemv_argmax: each gathered
   codeword serves every token, so a rank gathers V/N rows instead of V);
3. the cross-rank maximum of the 64-bit (logit, row) keys, rebased to global rows
   (vq2_peer_exchange, mode argmax keys) -- every rank ends with the next token of every rank.

The reference's PackedLMHead (vq2/runtime.py:136-144) is a single-GPU full GEMV; this splits its
rows, which is the one dense projection that shards naturally (the others stay replicas).
"""
import torch
import torch.distributed as dist

from . import _lib, kernels


class PeerExchange:
    """Symmetric buffer (torch symmetric memory, peer-mapped on every rank of ``group``) and
    local state for vq2_peer_exchange calls of at most ``max_bytes`` per rank."""

    def __init__(self, group, device, max_bytes, max_polls=0):
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_bytes = int(max_bytes)
        self.max_polls = max_polls
        lib = _lib.load()
        nbytes = lib.vq2_peer_exchange_buffer_bytes(self.max_bytes, self.world)
        if nbytes < 0:
            raise ValueError("bad exchange buffer size")
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, name)
        self.peers_dev = self.handle.buffer_ptrs_dev
        self.state = torch.zeros(1, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group)

    def _call(self, src, mode, row_offset, dst):
        import ctypes
        _lib.call("vq2_peer_exchange", _lib.ptr(src), src.numel() * src.element_size(), mode, row_offset,
                  ctypes.c_void_p(self.peers_dev), self.rank, self.world, self.max_bytes, _lib.ptr(self.state),
                  _lib.ptr(self.err), int(self.max_polls), _lib.ptr(dst), _lib.stream_ptr(src.device))
        return dst

    def gather(self, src):
        """[world, *src.shape]: every rank's src, in rank order."""
        src = src.contiguous()
        return self._call(src, 0, 0, torch.empty(self.world, *src.shape, dtype=src.dtype, device=src.device))

    def max_keys(self, keys, row_offset):
        """Elementwise maximum over ranks of greedy keys (int64 [n]) rebased by row_offset."""
        keys = keys.contiguous()
        return self._call(keys, 1, int(row_offset), torch.empty_like(keys))

    def check(self):
        if int(self.err.item()):
            raise RuntimeError(f"peer exchange timed out (status {int(self.err.item()):#x})")


def shard_rows(vocab, world, rank):
    """[lo, hi) rows of rank `rank`: contiguous, the first vocab % world ranks one row more."""
    base, extra = divmod(vocab, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class ShardedLMHead:
    """Greedy lm_head over this rank's rows ``[lo, hi)`` (``shard``: a PackedLinear of those rows,
    built with the full matrix's rotation tag so every shard rotates its input the same way)."""

    def __init__(self, shard, lo, vocab, exchange):
        self.shard, self.lo, self.vocab, self.ex = shard, lo, vocab, exchange

    def greedy(self, h):
        """h: this rank's hidden rows [M, H] -> int64 [world, M]: the next token of every rank's
        rows (ties to the smaller vocabulary row, as torch.argmax)."""
        allh = self.ex.gather(h.reshape(-1, h.shape[-1]))          # [world, M, H]
        M = allh.shape[1]
        cb0, cb1 = self.shard.codebooks()
        keys = kernels.gemv_argmax(allh.reshape(-1, allh.shape[-1]), self.shard.mat(), cb0, cb1, rot=self.shard.rot,
                                   keys=True)
        best = self.ex.max_keys(keys, self.lo)
        return (0xFFFFFFFF - (best & 0xFFFFFFFF)).reshape(self.ex.world, M)
