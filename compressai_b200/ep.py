"""Expert parallelism: the routed experts of every MoE layer are partitioned across the ranks of
a process group (one process per GPU, NCCL over NVLink/NVSwitch).

Partition: rank r of N owns experts [r*E/N, (r+1)*E/N) (contiguous, E % N == 0) in its own
record pool; the router and the shared expert's gate are replicated, so every rank computes
identical routing from the same hidden states (the ``route`` kernel is deterministic).
Per layer and batch of T tokens:

1. route (replicated) -> ids [T, k], weights [T, k];
2. local problems: id - r*E/N where the expert is local, -1 (zero contribution) elsewhere;
   the shared expert (when present) is one more problem on rank 0 only;
3. expert FFN over the local problems into an fp32 partial [T, H] (vq2_moe_expert_ffn);
4. the sum over ranks. Default (``reduce="peer"``): the combine kernel itself sums the ranks'
   partials over NVLink peer memory (vq2_moe_expert_ffn_ep: each CTA publishes its column slice
   of the partial into a symmetric buffer, signals the peers, waits for theirs and adds all
   slices in rank order) -- one kernel instead of combine + NCCL all_reduce + cast, graph
   capturable, identical output on every rank. ``reduce="nccl"``: fp32 partial then one NCCL
   all_reduce(SUM) (the baseline, also used when symmetric memory is unavailable).

At T = 1 the whole exchange is 8 KB per rank per layer (the hidden state is already replicated,
so no dispatch collective is needed); the reference has no multi-GPU path at all.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib, moe


class PeerReduceContext:
    """Symmetric buffer (torch symmetric memory, peer-mapped on every rank of ``group``) plus the
    local epochs and status word of vq2_moe_expert_ffn_ep; one per (group, device), shared by
    all layers (their calls are ordered on one stream)."""

    def __init__(self, group, device, max_tokens, hidden):
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.hidden = max_tokens, hidden
        lib = _lib.load()
        nbytes = lib.vq2_moe_peer_buffer_bytes(max_tokens, hidden, self.world)
        if nbytes < 0:
            raise ValueError("bad peer buffer size")
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, name)
        self.peers_dev = self.handle.buffer_ptrs_dev
        self.epochs = torch.zeros(2, dtype=torch.int32, device=device)   # sequence number, finished CTAs
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every rank's flags are zero before any rank writes into them

    def check(self):
        """Raise if a wait for a peer gave up."""
        if int(self.err.item()):
            raise RuntimeError(f"peer reduction timed out (status {int(self.err.item()):#x})")


def partition(num_experts, world, rank):
    """[lo, hi) experts owned by `rank`."""
    if num_experts % world != 0:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


def local_problems(ids, weights, lo, hi, shared_id=None, shared_w=None):
    """Map global expert ids [T, k] to local pool rows (-1 for remote experts); append the shared
    expert as one more problem per token when ``shared_id`` is given (rank 0)."""
    loc = torch.where((ids >= lo) & (ids < hi), ids - lo, torch.full_like(ids, -1)).to(torch.int32)
    w = weights.float()
    if shared_id is not None:
        T = ids.shape[0]
        loc = torch.cat([loc, torch.full((T, 1), shared_id, dtype=torch.int32, device=ids.device)], 1)
        w = torch.cat([w, shared_w.reshape(T, 1).float()], 1)
    return loc.contiguous(), w.contiguous()


class ExpertParallelMoEBlock(torch.nn.Module):
    """Sparse MoE block (router + routed experts + shared expert) with the routed experts split
    across the ranks of ``group``. ``pool`` holds this rank's E/N experts (+ the shared expert
    as its last row on rank 0). ``ffn`` computes one partial and defaults to the CUDA expert FFN;
    it is a parameter so the host logic can be exercised on CPU ranks with a stand-in."""

    def __init__(self, pool, cb16, num_experts, rot_in, rot_mid, group=None, shared_gate=None, top_k=8,
                 ffn=None, router=None, reduce="peer", peer_ctx=None, max_tokens=64):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.lo, self.hi = partition(num_experts, self.world, self.rank)
        self.pool, self.cb16 = pool, cb16
        self.num_experts, self.top_k = num_experts, top_k
        self.rot_in, self.rot_mid = rot_in, rot_mid
        self.shared_gate = shared_gate
        self.shared_row = (self.hi - self.lo) if (shared_gate is not None and self.rank == 0) else None
        self.ffn = ffn or self._cuda_ffn
        self.router = router or moe.route
        self.peer = None
        if reduce == "peer" and ffn is None and self.world > 1 and pool.raw.is_cuda:
            try:
                self.peer = peer_ctx or PeerReduceContext(group, pool.raw.device, max_tokens, pool.dims[1] * 8)
            except Exception as exc:  # no symmetric memory on this system: NCCL all_reduce
                self.peer_error = repr(exc)
        self.reduce_kind = "peer" if self.peer is not None else "nccl"

    def _cuda_ffn(self, h, ids, w, k):
        return moe.expert_ffn(h, ids.reshape(-1), w, self.pool, self.cb16, self.rot_in, self.rot_mid, k,
                              out_dtype=torch.float32)

    def forward(self, hidden_states, router_logits):
        T = hidden_states.shape[0]
        if self.shared_gate is not None:
            ids, w, sw = self.router(router_logits, self.top_k, hidden_states, self.shared_gate)
        else:
            (ids, w), sw = self.router(router_logits, self.top_k), None
        loc, lw = local_problems(ids, w, self.lo, self.hi, self.shared_row, sw)
        if self.peer is not None and T <= self.peer.max_tokens:
            return self._peer_ffn(hidden_states.reshape(T, -1).contiguous(), loc, lw, loc.shape[1])
        part = self.ffn(hidden_states.reshape(T, -1), loc, lw, loc.shape[1])
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        return part.to(hidden_states.dtype)

    def _peer_ffn(self, h, loc, lw, k):
        T = h.shape[0]
        gr, gc, dr, dc = self.pool.dims
        lib = _lib.load()
        ws_bytes = lib.vq2_moe_expert_ffn_workspace(T, k, gr, dr)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=h.device)
        out = torch.empty(T, gc * 8, dtype=h.dtype, device=h.device)
        pc = self.peer
        ri, rm = self.rot_in, self.rot_mid
        _lib.call("vq2_moe_expert_ffn_ep", _lib.ptr(h), _lib.dtype_code(h), T, k, _lib.ptr(loc), _lib.ptr(lw),
                  _lib.ptr(self.pool.raw), self.pool.E, gr, gc, dr, dc, _lib.ptr(self.cb16), _lib.dtype_code(self.cb16),
                  _lib.ptr(ri.perm), _lib.ptr(ri.sign), ri.hb, float(ri.scale), _lib.ptr(rm.perm), _lib.ptr(rm.sign),
                  rm.hb, float(rm.scale), _lib.ptr(ws), ws_bytes, ctypes.c_void_p(pc.peers_dev), pc.rank, pc.world,
                  pc.max_tokens, _lib.ptr(pc.epochs), _lib.ptr(pc.err), _lib.ptr(out), _lib.dtype_code(out),
                  _lib.stream_ptr(h.device))
        return out
