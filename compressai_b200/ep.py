"""Expert parallelism: the routed experts of every MoE layer are partitioned across the ranks of
a process group (one process per GPU, NCCL over NVLink/NVSwitch).

Partition: rank r of N owns experts [r*E/N, (r+1)*E/N) (contiguous, E % N == 0) in its own
record pool, followed by a copy of the shared expert (every rank holds it); the router and the
shared expert's gate are replicated, so every rank computes identical routing from the same
hidden states (the router kernel is deterministic). Per layer and batch of T tokens, one
vq2_moe_layer_ep call:

1. route (replicated) -> local problems: pool row e - r*E/N where expert e is local, -1 (zero
   contribution) elsewhere; the shared expert's problem of token t runs on rank t % N, so its
   work is spread over the ranks instead of doubling one rank's load;
2. gate_up and down GEMVs over the local problems;
3. the sum over ranks. Default (``reduce="peer"``): the combine kernel itself sums the ranks'
   partials over NVLink peer memory (each CTA publishes its column slice of the partial into a
   symmetric buffer, signals the peers, waits for theirs and adds all slices in rank order) --
   one kernel instead of combine + NCCL all_reduce + cast, graph capturable, identical output
   on every rank. ``reduce="nccl"``: fp32 partial then one NCCL all_reduce(SUM) (the baseline,
   also used when symmetric memory is unavailable).

At T = 1 the whole exchange is 8 KB per rank per layer (the hidden state is already replicated,
so no dispatch collective is needed); the reference has no multi-GPU path at all.
"""
import torch
import torch.distributed as dist

from . import _lib, moe


class PeerReduceContext:
    """Symmetric buffer (torch symmetric memory, peer-mapped on every rank of ``group``) plus the
    local epochs and status word of vq2_moe_expert_ffn_ep; one per (group, device), shared by
    all layers (their calls are ordered on one stream)."""

    def __init__(self, group, device, max_tokens, hidden, max_polls=0):
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.hidden = max_tokens, hidden
        self.max_polls = max_polls   # polls of a peer's flag before a wait gives up (0: about a second)
        lib = _lib.load()
        nbytes = lib.vq2_moe_peer_buffer_bytes(max_tokens, hidden, self.world)
        if nbytes < 0:
            raise ValueError("bad peer buffer size")
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, name)
        self.peers_dev = self.handle.buffer_ptrs_dev
        # sequence number, finished CTAs (peer combine), router arrivals, spare
        self.epochs = torch.zeros(4, dtype=torch.int32, device=device)
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


def local_problems(ids, weights, lo, hi, shared_id=None, shared_w=None, rank=0, world=1):
    """Map global expert ids [T, k] to local pool rows (-1 for remote experts); with
    ``shared_id``, append the shared expert as one more problem per token, local on rank
    t % world for token t (the router kernel's rule, restated for host-side stand-ins)."""
    loc = torch.where((ids >= lo) & (ids < hi), ids - lo, torch.full_like(ids, -1)).to(torch.int32)
    w = weights.float()
    if shared_id is not None:
        T = ids.shape[0]
        t = torch.arange(T, device=ids.device)
        sh = torch.where(t % world == rank, torch.full_like(t, shared_id), torch.full_like(t, -1)).to(torch.int32)
        loc = torch.cat([loc, sh[:, None]], 1)
        w = torch.cat([w, shared_w.reshape(T, 1).float()], 1)
    return loc.contiguous(), w.contiguous()


class ExpertParallelMoEBlock(torch.nn.Module):
    """Sparse MoE block (router + routed experts + shared expert) with the routed experts split
    across the ranks of ``group``. ``pool`` holds this rank's E/N experts (+ the shared expert as
    its last row when ``shared_gate`` is given, on every rank). ``ffn`` computes one partial from
    local problems; when given (a host-side stand-in for CPU ranks) the block routes with
    ``router`` and maps problems with ``local_problems``; by default the whole layer is one
    vq2_moe_layer(_ep) call."""

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
        self.shared_row = (self.hi - self.lo) if shared_gate is not None else None
        self.ffn = ffn
        self.router = router or moe.route
        self.peer = None
        if reduce == "peer" and ffn is None and self.world > 1 and pool.raw.is_cuda:
            try:
                self.peer = peer_ctx or PeerReduceContext(group, pool.raw.device, max_tokens, pool.dims[1] * 8)
            except Exception as exc:  # no symmetric memory on this system: NCCL all_reduce
                self.peer_error = repr(exc)
        self.reduce_kind = "peer" if self.peer is not None else "nccl"

    def forward(self, hidden_states, router_logits):
        T = hidden_states.shape[0]
        h = hidden_states.reshape(T, -1)
        if self.ffn is not None:  # host-side stand-in (CPU ranks): route, map, partial, all_reduce
            if self.shared_gate is not None:
                ids, w, sw = self.router(router_logits, self.top_k, h, self.shared_gate)
            else:
                (ids, w), sw = self.router(router_logits, self.top_k), None
            loc, lw = local_problems(ids, w, self.lo, self.hi, self.shared_row, sw, self.rank, self.world)
            part = self.ffn(h, loc, lw, loc.shape[1])
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            return part.to(hidden_states.dtype)
        if self.peer is not None and T <= self.peer.max_tokens:
            return moe.moe_layer(h, router_logits, self.pool, self.cb16, self.rot_in, self.rot_mid, self.top_k,
                                 shared_gate=self.shared_gate, lo=self.lo, hi=self.hi, rank=self.rank,
                                 world=self.world, peer=self.peer)
        part = moe.moe_layer(h, router_logits, self.pool, self.cb16, self.rot_in, self.rot_mid, self.top_k,
                             shared_gate=self.shared_gate, lo=self.lo, hi=self.hi, rank=self.rank, world=self.world,
                             out_dtype=torch.float32)
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        return part.to(hidden_states.dtype)
