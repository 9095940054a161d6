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
4. one all_reduce(SUM) of the partial over the group; every rank ends with the full output.

At T = 1 the whole exchange is one all_reduce of 8 KB per layer (the hidden state is already
replicated, so no dispatch collective is needed); the reference has no multi-GPU path at all.
"""
import torch
import torch.distributed as dist

from . import moe


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
                 ffn=None, router=None):
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
        part = self.ffn(hidden_states.reshape(T, -1), loc, lw, loc.shape[1])
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        return part.to(hidden_states.dtype)
