"""The 35B-A3B-shaped MoE decode stack: a random-init transformers Qwen3.5-MoE text model whose
linears are VQ 2 bpw and whose sparse MoE blocks run on this library's kernels.

Mirrors reference ``build_full_vq2_model`` (vq2/load_and_test_full_35b.py:124-223): the HF model
is built without materialising its dense weights, then
  * every nn.Linear of the attention and Gated-DeltaNet blocks becomes a PackedLinear (2 bpw,
    seeded random indices and ~0.02 row scales: no trained weights are available);
  * every Qwen3_5MoeSparseMoeBlock becomes a VQMoEBlock: the dense bf16 router (kept dense, as
    vq2/quantize_35b.py:139 does), the shared expert's sigmoid gate, and the 256 routed experts +
    the shared expert as expert records in HBM, one vq2_moe_layer call per layer (or, with a
    process group, the expert-parallel block: experts split across the ranks, the rank sum over
    NVLink peer memory);
  * embed_tokens becomes a PackedEmbedding and lm_head a PackedLinear (untied, as the 35B-A3B
    config has it);
  * norms, the DeltaNet convolution / decay parameters and the rotary tables stay the reference's
    PyTorch modules, initialised here.
"""
import math

import torch
import torch.nn as nn

from . import ep, moe, runtime, synth, vq


class VQMoEBlock(nn.Module):
    """Drop-in for Qwen3_5MoeSparseMoeBlock (modeling_qwen3_5_moe.py:773-791): forward(hidden
    [B, S, H]) -> [B, S, H]; router logits by the dense-router kernel, then one MoE layer call."""

    def __init__(self, router_weight, shared_gate, pool, cb16, num_experts, top_k, device, group=None,
                 peer_ctx=None, max_tokens=64):
        super().__init__()
        self.router_weight = router_weight
        self.shared_gate = shared_gate
        self.top_k = top_k
        self.rot_in = vq.get_rot("moe_expert_2048", pool.dims[1] * 8, device)
        self.rot_mid = vq.get_rot("moe_expert_512", pool.dims[0] // 2, device)
        if group is None:
            self.ep = None
            self.pool, self.cb16, self.num_experts = pool, cb16, num_experts
        else:
            self.ep = ep.ExpertParallelMoEBlock(pool, cb16, num_experts, self.rot_in, self.rot_mid, group=group,
                                                shared_gate=shared_gate, top_k=top_k, peer_ctx=peer_ctx,
                                                max_tokens=max_tokens)

    def forward(self, hidden_states):
        lead = hidden_states.shape[:-1]
        h = hidden_states.reshape(-1, hidden_states.shape[-1])
        logits = moe.router_logits_fn(h, self.router_weight)
        if self.ep is not None:
            y = self.ep(h, logits)
        else:
            y = moe.moe_layer(h, logits, self.pool, self.cb16, self.rot_in, self.rot_mid, self.top_k,
                              shared_gate=self.shared_gate, hi=self.num_experts)
        return y.reshape(*lead, y.shape[-1])


def _packed(out, n, tag, cbs, device, gen):
    idx = torch.randint(-32768, 32768, (out, n // 8), generator=gen, device=device, dtype=torch.int16)
    scale = (0.02 * torch.exp(0.1 * torch.randn(out, generator=gen, device=device))).half()
    return runtime.PackedLinear((out, n), (16,), tag, [idx], scale, cbs, device)


def _expert_pool(rows, device, gen, dims):
    pool = moe.ExpertRecordPool(rows, device, **dims)
    w16 = pool.raw.view(torch.int16)
    w16.copy_(torch.randint(-32768, 32768, w16.shape, generator=gen, device=device, dtype=torch.int16))
    pool.gu_scale.copy_(0.02 * torch.exp(0.1 * torch.randn(pool.gu_scale.shape, generator=gen, device=device)))
    pool.dn_scale.copy_(0.02 * torch.exp(0.1 * torch.randn(pool.dn_scale.shape, generator=gen, device=device)))
    return pool


@torch.no_grad()
def build_vq2_moe_model(config=None, device="cuda", seed=0, group=None, max_tokens=64):
    """Qwen3_5MoeForCausalLM (text) with VQ weights on ``device``; ``config`` defaults to the
    35B-A3B shape (Qwen3_5MoeTextConfig defaults: 40 layers, hidden 2048, 256 experts + 1 shared,
    top-8, expert inter 512). With ``group`` the experts of every layer are split across its
    ranks (every rank builds the same dense parts from the same seed)."""
    import torch.distributed as dist  # noqa: F401  (group sizes)
    from transformers import Qwen3_5MoeForCausalLM, Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    config = config or Qwen3_5MoeTextConfig()
    device = torch.device(device)
    with torch.device("meta"):
        model = Qwen3_5MoeForCausalLM(config)
    # drop the heavy meta modules before materialising the rest
    linears = []
    for name, mod in model.named_modules():
        if isinstance(mod, nn.Linear) and ".mlp." not in name and name != "lm_head":
            linears.append((name, mod.out_features, mod.in_features))
    for name, _, _ in linears:
        runtime._set_module(model, name, nn.Identity())
    for layer in model.model.layers:
        layer.mlp = nn.Identity()
    model.model.embed_tokens = nn.Identity()
    model.lm_head = nn.Identity()
    model.to_empty(device=device)
    gen = torch.Generator(device=device).manual_seed(seed)
    for name, p in model.named_parameters():   # norms, DeltaNet conv / decay parameters
        if name.endswith("A_log"):
            p.copy_(torch.log(torch.rand(p.shape, generator=gen, device=device) * 16 + 1e-3))
        elif name.endswith("dt_bias"):
            p.fill_(1.0)
        elif "conv1d" in name:
            p.copy_(torch.randn(p.shape, generator=gen, device=device) / math.sqrt(p.shape[-1]))
        else:  # RMSNorm weights (applied as 1 + w) and any other vector
            p.zero_()
    model.model.rotary_emb = M.Qwen3_5MoeTextRotaryEmbedding(config, device=device)
    model.to(torch.bfloat16)
    cbs = {k: torch.from_numpy(v).to(device) for k, v in synth.random_codebooks(1).items()}
    for name, out, n in linears:
        runtime._set_module(model, name, _packed(out, n, name.split(".")[-1], cbs, device, gen))
    H, E, K = config.hidden_size, config.num_experts, config.num_experts_per_tok
    inter = config.moe_intermediate_size
    if config.shared_expert_intermediate_size != inter:
        raise ValueError("the shared expert is stored as one more expert record: its width must match")
    dims = dict(gu_rows=2 * inter, gu_cols=H // 8, dn_rows=H, dn_cols=inter // 8)
    world, rank = (dist.get_world_size(group), dist.get_rank(group)) if group is not None else (1, 0)
    peer_ctx = None
    if group is not None and world > 1:
        try:
            peer_ctx = ep.PeerReduceContext(group, device, max_tokens=max_tokens, hidden=H)
        except Exception:
            peer_ctx = None
    for layer in model.model.layers:
        router = (0.02 * torch.randn(E, H, generator=gen, device=device)).to(torch.bfloat16)
        gate = 0.02 * torch.randn(H, generator=gen, device=device)
        full = _expert_pool(E + 1, device, gen, dims)      # the same experts on every rank (same seed)
        if group is not None and world > 1:
            lo, hi = ep.partition(E, world, rank)
            pool = moe.ExpertRecordPool(hi - lo + 1, device, **dims)
            pool.raw[: hi - lo].copy_(full.raw[lo:hi])
            pool.raw[hi - lo].copy_(full.raw[E])
            del full
            layer.mlp = VQMoEBlock(router, gate, pool, cbs["16"], E, K, device, group=group, peer_ctx=peer_ctx,
                                   max_tokens=max_tokens)
        else:
            layer.mlp = VQMoEBlock(router, gate, full, cbs["16"], E, K, device)
    emb = _packed(config.vocab_size, H, "embed", cbs, device, gen)
    model.model.embed_tokens = runtime.PackedEmbedding(emb)
    model.lm_head = _packed(config.vocab_size, H, "lm_head", cbs, device, gen)
    model.eval()
    return model


@torch.no_grad()
def decode(model, batch, prompt_len=4, steps=8, warmup=2, seed=0):
    """Greedy decode of ``batch`` sequences: prefill ``prompt_len`` tokens, then ``warmup`` +
    ``steps`` one-token steps through the HF cache; returns (seconds per timed step, final ids)."""
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev).manual_seed(seed)
    ids = torch.randint(0, model.config.vocab_size, (batch, prompt_len), generator=g, device=dev)
    out = model(input_ids=ids, use_cache=True)
    past = out.past_key_values
    nxt = out.logits[:, -1].argmax(-1, keepdim=True)
    for _ in range(warmup):
        out = model(input_ids=nxt, past_key_values=past, use_cache=True)
        past = out.past_key_values
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        out = model(input_ids=nxt, past_key_values=past, use_cache=True)
        past = out.past_key_values
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / steps, nxt
