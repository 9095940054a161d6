"""The 35B-A3B-shaped decode stack (compressai_b200.stack) on a small config: the dense router
kernel against torch fp32, the VQ MoE block against the one-call layer fed torch-computed logits,
and greedy decode through the transformers Qwen3.5-MoE modules (Gated DeltaNet + full attention
layers, HF cache) with every linear VQ-packed: finite and deterministic."""
import pytest
import torch

from compressai_b200 import moe, stack

pytestmark = pytest.mark.gpu
DEV = "cuda"


def small_config():
    from transformers import Qwen3_5MoeTextConfig
    return Qwen3_5MoeTextConfig(hidden_size=512, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                                head_dim=128, linear_key_head_dim=64, linear_value_head_dim=64,
                                linear_num_key_heads=4, linear_num_value_heads=8, moe_intermediate_size=256,
                                shared_expert_intermediate_size=256, num_experts=32, num_experts_per_tok=4,
                                vocab_size=1024)


@pytest.mark.parametrize("T", [1, 5, 64])
@pytest.mark.parametrize("hdt", [torch.bfloat16, torch.float16, torch.float32])
def test_router_logits_kernel(T, hdt):
    h = torch.randn(T, 2048, device=DEV).to(hdt)
    W = (0.02 * torch.randn(256, 2048, device=DEV)).to(torch.bfloat16)
    got = moe.router_logits_fn(h, W)
    want = h.float() @ W.float().t()
    assert ((got - want).abs().max() / want.abs().max()).item() < 1e-5


def test_vq_moe_block_matches_layer_with_reference_logits():
    torch.manual_seed(0)
    model = stack.build_vq2_moe_model(small_config(), DEV, seed=3)
    blk = model.model.layers[0].mlp
    h = torch.randn(2, 3, 512, device=DEV).to(torch.bfloat16)
    y = blk(h).float()
    logits = h.reshape(-1, 512).float() @ blk.router_weight.float().t()
    want = moe.moe_layer(h.reshape(-1, 512), logits, blk.pool, blk.cb16, blk.rot_in, blk.rot_mid, blk.top_k,
                         shared_gate=blk.shared_gate, hi=blk.num_experts).float().reshape(2, 3, 512)
    assert ((y - want).abs().max() / want.abs().max()).item() < 1e-2   # bf16 outputs


def test_small_stack_greedy_decode_is_finite_and_deterministic():
    model = stack.build_vq2_moe_model(small_config(), DEV, seed=4)
    t1, ids1 = stack.decode(model, batch=3, prompt_len=5, steps=3, warmup=1, seed=9)
    t2, ids2 = stack.decode(model, batch=3, prompt_len=5, steps=3, warmup=1, seed=9)
    assert t1 > 0 and torch.equal(ids1, ids2)
    out = model(input_ids=ids1, use_cache=False)
    assert torch.isfinite(out.logits.float()).all()
