"""Runtime pieces around the GEMV on the GPU: fixed-width stream unpack, container read onto the
device, row decode (PackedLinear.weight_rows, PackedEmbedding) against the fp64 oracle, and
load_packed end to end -- a small transformers model whose linears and tied embedding come
from a .vq2r container runs through PackedLinear / PackedEmbedding / PackedLMHead and matches
the same model with the oracle's dequantized weights."""
import os

import numpy as np
import pytest
import torch

from compressai_b200 import runtime, synth
from oracle import vq2_oracle as O
from tests.conftest import GOLDEN, golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.mark.parametrize("bits", [4, 8, 12, 16])
@pytest.mark.parametrize("n", [1, 2, 7, 1000, 1001])
def test_unpack_fixed_gpu_matches_reference(bits, n):
    d = golden("fixed.npz")
    out = runtime.unpack_fixed_gpu(d[f"b{bits}_n{n}_buf"], bits, n, DEV).cpu().numpy()
    ref = d[f"b{bits}_n{n}_out"]
    got = out.view(np.uint16).astype(np.int64) if bits > 8 else out.astype(np.int64)
    assert np.array_equal(got, ref)


def test_read_container_unpacks_on_the_gpu():
    d = golden("fixed.npz")
    C = runtime.read_container(os.path.join(GOLDEN, "vq2_small.pt"), device=DEV)
    for nm in C["names"]:
        for i, t in enumerate(C["idx"][nm]):
            assert t.is_cuda
            assert np.array_equal(t.cpu().numpy(), d[f"ctr_{nm}_{i}"]), (nm, i)


@pytest.fixture(scope="module")
def cbs():
    return synth.random_codebooks(6)


@pytest.mark.parametrize("bits", [(16,), (16, 8)])
@pytest.mark.parametrize("n", [256, 2048, 6144])
def test_weight_rows_and_embedding_vs_oracle(cbs, bits, n):
    out = 700
    idx, scale = synth.random_matrix(n + len(bits), out, n, bits)
    cbd = {k: torch.from_numpy(v).to(DEV) for k, v in cbs.items()}
    lin = runtime.PackedLinear((out, n), bits, "embed_test", [torch.from_numpy(a) for a in idx],
                               torch.from_numpy(scale), cbd, DEV)
    q = lin.weight_rows(100, 260).float().cpu().numpy()
    ref_q = O.rotated_rows([a[100:260] for a in idx], bits, cbs, scale[100:260])
    assert rel_err(q, ref_q) < 2e-3   # fp16 result
    ids = torch.tensor([[5, 699, 5], [0, 123, 600]], device=DEV)
    emb32 = runtime.PackedEmbedding(lin, out_dtype=torch.float32)(ids).cpu().numpy()
    emb = runtime.PackedEmbedding(lin)(ids)
    assert emb.dtype == torch.bfloat16 and emb.shape == (2, 3, n)
    flat = ids.cpu().numpy().reshape(-1)
    W = O.dequant([a[flat] for a in idx], bits, cbs, scale[flat], *O.rot_params("embed_test", n))
    assert rel_err(emb32.reshape(-1, n), W) < 1e-5
    assert rel_err(emb.float().cpu().numpy().reshape(-1, n), W) < 4e-3


def test_embedding_out_of_range_ids_give_zero_rows(cbs):
    from compressai_b200 import _lib
    idx, scale = synth.random_matrix(3, 64, 256)
    cbd = {k: torch.from_numpy(v).to(DEV) for k, v in cbs.items()}
    lin = runtime.PackedLinear((64, 256), (16,), "t", [torch.from_numpy(idx[0])], torch.from_numpy(scale), cbd, DEV)
    ids = torch.tensor([3, 64, -1], device=DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full((3, 256), 7.0, device=DEV)
    cb0, _ = lin.codebooks()
    _lib.call("vq2_embed_rows", _lib.ptr(ids), 3, 64, _lib.ptr(lin.idx0), None, _lib.ptr(cb0), None,
              _lib.ptr(lin.scale), _lib.VQ2_F16, 256, _lib.ptr(lin.rot.perm), _lib.ptr(lin.rot.sign), lin.rot.hb,
              float(lin.rot.scale), _lib.ptr(out), _lib.VQ2_F32, _lib.ptr(bad), _lib.stream_ptr(DEV))
    assert int(bad.item()) == 1
    assert not out[1:].abs().any() and out[0].abs().sum() > 0


def test_load_packed_small_model_matches_dequantized_model(cbs, tmp_path):
    """load_packed on a .vq2r container of a small Qwen3 (2 layers, hidden 256, tied embedding):
    logits of the packed model (PackedLinear everywhere, PackedEmbedding, tied PackedLMHead) match
    the same architecture in fp32 with W = Rot.inv(Q) from the oracle for every matrix."""
    from transformers import AutoModelForCausalLM, Qwen3Config
    cfg = Qwen3Config(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=512, tie_word_embeddings=True,
                      max_position_embeddings=64)
    torch.manual_seed(0)
    ref = AutoModelForCausalLM.from_config(cfg).float().eval()
    rng = np.random.default_rng(21)
    names, meta, idx, scales, dense = [], {}, {}, {}, {}
    params = dict(ref.named_parameters())
    for pn, p in params.items():
        if p.dim() != 2 or pn == "lm_head.weight":
            continue
        nm = pn[:-len(".weight")]
        out, n = p.shape
        bits = (16, 8) if nm.endswith("down_proj") else (16,)
        tag = "embed" if nm.endswith("embed_tokens") else nm.split(".")[-1]
        ia = [rng.integers(0, 1 << 16, (out, n // 8)).astype(np.uint16).view(np.int16)]
        if len(bits) > 1:
            ia.append(rng.integers(0, 256, (out, n // 8)).astype(np.uint8))
        sc = (0.02 * np.exp(0.1 * rng.standard_normal(out))).astype(np.float16)
        W = O.dequant(ia, bits, cbs, sc, *O.rot_params(tag, n))
        with torch.no_grad():
            p.copy_(torch.from_numpy(W))
        names.append(nm)
        meta[nm] = {"shape": [out, n], "cfg": list(bits), "tag": tag}
        idx[nm] = [torch.from_numpy(a) for a in ia]
        scales[nm] = torch.from_numpy(sc)
    for pn, p in params.items():
        if p.dim() == 1:
            dense[pn] = p.detach().clone()
    C = {"format": "vq2r", "names": names, "meta": meta, "idx": idx, "scales": scales,
         "codebooks": {k: torch.from_numpy(v) for k, v in cbs.items()},
         "codebooks_embed": {k: torch.from_numpy(v) for k, v in cbs.items()}, "dense": dense}
    path = str(tmp_path / "small.vq2r")
    torch.save(C, path)
    model = runtime.load_packed(path, DEV, config=cfg)
    assert isinstance(model.model.embed_tokens, runtime.PackedEmbedding)
    assert isinstance(model.lm_head, runtime.PackedLMHead)
    assert isinstance(model.model.layers[0].self_attn.q_proj, runtime.PackedLinear)
    ids = torch.from_numpy(rng.integers(0, 512, (2, 6))).to(DEV)
    with torch.no_grad():
        got = model(ids).logits.float().cpu().numpy()
        want = ref(ids.cpu()).logits.numpy()
    assert rel_err(got, want) < 5e-2   # bf16 activations between the layers
    assert (got.argmax(-1) == want.argmax(-1)).mean() >= 0.9
