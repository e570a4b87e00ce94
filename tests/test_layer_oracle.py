"""CPU tests of the layer-level oracle.

1. lema_b200's LlamaBlock with bf16 nn.Linear projections computes the same
   thing as HF LlamaDecoderLayer driven the way the reference adapter drives it
   (src/lema/adapters/_llama.py:183-252).
2. LlamaBlock with the oracle's W8A8 linears swapped in (eager attention, CPU)
   reproduces the golden fixture generated from the reference's own Python
   path (tests/golden/make_golden_layer.py) bit for bit: outputs, input
   gradient and LoRA gradients.
"""
import pytest
import torch
from transformers.models.llama.modeling_llama import LlamaConfig, LlamaDecoderLayer

from lema_b200.llama import LlamaBlock, LlamaShape, rope_cos_sin
from oracle.oracle import torch_bf16_to_bits
from oracle.torch_ref import swap_linears

from layer_fixture import bf16, block_from_fixture, load


def test_block_matches_hf_decoder_layer_fp32():
    shape = LlamaShape(hidden=64, heads=4, kv_heads=2, intermediate=160, vocab=100, layers=1)
    cfg = LlamaConfig(hidden_size=64, num_attention_heads=4, num_key_value_heads=2,
                      intermediate_size=160, rms_norm_eps=1e-5, rope_theta=10000.0,
                      max_position_embeddings=64)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    hf = LlamaDecoderLayer(cfg, layer_idx=0).float()
    for p in hf.parameters():
        torch.nn.init.normal_(p, std=0.05)
    mine = LlamaBlock(shape, quantized=False, dtype=torch.float32)
    mine.self_attn.attn_impl = "eager"
    mine.load_state_dict(hf.state_dict())
    x = torch.randn(2, 24, 64)
    pos = torch.arange(24)[None].expand(2, -1)
    cos, sin = rope_cos_sin(shape, 24, "cpu", torch.float32)
    mask = torch.full((24, 24), float("-inf")).triu(1)[None, None].expand(2, 1, 24, 24)
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    hf_cos, hf_sin = LlamaRotaryEmbedding(cfg)(x, pos)
    assert torch.allclose(hf_cos[0], cos[0]) and torch.allclose(hf_sin[0], sin[0])
    ref = hf(x, attention_mask=mask, position_ids=pos, position_embeddings=(hf_cos, hf_sin))
    ref = ref[0] if isinstance(ref, tuple) else ref
    out = mine(x, cos, sin)
    assert torch.allclose(out, ref, atol=1e-6, rtol=1e-5), (out - ref).abs().max()


def test_oracle_block_reproduces_reference_fixture():
    d, shape, rank, alpha = load()
    blk = block_from_fixture(d, shape, rank, alpha, "cpu", quantized=False)
    blk.self_attn.attn_impl = "eager"
    swap_linears(blk)
    x = bf16(d["x"]).clone().requires_grad_(True)
    cos, sin = rope_cos_sin(shape, x.shape[1], "cpu", torch.bfloat16)
    y = blk(x, cos, sin)
    y.backward(bf16(d["dy"]))
    assert (torch_bf16_to_bits(y) == d["y"]).all()
    assert (torch_bf16_to_bits(x.grad) == d["dx"]).all()
    for proj in ("q_proj", "v_proj"):
        m = blk.projection(proj)
        assert (torch_bf16_to_bits(m.lora_A.grad) == d[f"grad/self_attn.{proj}.lora_A"]).all()
        assert (torch_bf16_to_bits(m.lora_B.grad) == d[f"grad/self_attn.{proj}.lora_B"]).all()


def test_chunked_attention_equals_full_attention():
    """Query-chunked causal attention (the reference's chunked_attention shape of
    computation, used for long sequences) equals full causal attention."""
    shape = LlamaShape(hidden=64, heads=4, kv_heads=2, intermediate=160, vocab=100, layers=1)
    torch.manual_seed(1)
    blk = LlamaBlock(shape, quantized=False, dtype=torch.float32)
    for p in blk.parameters():
        torch.nn.init.normal_(p, std=0.05)
    x = torch.randn(2, 130, 64)
    cos, sin = rope_cos_sin(shape, 130, "cpu", torch.float32)
    full = blk(x, cos, sin)
    blk.self_attn.attn_chunk = 32
    chunked = blk(x, cos, sin)
    assert torch.allclose(full, chunked, atol=1e-6, rtol=1e-5)


def test_oracle_model_reproduces_reference_trainer_step():
    """tests/golden/llama_model_w8a8.npz was written by tests/golden/make_golden_model.py
    from one LemaTrainer.train_step of the reference (2 Llama blocks with the oracle's
    W8A8 linears, LoRA r4 on q/v, bf16, CPU). This build's embedding, blocks and head
    with the same weights give the same logits, loss and LoRA gradients."""
    import numpy as np
    import torch.nn.functional as F
    from pathlib import Path

    from lema_b200.llama import LlamaHead, apply_lora
    d = np.load(Path(__file__).parent / "golden" / "llama_model_w8a8.npz")
    hidden, heads, inter, layers, vocab, seq, batch, rank, alpha = (int(v) for v in d["meta"])
    shape = LlamaShape(hidden=hidden, heads=heads, kv_heads=heads, intermediate=inter,
                       vocab=vocab, layers=layers)
    ck = {k[len("ckpt/"):]: bf16(d[k]) for k in d.files if k.startswith("ckpt/")}
    embed = torch.nn.Embedding(vocab, hidden, dtype=torch.bfloat16)
    embed.weight.data.copy_(ck["model.embed_tokens.weight"])
    head = LlamaHead(shape)
    head.norm.weight.data.copy_(ck["model.norm.weight"])
    head.lm_head.weight.data.copy_(ck["lm_head.weight"])
    blocks, loras = [], []
    for i in range(layers):
        blk = LlamaBlock(shape, quantized=False)
        p = f"model.layers.{i}."
        blk.input_layernorm.weight.data.copy_(ck[p + "input_layernorm.weight"])
        blk.post_attention_layernorm.weight.data.copy_(ck[p + "post_attention_layernorm.weight"])
        for part, names in (("self_attn", ("q_proj", "k_proj", "v_proj", "o_proj")),
                            ("mlp", ("gate_proj", "up_proj", "down_proj"))):
            for n in names:
                blk.base_projection(n).weight.data.copy_(ck[f"{p}{part}.{n}.weight"])
        blk.self_attn.attn_impl = "eager"
        swap_linears(blk)
        params = {n: (torch.nn.Parameter(bf16(d[f"lora/{i + 1}.self_attn.{n}/A"]).clone()),
                      torch.nn.Parameter(bf16(d[f"lora/{i + 1}.self_attn.{n}/B"]).clone()))
                  for n in ("q_proj", "v_proj")}
        apply_lora(blk, rank, alpha, targets=("q_proj", "v_proj"), params=params)
        blocks.append(blk)
        loras.append(params)
    ids = torch.from_numpy(d["ids"])
    cos, sin = rope_cos_sin(shape, seq, "cpu", torch.bfloat16)
    h = embed(ids)
    for blk in blocks:
        h = blk(h, cos, sin)
    logits = head(h)
    loss = F.cross_entropy(logits[:, :-1].reshape(-1, vocab), ids[:, 1:].reshape(-1))
    loss.backward()
    assert (torch_bf16_to_bits(logits.detach()) == d["logits"]).all()
    assert float(loss.detach()) == float(d["loss"])
    for i, params in enumerate(loras):
        for n, (a, b) in params.items():
            assert (torch_bf16_to_bits(a.grad) == d[f"grad/{i + 1}.self_attn.{n}/A"]).all(), (i, n)
            assert (torch_bf16_to_bits(b.grad) == d[f"grad/{i + 1}.self_attn.{n}/B"]).all(), (i, n)


@pytest.mark.parametrize("case", ["ragged", "one_chunk"])
def test_chunked_attention_oracle_reproduces_reference(case):
    """tests/golden/chunked_attention.npz holds the output of the reference's own
    chunked_attention (src/lema/_tensorstore.py:565-608) over query chunks as its
    RoPE adapter drives it; the oracle's restatement gives the same bits."""
    import numpy as np
    from pathlib import Path

    from oracle.torch_ref import chunked_causal_attention_ref
    d = np.load(Path(__file__).parent / "golden" / "chunked_attention.npz")
    B, H, Hkv, S, D, chunk = (int(v) for v in d[f"{case}/meta"])
    q, k, v = (bf16(d[f"{case}/{n}"]) for n in ("q", "k", "v"))
    assert q.shape == (B, H, S, D) and k.shape == (B, Hkv, S, D)
    o = chunked_causal_attention_ref(q, k, v, D ** -0.5, chunk)
    assert (torch_bf16_to_bits(o) == d[f"{case}/o"]).all()
