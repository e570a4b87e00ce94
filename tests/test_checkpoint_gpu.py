"""GPU tests of the trainer's weight loading: a Hugging Face checkpoint (the
safetensors files the reference's GlobalBinaryIndex reads) is quantised into
the int8 segments exactly as the W8A8 linear quantises weights, and an int8
segment file written by ``save_segments`` loads back bit for bit and gives the
same step."""
import pytest
import torch
from torch.nn.attention import SDPBackend, sdpa_kernel

from lema_b200 import ops
from lema_b200.llama import LlamaShape
from lema_b200.moe import MixtralShape
from lema_b200.trainer import StreamedLoraTrainer

pytestmark = pytest.mark.gpu

LLAMA = LlamaShape(hidden=256, heads=4, kv_heads=4, intermediate=688, vocab=512, layers=3)
MIXTRAL = MixtralShape(hidden=256, heads=4, kv_heads=2, intermediate=512, vocab=512, layers=2,
                       experts=4, top_k=2)


def _hf_llama(path):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=4,
                      intermediate_size=688, num_hidden_layers=3, vocab_size=512,
                      rms_norm_eps=1e-5, rope_theta=1e4, tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" in n:
                p.uniform_(0.5, 1.5)  # non-trivial norm weights
    m.save_pretrained(path)
    return {k: v.detach().clone() for k, v in m.state_dict().items()}


def _hf_mixtral(path):
    from transformers import MixtralConfig, MixtralForCausalLM
    torch.manual_seed(1)
    cfg = MixtralConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2,
                        intermediate_size=512, num_hidden_layers=2, vocab_size=512,
                        num_local_experts=4, num_experts_per_tok=2, rms_norm_eps=1e-5,
                        tie_word_embeddings=False)
    m = MixtralForCausalLM(cfg).to(torch.bfloat16)
    m.save_pretrained(path)
    return {k: v.detach().clone() for k, v in m.state_dict().items()}


def _ids(dev, vocab):
    g = torch.Generator(device=dev).manual_seed(3)
    return torch.randint(0, vocab, (2, 64), device=dev, generator=g)


def test_llama_checkpoint_quantised_into_segments(cuda_device, tmp_path):
    sd = _hf_llama(tmp_path / "hf")
    tr = StreamedLoraTrainer(LLAMA, cuda_device, batch=2, seq=64, seed=0,
                             weights=str(tmp_path / "hf"))
    ws = tr.ws
    for b in range(LLAMA.layers):
        for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                     "down_proj"):
            part = "self_attn" if name.endswith(("q_proj", "k_proj", "v_proj", "o_proj")) \
                else "mlp"
            w = sd[f"model.layers.{b}.{part}.{name}.weight"].to(cuda_device)
            wq, sw = ops.quantize_weight(w)
            assert torch.equal(ws._view(ws.ram[b], name + ".wq"), wq.cpu())
            assert torch.equal(ws._view(ws.ram[b], name + ".sw"), sw.cpu())
        for norm in ("input_layernorm", "post_attention_layernorm"):
            assert torch.equal(ws._view(ws.ram[b], norm),
                               sd[f"model.layers.{b}.{norm}.weight"])
    assert torch.equal(tr.embed.weight.cpu(), sd["model.embed_tokens.weight"])
    assert torch.equal(tr.head.lm_head.weight.cpu(), sd["lm_head.weight"])
    assert torch.equal(tr.head.norm.weight.cpu(), sd["model.norm.weight"])
    # the save / load round trip: same bytes, same step
    path = str(tmp_path / "w8a8.safetensors")
    tr.save_segments(path)
    with sdpa_kernel(SDPBackend.MATH):
        l0 = float(tr.train_step(_ids(cuda_device, LLAMA.vocab)))
    ram0 = tr.ws.ram.clone()
    tr.close()
    tr2 = StreamedLoraTrainer(LLAMA, cuda_device, batch=2, seq=64, seed=0, weights=path)
    assert torch.equal(tr2.ws.ram, ram0)
    with sdpa_kernel(SDPBackend.MATH):
        l1 = float(tr2.train_step(_ids(cuda_device, LLAMA.vocab)))
    tr2.close()
    assert l0 == l1
    # a file for another shape is refused
    with pytest.raises(ValueError):
        StreamedLoraTrainer(LlamaShape(hidden=256, heads=4, kv_heads=4, intermediate=688,
                                       vocab=512, layers=2), cuda_device, batch=2, seq=64,
                            weights=path)


def test_mixtral_checkpoint_experts_quantised(cuda_device, tmp_path):
    sd = _hf_mixtral(tmp_path / "hf")
    tr = StreamedLoraTrainer(MIXTRAL, cuda_device, batch=2, seq=64, seed=0,
                             weights=str(tmp_path / "hf"))
    ws = tr.ws
    for b in range(MIXTRAL.layers):
        p = f"model.layers.{b}.mlp"
        gu, dn = sd[f"{p}.experts.gate_up_proj"], sd[f"{p}.experts.down_proj"]
        for e in range(MIXTRAL.experts):
            q, s = ops.quantize_weight(gu[e].to(cuda_device))
            assert torch.equal(ws._view(ws.ram[b], "experts.gate_up.wq")[e], q.cpu())
            assert torch.equal(ws._view(ws.ram[b], "experts.gate_up.sw")[e], s.cpu())
            q, s = ops.quantize_weight(dn[e].to(cuda_device))
            assert torch.equal(ws._view(ws.ram[b], "experts.down.wq")[e], q.cpu())
        assert torch.equal(ws._view(ws.ram[b], "router"), sd[f"{p}.gate.weight"])
    with sdpa_kernel(SDPBackend.MATH):
        loss = float(tr.train_step(_ids(cuda_device, MIXTRAL.vocab)))
    tr.close()
    assert loss == loss and 0 < loss < 20
