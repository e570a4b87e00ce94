"""Writes tests/golden/llama_model_w8a8.npz from the reference's own trainer.

Run from the repo root in a checkout that has the reference source next to it:

    python tests/golden/make_golden_model.py <reference>/src

It saves a tiny random Llama checkpoint (2 blocks, hidden 128, 4 heads x 32,
MLP 352, vocab 256) as safetensors, builds the reference's ``LemaModel`` over it
(LoRA r4 alpha 8 on q_proj / v_proj, bf16, CPU, eager attention), swaps the
oracle's W8A8 linear (oracle/torch_ref.py) into the seven projections of every
decoder layer the reference constructs (quantising the weight each projection
holds at call time, since the reference reuses pooled modules) and rebinds that layer's LoRA parameters (the
reference binds them only when a pooled module is first created,
src/lema/adapters/_llama.py:83-84, so a reused module would keep another
layer's), seeds every LoRA B non-zero, and runs one
``LemaTrainer.train_step`` (src/lema/_trainer.py:75-194) without an optimizer.
It stores the checkpoint tensors, the LoRA parameters, the token ids, the
logits, the loss and every LoRA gradient (bf16 as uint16 bit patterns). The
script is the only place that reads the reference; tests read the .npz.
"""
import json
import os
import sys
import tempfile

import numpy as np
import torch
from safetensors.torch import save_file

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from oracle.torch_ref import OracleW8A8Linear  # noqa: E402

HIDDEN, HEADS, INTER, LAYERS, VOCAB, SEQ, BATCH = 128, 4, 352, 2, 256, 32, 2
RANK, ALPHA = 4, 8
PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def route_through_oracle(module):
    """Every projection (or a LoRA wrapper's base layer) computes the oracle's W8A8
    linear of the weight it holds at call time. The nn.Linear objects stay in
    place: the reference copies each layer's weights into the parameters it
    recorded when the pooled module was created."""
    for parent in list(module.modules()):
        for name, child in list(parent.named_children()):
            if name not in PROJ:
                continue
            lin = child.base_layer if hasattr(child, "base_layer") else child
            if isinstance(lin, torch.nn.Linear) and not getattr(lin, "_oracle", False):
                lin._oracle = True
                lin.forward = (lambda x, lin=lin: OracleW8A8Linear.from_linear(lin)(x))


def main(ref_src: str):
    sys.path.insert(0, ref_src)
    from lema import LemaConfig, LemaModel

    torch.manual_seed(3)  # the reference draws LoRA A (kaiming) from the global generator
    g = torch.Generator().manual_seed(2024)
    sd = {"model.embed_tokens.weight": 0.02 * torch.randn(VOCAB, HIDDEN, generator=g),
          "model.norm.weight": 1.0 + 0.1 * torch.randn(HIDDEN, generator=g),
          "lm_head.weight": 0.02 * torch.randn(VOCAB, HIDDEN, generator=g)}
    for i in range(LAYERS):
        p = f"model.layers.{i}"
        sd[f"{p}.input_layernorm.weight"] = 1.0 + 0.1 * torch.randn(HIDDEN, generator=g)
        sd[f"{p}.post_attention_layernorm.weight"] = 1.0 + 0.1 * torch.randn(HIDDEN, generator=g)
        for n, (o, k) in {"self_attn.q_proj": (HIDDEN, HIDDEN), "self_attn.k_proj": (HIDDEN, HIDDEN),
                          "self_attn.v_proj": (HIDDEN, HIDDEN), "self_attn.o_proj": (HIDDEN, HIDDEN),
                          "mlp.gate_proj": (INTER, HIDDEN), "mlp.up_proj": (INTER, HIDDEN),
                          "mlp.down_proj": (HIDDEN, INTER)}.items():
            sd[f"{p}.{n}.weight"] = 0.02 * torch.randn(o, k, generator=g)
    sd = {k: v.to(torch.bfloat16).contiguous() for k, v in sd.items()}
    out = {f"ckpt/{k}": O.torch_bf16_to_bits(v).copy() for k, v in sd.items()}
    with tempfile.TemporaryDirectory() as d:
        save_file(sd, os.path.join(d, "model.safetensors"))
        cfg = {"model_type": "llama", "architectures": ["LlamaForCausalLM"],
               "hidden_size": HIDDEN, "num_attention_heads": HEADS,
               "num_key_value_heads": HEADS, "intermediate_size": INTER,
               "num_hidden_layers": LAYERS, "vocab_size": VOCAB, "rms_norm_eps": 1e-5,
               "rope_theta": 10000.0, "max_position_embeddings": 512,
               "tie_word_embeddings": False, "hidden_act": "silu", "torch_dtype": "bfloat16",
               "dtype": "bfloat16"}
        with open(os.path.join(d, "config.json"), "w") as f:
            json.dump(cfg, f)
        lcfg = LemaConfig(model_name_or_path=d, model_type="llama",
                          gbi_path=os.path.join(d, "model.safetensors"), device="cpu",
                          dtype="bfloat16", lora_rank=RANK, lora_alpha=ALPHA,
                          lora_target_modules=["q_proj", "v_proj"], save_steps=0,
                          backend="python", attn_implementation="eager")
        model = LemaModel(lcfg)
        model.initialize_lora()
        orig = model.adapter.construct_layer_module

        def construct(layer_id, *a, **k):
            module = orig(layer_id, *a, **k)
            if 1 <= layer_id <= LAYERS:
                # the reference binds a layer's LoRA parameters only when it creates a
                # pooled module (src/lema/adapters/_llama.py:83-84), so a module reused
                # for another layer keeps the first layer's; rebind them every time
                model.lora_manager.update_lora_params(layer_id, module)
                route_through_oracle(module)
            return module
        model.adapter.construct_layer_module = construct
        torch.manual_seed(5)
        ids = torch.randint(0, VOCAB, (BATCH, SEQ), generator=torch.Generator().manual_seed(9))
        trainer = model.get_trainer(None)
        # every LoRA B non-zero so that every gradient is non-trivial
        for layer_id in range(1, LAYERS + 1):
            blk = construct(layer_id, None, model.lora_manager)
            model.adapter.release_layer_module(blk)
        with torch.no_grad():
            for key, p in sorted(model.lora_manager.params.items()):
                p["B"].copy_((0.02 * torch.randn(p["B"].shape, generator=g)).to(p["B"].dtype))
                out[f"lora/{key}/A"] = O.torch_bf16_to_bits(p["A"]).copy()
                out[f"lora/{key}/B"] = O.torch_bf16_to_bits(p["B"]).copy()
        fwd = model.adapter.forward_layer
        stage = {"i": 0}

        def forward_layer(module, x, **k):
            y = fwd(module, x, **k)
            if not torch.is_grad_enabled():  # the no-grad forward: each layer's output
                yt = y[0] if isinstance(y, tuple) else y
                out[f"stage/{stage['i']}"] = O.torch_bf16_to_bits(yt.detach().to(torch.bfloat16)).copy()
                stage["i"] += 1
            return y
        model.adapter.forward_layer = forward_layer
        logits, loss = trainer.train_step(ids, labels=ids)
        out["ids"] = ids.numpy()
        out["logits"] = O.torch_bf16_to_bits(logits.detach()).copy()
        out["loss"] = np.float64(loss)
        for key, p in sorted(model.lora_manager.params.items()):
            out[f"grad/{key}/A"] = O.torch_bf16_to_bits(p["A"].grad).copy()
            out[f"grad/{key}/B"] = O.torch_bf16_to_bits(p["B"].grad).copy()
        out["meta"] = np.array([HIDDEN, HEADS, INTER, LAYERS, VOCAB, SEQ, BATCH, RANK, ALPHA])
        trainer.close()
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "llama_model_w8a8.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, "loss", float(loss), "lora keys", sorted(model.lora_manager.params))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_model.py <reference>/src")
    main(sys.argv[1])
