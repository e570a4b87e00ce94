"""Writes tests/golden/llama_layer_w8a8.npz from the reference's own Python path.

Run from the repo root in a checkout that has the reference source next to it:

    python tests/golden/make_golden_layer.py <reference>/src

It builds one Llama decoder layer with the reference's adapter
(``LlamaAdapter.construct_layer_module``, src/lema/adapters/_llama.py:59-107)
and LoRA manager (src/lema/_lora.py:28-88, rank 4, alpha 8, targets q_proj and
v_proj), in bf16 on the CPU with eager attention, swaps the oracle's W8A8
linear (oracle/torch_ref.py) into the seven projections, runs the reference's
``forward_layer`` (src/lema/adapters/_llama.py:183-252) and backward, and saves
inputs, weights, outputs and gradients. bf16 tensors are stored as uint16 bit
patterns. Shapes: hidden 128, 4 heads x 32, MLP 352, seq 32, batch 2.
The script is the only place that reads the reference; tests read the .npz.
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from oracle.torch_ref import swap_linears  # noqa: E402

HIDDEN, HEADS, INTER, SEQ, BATCH, VOCAB = 128, 4, 352, 32, 2, 256
RANK, ALPHA = 4, 8


def main(ref_src: str):
    sys.path.insert(0, ref_src)
    from lema._lora import LoRAManager
    from lema.adapters._llama import LlamaAdapter

    cfg = {"model_type": "llama", "hidden_size": HIDDEN, "num_attention_heads": HEADS,
           "num_key_value_heads": HEADS, "intermediate_size": INTER, "num_hidden_layers": 1,
           "vocab_size": VOCAB, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
           "max_position_embeddings": 512, "dtype": "bfloat16", "attn_implementation": "eager"}
    adapter = LlamaAdapter(cfg)
    lora = LoRAManager({"r": RANK, "alpha": ALPHA, "target_modules": ["q_proj", "v_proj"]},
                       device="cpu", dtype=torch.bfloat16)
    torch.manual_seed(0)
    module = adapter.construct_layer_module(1, None, lora)
    g = torch.Generator().manual_seed(1234)
    out = {}
    with torch.no_grad():
        for name, p in module.named_parameters():
            if name.endswith("layernorm.weight"):
                p.copy_((1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(p.dtype))
            elif name.endswith("lora_A"):
                p.copy_((torch.rand(p.shape, generator=g) * 2 - 1).mul(0.1).to(p.dtype))
            elif name.endswith("lora_B"):
                p.copy_((0.02 * torch.randn(p.shape, generator=g)).to(p.dtype))
            else:
                p.copy_((0.02 * torch.randn(p.shape, generator=g)).to(p.dtype))
            out["param/" + name] = O.torch_bf16_to_bits(p)
    swap_linears(module)
    x = torch.randn(BATCH, SEQ, HIDDEN, generator=g).to(torch.bfloat16).requires_grad_(True)
    y = adapter.forward_layer(module, x, gradient_checkpointing=False)
    dy = torch.randn(y.shape, generator=g).to(torch.bfloat16)
    y.backward(dy)
    out["x"] = O.torch_bf16_to_bits(x)
    out["dy"] = O.torch_bf16_to_bits(dy)
    out["y"] = O.torch_bf16_to_bits(y)
    out["dx"] = O.torch_bf16_to_bits(x.grad)
    for name, p in module.named_parameters():
        if "lora_" in name:
            out["grad/" + name] = O.torch_bf16_to_bits(p.grad)
    out["meta"] = np.array([HIDDEN, HEADS, INTER, SEQ, BATCH, RANK, ALPHA], dtype=np.int64)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "llama_layer_w8a8.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, sorted(out))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_layer.py <reference>/src")
    main(sys.argv[1])
