"""Helpers shared by the layer-level tests: load the reference-path golden
fixture (tests/golden/llama_layer_w8a8.npz) into a lema_b200 LlamaBlock."""
from pathlib import Path

import numpy as np
import torch

from lema_b200.llama import LlamaBlock, LlamaShape, apply_lora

GOLDEN = Path(__file__).parent / "golden" / "llama_layer_w8a8.npz"


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def load():
    d = np.load(GOLDEN)
    hidden, heads, inter, seq, batch, rank, alpha = (int(v) for v in d["meta"])
    shape = LlamaShape(hidden=hidden, heads=heads, kv_heads=heads, intermediate=inter,
                       vocab=256, layers=1)
    return d, shape, rank, alpha


def block_from_fixture(d, shape, rank, alpha, device, quantized: bool):
    """LlamaBlock with the fixture's weights; W8A8Linear projections when
    ``quantized`` (weights quantised on the device), else bf16 nn.Linear."""
    blk = LlamaBlock(shape, quantized=quantized, device=device)
    params = {}
    for key in d.files:
        if not key.startswith("param/"):
            continue
        name = key[len("param/"):]
        t = bf16(d[key]).to(device)
        if "lora_" in name:
            proj = name.split(".")[1]
            slot = 0 if "lora_A" in name else 1
            params.setdefault(proj, [None, None])[slot] = torch.nn.Parameter(t.clone())
            continue
        name = name.replace(".base_layer", "")
        mod_name, _, leaf = name.rpartition(".")
        mod = blk.get_submodule(mod_name)
        if quantized and hasattr(mod, "load_float_weight"):
            mod.load_float_weight(t)
        else:
            getattr(mod, leaf).data.copy_(t)
    apply_lora(blk, rank, alpha, targets=("q_proj", "v_proj"),
               params={k: tuple(v) for k, v in params.items()})
    return blk
