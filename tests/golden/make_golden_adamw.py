"""Writes tests/golden/full_ft_adamw.npz from the reference's own optimizer code.

Run from the repo root in a checkout that has the reference source next to it:

    python tests/golden/make_golden_adamw.py <reference>/src

It runs the reference's per-layer clip and AdamW step of selective full
fine-tuning (``FullFTManager.clip_grad_norm_`` and ``step_layer``,
src/lema/_full_ft.py:194-229) on the CPU for three accumulation boundaries of
one layer with two trainable bf16 projections, lr 1e-3 and weight decay 0.01,
and saves the initial weights, each boundary's accumulated gradients, and the
weights and moments after each step (bf16 as uint16 bit patterns). The manager's
state is set directly (no checkpoint or adapter behind it): only the attributes
those two methods read. The script is the only place that reads the reference;
tests read the .npz.
"""
import os
import sys
import types

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

SHAPES = {"q_proj": (32, 48), "v_proj": (24, 48)}
LR, WD, STEPS = 1e-3, 0.01, 3


def main(ref_src: str):
    sys.path.insert(0, ref_src)
    from lema._full_ft import FullFTManager

    m = FullFTManager.__new__(FullFTManager)
    m.config = types.SimpleNamespace(learning_rate=LR, weight_decay=WD, device="cpu")
    m.layer_steps = {}
    m.true_weights, m.opt_states, m.accumulators = {}, {}, {}
    m.selected_layer_keys = {0: []}
    m.module_name_to_key = {0: {}}
    g = torch.Generator().manual_seed(7)
    out = {}
    for name, shape in SHAPES.items():
        key = (0, f"model.layers.0.self_attn.{name}.weight")
        w = (0.02 * torch.randn(shape, generator=g)).to(torch.bfloat16)
        m.true_weights[key] = w
        m.opt_states[key] = {"exp_avg": torch.zeros(shape), "exp_avg_sq": torch.zeros(shape)}
        m.accumulators[key] = torch.zeros(shape)
        m.selected_layer_keys[0].append(key)
        m.module_name_to_key[0][f"self_attn.{name}.weight"] = key
        out[f"w0/{name}"] = O.torch_bf16_to_bits(w).copy()  # step_layer updates w in place
    for step in range(1, STEPS + 1):
        for name, shape in SHAPES.items():
            key = (0, f"model.layers.0.self_attn.{name}.weight")
            # the second boundary's gradients exceed the clip norm, the others do not
            grad = torch.randn(shape, generator=g) * (0.05 if step == 2 else 1e-3)
            m.accumulators[key].copy_(grad)
            out[f"g{step}/{name}"] = grad.numpy().copy()
        norm = m.clip_grad_norm_(0, 1.0)
        out[f"norm{step}"] = np.float64(norm)
        m.step_layer(0)
        for name in SHAPES:
            key = (0, f"model.layers.0.self_attn.{name}.weight")
            out[f"w{step}/{name}"] = O.torch_bf16_to_bits(m.true_weights[key]).copy()
            out[f"m{step}/{name}"] = m.opt_states[key]["exp_avg"].numpy().copy()
            out[f"v{step}/{name}"] = m.opt_states[key]["exp_avg_sq"].numpy().copy()
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "full_ft_adamw.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_adamw.py <reference>/src")
    main(sys.argv[1])
