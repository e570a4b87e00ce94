"""Selective full fine-tuning of W8A8 projections (row A9).

Mirrors the reference's ``FullFTManager`` (src/lema/_full_ft.py): chosen
projections of chosen layers are trainable; their true weights (model dtype,
bf16) and fp32 AdamW moments live in host RAM (pinned here), their gradients
accumulate in fp32 (``accumulate_grads``, :186-192 — on the device here), and
at each accumulation boundary every selected layer is clipped to norm 1 over
its accumulators (:194-202) and stepped with the same AdamW arithmetic
(:204-229: decoupled weight decay, bias-corrected moments, eps 1e-8, the
update computed in fp32 and the weight stored back in bf16).

What W8A8 adds: the forward of a trainable projection uses the int8 copy of
its *current* true weight, so after each step the new bf16 weight is
re-quantised per output channel on the device (K1) and the int8 rows and
scales are written back into the layer's pinned-RAM segment, from which the
next forward streams them. The backward is straight-through: dx as for frozen
projections, dW = dy^T . x with fp32 accumulation (``lema_bf16_gemm_tn_f32``).

The reference clips and steps the selected layers after the whole backward;
each layer's clip and step read only that layer's accumulators, final once its
own backward is done, so ``step_layer_async`` runs them right then on a side
stream (device-side clip, non-blocking pinned copies both ways), overlapping
the optimizer's PCIe round trips with the backward of the remaining layers.
``finish`` waits for that stream before the pinned weights are read again.
"""
from __future__ import annotations

import torch

from . import ops


class SelectiveFullFT:
    def __init__(self, ws, layers, modules, true_weights: dict, device, lr: float,
                 weight_decay: float):
        self.ws = ws
        self.layers = tuple(layers)
        self.modules = tuple(modules)
        self.device = torch.device(device)
        self.lr = lr
        self.wd = weight_decay
        self.true: dict[tuple[int, str], torch.Tensor] = {}
        self.m: dict[tuple[int, str], torch.Tensor] = {}
        self.v: dict[tuple[int, str], torch.Tensor] = {}
        self.acc: dict[tuple[int, str], torch.Tensor] = {}
        for key, w in true_weights.items():
            self.true[key] = w.detach().to("cpu", torch.bfloat16).contiguous().pin_memory()
            self.m[key] = torch.zeros(w.shape, dtype=torch.float32).pin_memory()
            self.v[key] = torch.zeros(w.shape, dtype=torch.float32).pin_memory()
            self.acc[key] = torch.zeros(w.shape, dtype=torch.float32, device=self.device)
        self.layer_steps: dict[int, int] = {}
        self.stream = torch.cuda.Stream(self.device)

    def attach(self, layer: int, block) -> None:
        """Makes the selected projections of ``block`` (bound to ``layer``) trainable."""
        for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            base = block.base_projection(name)
            base.wgrad_acc = self.acc.get((layer, name))

    def layer_grads(self, layer: int) -> list[torch.Tensor]:
        return [self.acc[(layer, n)] for n in self.modules if (layer, n) in self.acc]

    def clip_layer_(self, layer: int, max_norm: float = 1.0) -> torch.Tensor:
        """Scales the layer's accumulators by max_norm / norm when their joint
        norm exceeds max_norm (reference :194-202), on the device: the per-tensor
        fp32 sums of squares are added in fp64 as the reference's Python floats are,
        and the fp32 multiply by 1.0 when no clipping is due leaves them unchanged.
        Returns the norm (device tensor)."""
        accs = self.layer_grads(layer)
        total = torch.zeros((), dtype=torch.float64, device=self.device)
        for a in accs:
            total = total + a.pow(2).sum().double()
        norm = total.sqrt()
        coeff = torch.where(norm > max_norm, max_norm / norm, torch.ones_like(norm))
        coeff = coeff.float()
        for a in accs:
            a.mul_(coeff)
        return norm

    @torch.no_grad()
    def step_layer(self, layer: int) -> None:
        """The reference's AdamW step (src/lema/_full_ft.py:204-229) of every
        selected projection of ``layer``: weight and moments in from pinned RAM,
        one fused kernel (``lema_adamw_requant_rows``: the AdamW arithmetic, the
        per-output-channel int8 re-quantisation of the new weight, the cleared
        accumulator), weight, moments and the int8 rows back to pinned RAM."""
        step = self.layer_steps.get(layer, 0) + 1
        self.layer_steps[layer] = step
        for name in self.modules:
            key = (layer, name)
            if key not in self.true:
                continue
            w = self.true[key].to(self.device, non_blocking=True)
            m = self.m[key].to(self.device, non_blocking=True)
            v = self.v[key].to(self.device, non_blocking=True)
            wq, sw = ops.adamw_requant_rows(w, self.acc[key], m, v, step, self.lr, self.wd)
            ram = self.ws.ram[layer]
            # pinned destinations, copies ordered on this stream (the device
            # temporaries are freed only after them, stream-ordered)
            self.ws._view(ram, name + ".wq").copy_(wq, non_blocking=True)
            self.ws._view(ram, name + ".sw").copy_(sw, non_blocking=True)
            self.true[key].copy_(w, non_blocking=True)
            self.m[key].copy_(m, non_blocking=True)
            self.v[key].copy_(v, non_blocking=True)

    def step_layer_async(self, layer: int, reduce_entry=None, reducer=None) -> None:
        """Clips and steps ``layer`` on the side stream once the current stream's
        work so far (the layer's backward) is done; with data parallelism the
        layer's gradient bucket is first averaged over the ranks (the side stream
        waits for its all-reduce)."""
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            if reduce_entry is not None:
                reducer.finish(reduce_entry)
            self.clip_layer_(layer, 1.0)
            self.step_layer(layer)

    def finish(self) -> None:
        """Waits (host) for every pending layer step: the pinned weights, moments
        and int8 segments are then current."""
        self.stream.synchronize()

    def step(self) -> None:
        for layer in self.layers:
            self.clip_layer_(layer, 1.0)
            self.step_layer(layer)
        torch.cuda.current_stream(self.device).synchronize()
