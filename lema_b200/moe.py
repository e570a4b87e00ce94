"""Mixtral-shaped sparse MoE layer with grouped W8A8 experts (row A8).

Same computation as HF ``MixtralSparseMoeBlock`` in the transformers version
the reference pins (driven by src/lema/adapters/_mixtral.py:266-268 with the
``grouped_mm`` experts implementation selected at :21-22):

* router: ``F.linear`` in the model dtype (bf16, not quantised), softmax in
  fp32, top-k, the k weights renormalised to sum to 1;
* experts: fused ``gate_up_proj [E, 2I, H]`` and ``down_proj [E, H, I]``;
  ``down(silu(gate) * up)`` per routed token;
* combine: ``(expert_out * weight).to(bf16)`` accumulated per token in bf16.

On the device the experts run as two grouped W8A8 GEMMs over the routed
tokens sorted by expert (``lema_grouped_w8a8_gemm``): each token is quantised
once per token (its k copies share the int8 row and scale), the SwiGLU output
is quantised per routed row, and the backward is the straight-through
grouped dgrad (``lema_grouped_w8a8_dgrad``). The per-expert row counts are read
back to the host once per layer call to size the grouped launch.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .llama import LlamaAttention, LlamaBlock, LlamaShape, RMSNorm


@dataclass(frozen=True)
class MixtralShape(LlamaShape):
    """Mixtral-8x7B sizes: GQA 32 q / 8 kv heads, 8 experts, top-2, FFN 14336."""

    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    intermediate: int = 14336
    vocab: int = 32000
    layers: int = 32
    eps: float = 1e-5
    theta: float = 1e6
    experts: int = 8
    top_k: int = 2


class Router(nn.Module):
    """Top-k softmax router (HF MixtralTopKRouter)."""

    def __init__(self, shape: MixtralShape, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.top_k = shape.top_k
        self.weight = nn.Parameter(torch.zeros(shape.experts, shape.hidden, device=device,
                                               dtype=dtype))

    def forward(self, x2d: torch.Tensor):
        logits = F.linear(x2d, self.weight)
        probs = torch.softmax(logits.float(), dim=-1)
        top_v, top_i = torch.topk(probs, self.top_k, dim=-1)
        top_v = top_v / top_v.sum(dim=-1, keepdim=True)
        return probs, top_v, top_i


class FloatExperts(nn.Module):
    """Reference-layout float experts (HF MixtralExperts), for parity tests."""

    def __init__(self, shape: MixtralShape, device=None, dtype=torch.bfloat16):
        super().__init__()
        E, I, H = shape.experts, shape.intermediate, shape.hidden
        self.gate_up_proj = nn.Parameter(torch.zeros(E, 2 * I, H, device=device, dtype=dtype))
        self.down_proj = nn.Parameter(torch.zeros(E, H, I, device=device, dtype=dtype))

    def forward(self, x2d, top_i, top_w):
        final = torch.zeros_like(x2d)
        E = self.gate_up_proj.shape[0]
        mask = F.one_hot(top_i, num_classes=E).permute(2, 1, 0)
        for e in range(E):
            pos, tok = torch.where(mask[e])
            if tok.numel() == 0:
                continue
            gate, up = F.linear(x2d[tok], self.gate_up_proj[e]).chunk(2, dim=-1)
            h = F.linear(F.silu(gate) * up, self.down_proj[e])
            h = h * top_w[tok, pos, None]
            final.index_add_(0, tok, h.to(final.dtype))
        return final


def route_sort(top_i: torch.Tensor, E: int):
    """Sorts the (token, slot) assignments by expert. Returns (order, token of each
    sorted assignment, slot of each, host offsets [E+1])."""
    T, k = top_i.shape
    flat = top_i.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=E)
    offsets = [0] + torch.cumsum(counts, 0).tolist()
    if len(offsets) != E + 1:
        raise ValueError(f"routing index out of range for {E} experts")
    return order, order // k, order % k, offsets


class _GroupedExpertsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, top_w, top_i, wq_gu, sw_gu, wq_dn, sw_dn):
        E, I2, H = wq_gu.shape
        I = I2 // 2
        T = x2d.shape[0]
        order, tok, slot, offsets = route_sort(top_i, E)
        xq, sx = ops.quantize_rows(x2d.contiguous())
        xq_s = xq.index_select(0, tok)
        sx_s = sx.index_select(0, tok)
        gu = ops.grouped_w8a8_gemm(xq_s, sx_s, wq_gu, sw_gu, offsets)      # [R, 2I]
        gate, up = gu[:, :I], gu[:, I:]
        mid = F.silu(gate) * up                                             # [R, I] bf16
        mq, sm = ops.quantize_rows(mid)
        out_s = ops.grouped_w8a8_gemm(mq, sm, wq_dn, sw_dn, offsets)       # [R, H]
        w_s = top_w[tok, slot]                                              # fp32 [R]
        contrib = (out_s * w_s[:, None]).to(x2d.dtype)
        final = torch.zeros_like(x2d)
        final.index_add_(0, tok, contrib)
        ctx.save_for_backward(gu, out_s, w_s, tok, slot, wq_gu, sw_gu, wq_dn, sw_dn)
        ctx.offsets = offsets
        ctx.T = T
        return final

    @staticmethod
    def backward(ctx, d_final):
        gu, out_s, w_s, tok, slot, wq_gu, sw_gu, wq_dn, sw_dn = ctx.saved_tensors
        offsets = ctx.offsets
        I = gu.shape[1] // 2
        d_rows = d_final.index_select(0, tok)                               # [R, H]
        d_w = (d_rows.float() * out_s.float()).sum(-1)                      # grad of routing weights
        d_out = (d_rows.float() * w_s[:, None]).to(torch.bfloat16)
        d_mid = ops.grouped_w8a8_dgrad(d_out, wq_dn, sw_dn, offsets)       # [R, I]
        gate, up = gu[:, :I].float(), gu[:, I:].float()
        sg = torch.sigmoid(gate)
        silu = gate * sg
        dm = d_mid.float()
        d_gate = dm * up * (sg * (1 + gate * (1 - sg)))
        d_up = dm * silu
        d_gu = torch.cat([d_gate, d_up], dim=1).to(torch.bfloat16)         # [R, 2I]
        d_x_s = ops.grouped_w8a8_dgrad(d_gu, wq_gu, sw_gu, offsets)        # [R, H]
        d_x = torch.zeros(ctx.T, d_x_s.shape[1], dtype=torch.float32, device=d_x_s.device)
        d_x.index_add_(0, tok, d_x_s.float())
        d_top_w = torch.zeros(ctx.T, w_s.numel() // ctx.T, dtype=torch.float32,
                              device=d_x_s.device)
        d_top_w[tok, slot] = d_w
        return d_x.to(d_final.dtype), d_top_w, None, None, None, None, None


class W8A8Experts(nn.Module):
    """Frozen experts: int8 gate_up [E, 2I, H] and down [E, H, I] with per-output-channel
    fp32 scales; forward through the grouped W8A8 GEMMs. ``forward(x2d, top_i, top_w)``
    takes the arguments of HF's fused-experts modules (MixtralExperts, Lfm2MoeExperts:
    hidden states [T, H], top-k indices and weights [T, k]) and combines like them."""

    def __init__(self, shape: MixtralShape | None = None, device=None,
                 dims: tuple[int, int, int] | None = None):
        super().__init__()
        E, I, H = dims if dims is not None else (shape.experts, shape.intermediate,
                                                  shape.hidden)
        self.register_buffer("wq_gate_up", torch.zeros(E, 2 * I, H, dtype=torch.int8, device=device))
        self.register_buffer("sw_gate_up", torch.ones(E, 2 * I, dtype=torch.float32, device=device))
        self.register_buffer("wq_down", torch.zeros(E, H, I, dtype=torch.int8, device=device))
        self.register_buffer("sw_down", torch.ones(E, H, dtype=torch.float32, device=device))

    @torch.no_grad()
    def load_float(self, gate_up: torch.Tensor, down: torch.Tensor) -> None:
        self.requantize_gate_up_(gate_up)
        self.requantize_down_(down)

    @classmethod
    def from_fused(cls, gate_up: torch.Tensor, down: torch.Tensor) -> "W8A8Experts":
        """Quantises HF fused expert weights (gate_up [E, 2I, H], down [E, H, I],
        on the device) per output channel."""
        E, I2, H = gate_up.shape
        m = cls(device=gate_up.device, dims=(E, I2 // 2, H))
        m.load_float(gate_up, down)
        return m

    @torch.no_grad()
    def requantize_gate_up_(self, gate_up: torch.Tensor) -> None:
        E, I2, H = self.wq_gate_up.shape
        q, s = ops.quantize_weight(gate_up.reshape(E * I2, H).to(self.wq_gate_up.device))
        self.wq_gate_up.copy_(q.reshape(E, I2, H))
        self.sw_gate_up.copy_(s.reshape(E, I2))

    @torch.no_grad()
    def requantize_down_(self, down: torch.Tensor) -> None:
        E, H, I = self.wq_down.shape
        q, s = ops.quantize_weight(down.reshape(E * H, I).to(self.wq_down.device))
        self.wq_down.copy_(q.reshape(E, H, I))
        self.sw_down.copy_(s.reshape(E, H))

    def forward(self, x2d, top_i, top_w):
        return _GroupedExpertsFn.apply(x2d, top_w, top_i, self.wq_gate_up, self.sw_gate_up,
                                       self.wq_down, self.sw_down)


class SparseMoe(nn.Module):
    def __init__(self, shape: MixtralShape, quantized: bool = True, device=None,
                 dtype=torch.bfloat16):
        super().__init__()
        self.gate = Router(shape, device, dtype)
        self.experts = W8A8Experts(shape, device) if quantized else FloatExperts(shape, device,
                                                                                  dtype)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        B, S, H = h.shape
        x2d = h.reshape(-1, H)
        _, top_w, top_i = self.gate(x2d)
        return self.experts(x2d, top_i, top_w).reshape(B, S, H)


class MixtralBlock(LlamaBlock):
    """Mixtral decoder layer: RMSNorm, GQA attention (W8A8 q/k/v/o), RMSNorm,
    sparse MoE with W8A8 experts, two residual adds. The attention half takes the
    fused producer path of LlamaBlock (RMSNorm -> quantise, stacked q/k/v GEMM,
    RoPE with the LoRA addends); the MoE half runs the bf16 router and the two
    grouped W8A8 GEMMs (SparseMoe)."""

    FUSABLE = ("q_proj", "k_proj", "v_proj", "o_proj")
    FUSED_GROUPS = (("qkv", ("q_proj", "k_proj", "v_proj")), ("o", ("o_proj",)))

    def __init__(self, shape: MixtralShape, quantized: bool = True, device=None,
                 dtype=torch.bfloat16):
        nn.Module.__init__(self)
        self.shape = shape
        self.input_layernorm = RMSNorm(shape.hidden, shape.eps, device, dtype)
        self.self_attn = LlamaAttention(shape, quantized, device, dtype)
        self.post_attention_layernorm = RMSNorm(shape.hidden, shape.eps, device, dtype)
        self.mlp = SparseMoe(shape, quantized, device, dtype)

    def projection(self, name: str) -> nn.Module:
        if name not in self.FUSABLE:
            raise KeyError(f"{name} is not a projection of a Mixtral block (the experts are "
                           "grouped tensors)")
        return getattr(self.self_attn, name)

    def _mlp_fused(self, h2):
        return h2 + self.mlp(self.post_attention_layernorm(h2))
