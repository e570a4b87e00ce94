"""CPU torch modules built on the W8A8 oracle — TEST INFRASTRUCTURE ONLY.

``OracleW8A8Linear`` is an ``nn.Linear`` whose forward is the oracle's W8A8
contract (quantise the bf16 input per token and the weight per output
channel, exact int8 GEMM, fp32 dequant epilogue, bf16 out) and whose backward
is the straight-through dgrad ``dx = dy . bf16(wq * sw)`` with fp32
accumulation. It is swapped into the reference's own HF layers (via the
reference adapter, src/lema/adapters/_llama.py:59-107, and LoRAWrapper,
src/lema/_lora.py:13-26) to produce golden fixtures, and into
lema_b200.llama.LlamaBlock on the CPU to form the layer-level oracle.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from . import oracle as O


def _bits(t: torch.Tensor) -> np.ndarray:
    return O.torch_bf16_to_bits(t.detach().to(torch.bfloat16))


class _OracleFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, mod, bias):
        xq, sx = O.c_quantize_rows(_bits(x2d))
        acc = O.c_int8_gemm(xq, mod.wq)
        b = None if bias is None else _bits(bias)
        y = O.bits_to_torch_bf16(O.c_epilogue(acc, sx, mod.sw, b))
        ctx.mod = mod
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        dyb = dy.to(torch.bfloat16).float()
        dx = (dyb @ ctx.mod.wdeq_f32()).to(torch.bfloat16)
        db = dy.float().sum(0).to(torch.bfloat16) if ctx.has_bias else None
        return dx, None, db


class OracleW8A8Linear(nn.Linear):
    """CPU W8A8 linear (oracle arithmetic), frozen base, STE backward."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None):
        out_f, in_f = weight.shape
        nn.Module.__init__(self)
        self.in_features = in_f
        self.out_features = out_f
        self.weight = nn.Parameter(weight.detach().to(torch.bfloat16).clone(), requires_grad=False)
        self.bias = None if bias is None else nn.Parameter(bias.detach().to(torch.bfloat16).clone(),
                                                           requires_grad=False)
        self.wq, self.sw = O.c_quantize_rows(_bits(self.weight))
        self._wdeq = None

    def wdeq_f32(self) -> torch.Tensor:
        """fp32 copy of bf16(wq * sw) [out, in] (the frozen weight: built once)."""
        if self._wdeq is None:
            wdT = O.c_dequant_transpose(self.wq, self.sw)
            self._wdeq = O.bits_to_torch_bf16(np.ascontiguousarray(wdT.T)).float()
        return self._wdeq

    @classmethod
    def from_linear(cls, lin: nn.Linear) -> "OracleW8A8Linear":
        return cls(lin.weight, lin.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        K = x.shape[-1]
        y = _OracleFn.apply(x.reshape(-1, K), self, self.bias)
        return y.reshape(*x.shape[:-1], self.out_features).to(x.dtype)


def swap_linears(module: nn.Module, names=("q_proj", "k_proj", "v_proj", "o_proj",
                                           "gate_proj", "up_proj", "down_proj")) -> None:
    """Replaces every nn.Linear named in ``names`` (or the ``base_layer`` of a LoRA
    wrapper with that name) by an OracleW8A8Linear holding the same weight."""
    for parent in list(module.modules()):
        for name, child in list(parent.named_children()):
            if name not in names:
                continue
            if hasattr(child, "base_layer") and isinstance(child.base_layer, nn.Linear):
                if not isinstance(child.base_layer, OracleW8A8Linear):
                    child.base_layer = OracleW8A8Linear.from_linear(child.base_layer)
            elif isinstance(child, nn.Linear) and not isinstance(child, OracleW8A8Linear):
                setattr(parent, name, OracleW8A8Linear.from_linear(child))


class OracleExperts(nn.Module):
    """CPU MoE experts on the oracle's W8A8 arithmetic, looping over experts the
    way HF MixtralExperts does: per expert, OracleW8A8Linear(gate_up[e]) on the
    routed token rows, silu(gate) * up, OracleW8A8Linear(down[e]), times the
    routing weight (fp32), cast to bf16, index_add into the output."""

    def __init__(self, gate_up: torch.Tensor, down: torch.Tensor):
        super().__init__()
        self.gu = nn.ModuleList(OracleW8A8Linear(gate_up[e]) for e in range(gate_up.shape[0]))
        self.dn = nn.ModuleList(OracleW8A8Linear(down[e]) for e in range(down.shape[0]))

    def forward(self, x2d, top_i, top_w):
        final = torch.zeros_like(x2d)
        E = len(self.gu)
        mask = torch.nn.functional.one_hot(top_i, num_classes=E).permute(2, 1, 0)
        for e in range(E):
            pos, tok = torch.where(mask[e])
            if tok.numel() == 0:
                continue
            gate, up = self.gu[e](x2d[tok]).chunk(2, dim=-1)
            h = self.dn[e](torch.nn.functional.silu(gate) * up)
            h = h * top_w[tok, pos, None]
            final.index_add_(0, tok, h.to(final.dtype))
        return final


def chunked_causal_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 scale: float, chunk: int) -> torch.Tensor:
    """The reference's chunked causal attention as its RoPE adapters drive it
    (src/lema/adapters/_chunked_rope.py:63-117 calling
    src/lema/_tensorstore.py:565-608), restated: K and V expanded to every
    query head (GQA); for query chunk c, the fp32 scores against key chunks
    0..c are concatenated along the key axis and scaled, keys after the query
    position are set to finfo(fp32).min, the softmax runs in fp32 as max, exp,
    sum and divide, the weights multiply the concatenated V in fp32 and the
    result is cast to q's dtype. q [B, H, S, D], k/v [B, Hkv, S, D]."""
    rep = q.shape[1] // k.shape[1]
    if rep > 1:
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    S = q.shape[2]
    outs = []
    for s in range(0, S, chunk):
        e = min(s + chunk, S)
        qf = q[:, :, s:e].float()
        parts = [qf @ k[:, :, c0:min(c0 + chunk, S)].float().transpose(-2, -1)
                 for c0 in range(0, e, chunk)]
        scores = torch.cat(parts, dim=-1) * scale
        q_pos = torch.arange(s, e, device=q.device)
        k_pos = torch.arange(0, scores.shape[-1], device=q.device)
        masked = (q_pos[:, None] < k_pos[None, :])[None, None]
        scores = torch.where(masked, torch.full_like(scores, torch.finfo(scores.dtype).min),
                             scores)
        m = scores.max(dim=-1, keepdim=True).values
        p = (scores - m).exp()
        p = p / p.sum(dim=-1, keepdim=True)
        outs.append((p @ v[:, :, :e].float()).to(q.dtype))
    return torch.cat(outs, dim=2)


def adamw_step_ref(w_bf16: np.ndarray, g: np.ndarray, m: np.ndarray, v: np.ndarray, step: int,
                   lr: float, wd: float) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """numpy fp32 restatement of the reference's per-layer AdamW
    (src/lema/_full_ft.py:204-229): decoupled weight decay, bias-corrected
    moments, eps 1e-8, the update in fp32, the weight stored back in bf16.
    w_bf16 is bf16 bits; returns (new weight bits, m, v)."""
    beta1, beta2, eps = np.float32(0.9), np.float32(0.999), np.float32(1e-8)
    b1 = 1 - 0.9 ** step
    b2 = 1 - 0.999 ** step
    w = O.bf16_bits_to_f32(w_bf16).astype(np.float32)
    g = g.astype(np.float32)
    if wd:
        w = (w * np.float32(1 - lr * wd)).astype(np.float32)
    m = (m * beta1 + g * np.float32(1 - 0.9)).astype(np.float32)
    v = (v * beta2 + g * g * np.float32(1 - 0.999)).astype(np.float32)
    denom = (np.sqrt(v) / np.float32(np.sqrt(b2)) + eps).astype(np.float32)
    w = (w + np.float32(-(lr / b1)) * (m / denom)).astype(np.float32)
    return O.f32_to_bf16_bits(w), m, v
