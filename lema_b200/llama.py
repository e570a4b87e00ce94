"""Llama decoder block with W8A8 projections, as streamed by the trainer.

The math mirrors HF ``LlamaDecoderLayer`` as the reference adapter drives it
(src/lema/adapters/_llama.py:236-252): RMSNorm computed in fp32 and cast back
before the weight multiply, RoPE with cos/sin built in fp32 from
``theta ** (-2i/d)``, causal attention with scale ``head_dim ** -0.5``,
SwiGLU MLP ``down(silu(gate(x)) * up(x))``, two residual adds. Parameter
names match HF (``self_attn.q_proj.weight``, ``mlp.down_proj.weight``, ...) so
checkpoints and the reference's name-based weight mapping
(src/lema/adapters/_llama.py:41-57, 118-151) line up.

Attention runs through ``torch.nn.functional.scaled_dot_product_attention``
with ``is_causal=True`` (bf16 flash kernel on the GPU) by default; with
``attn_impl = "tcgen05"`` (opt-in, head_dim 128) it runs on this library's own
tensor-core kernels (``ops.AttentionFn``) straight from the token-major q / k / v.
It is not part of the W8A8 path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .modules import LoRALinear, W8A8Linear

PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


@dataclass(frozen=True)
class LlamaShape:
    """Architecture sizes (Llama-2-7B defaults)."""

    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 32
    intermediate: int = 11008
    vocab: int = 32000
    layers: int = 32
    eps: float = 1e-5
    theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def proj_shapes(self) -> dict[str, tuple[int, int]]:
        """name -> (out_features, in_features) of each projection."""
        hd = self.head_dim
        return {
            "q_proj": (self.heads * hd, self.hidden),
            "k_proj": (self.kv_heads * hd, self.hidden),
            "v_proj": (self.kv_heads * hd, self.hidden),
            "o_proj": (self.hidden, self.heads * hd),
            "gate_proj": (self.intermediate, self.hidden),
            "up_proj": (self.intermediate, self.hidden),
            "down_proj": (self.hidden, self.intermediate),
        }

    def linear_params_per_block(self) -> int:
        return sum(o * i for o, i in self.proj_shapes().values())


class RMSNorm(nn.Module):
    def __init__(self, hidden: int, eps: float, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden, device=device, dtype=dtype))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        in_dtype = x.dtype
        h = x.to(torch.float32)
        var = h.pow(2).mean(-1, keepdim=True)
        h = h * torch.rsqrt(var + self.variance_epsilon)
        return self.weight * h.to(in_dtype)


def rope_cos_sin(shape: LlamaShape, seq_len: int, device, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [1, seq, head_dim] for positions 0..seq-1 (computed in fp32)."""
    d = shape.head_dim
    inv_freq = 1.0 / (shape.theta ** (torch.arange(0, d, 2, dtype=torch.int64, device=device)
                                      .to(torch.float32) / d))
    pos = torch.arange(seq_len, device=device, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype)[None], emb.sin().to(dtype)[None]


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rope(q, k, cos, sin):
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return (q * cos) + (_rotate_half(q) * sin), (k * cos) + (_rotate_half(k) * sin)


def _linear(out_f: int, in_f: int, quantized: bool, device, dtype) -> nn.Module:
    if quantized:
        return W8A8Linear(in_f, out_f, bias=False, device=device)
    return nn.Linear(in_f, out_f, bias=False, device=device, dtype=dtype)


def _eager_causal_attention(q, k, v, scale):
    """HF eager attention with the reference adapter's additive fp32 causal mask
    (src/lema/adapters/_llama.py:202-205): softmax in fp32, cast back to q's dtype."""
    rep = q.shape[1] // k.shape[1]
    if rep > 1:
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    S = q.shape[2]
    mask = torch.full((S, S), float("-inf"), device=q.device).triu(1)
    w = torch.matmul(q, k.transpose(2, 3)) * scale + mask
    w = torch.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(w, v)


def _chunked_causal_attention(q, k, v, scale, chunk, gqa):
    """Exact causal attention computed one query chunk at a time against all keys
    up to the chunk's end, as the reference's chunked attention does (full score
    rows per query chunk, src/lema/_tensorstore.py:565-608), with a lower-right
    aligned causal mask inside each chunk."""
    from torch.nn.attention.bias import causal_lower_right
    S = q.shape[2]
    outs = []
    for c0 in range(0, S, chunk):
        c1 = min(S, c0 + chunk)
        mask = causal_lower_right(c1 - c0, c1)
        outs.append(F.scaled_dot_product_attention(q[:, :, c0:c1], k[:, :, :c1], v[:, :, :c1],
                                                   attn_mask=mask, scale=scale, enable_gqa=gqa))
    return torch.cat(outs, dim=2)


def _tc_attention(q2d, k2d, v2d, B: int, S: int, shape: LlamaShape) -> torch.Tensor:
    """Causal attention of token-major q [B*S, H*d], k / v [B*S, Hkv*d] on the
    tcgen05 kernels; returns o [B*S, H*d]."""
    if shape.head_dim != 128:
        raise ValueError(f"attn_impl='tcgen05' needs head_dim 128, got {shape.head_dim}")
    from . import ops
    return ops.AttentionFn.apply(q2d, k2d, v2d, B, S, shape.heads, shape.kv_heads,
                                 shape.head_dim ** -0.5)


class LlamaAttention(nn.Module):
    def __init__(self, shape: LlamaShape, quantized: bool, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.shape = shape
        # "sdpa"; "eager" reproduces HF eager attention op for op; "tcgen05" runs
        # this library's attention kernels (head_dim 128)
        self.attn_impl = "sdpa"
        self.attn_chunk = 0      # > 0: exact attention in query chunks of this many tokens
        ps = shape.proj_shapes()
        for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, n, _linear(*ps[n], quantized, device, dtype))

    def forward(self, h: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        B, S, _ = h.shape
        d = self.shape.head_dim
        q = self.q_proj(h).view(B, S, -1, d).transpose(1, 2)
        k = self.k_proj(h).view(B, S, -1, d).transpose(1, 2)
        v = self.v_proj(h).view(B, S, -1, d).transpose(1, 2)
        q, k = apply_rope(q, k, cos, sin)
        if self.attn_impl == "tcgen05":
            o2d = _tc_attention(q.transpose(1, 2).reshape(B * S, -1),
                                k.transpose(1, 2).reshape(B * S, -1),
                                v.transpose(1, 2).reshape(B * S, -1), B, S, self.shape)
            return self.o_proj(o2d.view(B, S, -1))
        if self.attn_impl == "eager":
            o = _eager_causal_attention(q, k, v, d ** -0.5)
        elif self.attn_chunk and S > self.attn_chunk:
            o = _chunked_causal_attention(q, k, v, d ** -0.5, self.attn_chunk,
                                          self.shape.heads != self.shape.kv_heads)
        else:
            gqa = self.shape.heads != self.shape.kv_heads
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=d ** -0.5,
                                               enable_gqa=gqa)
        o = o.transpose(1, 2).reshape(B, S, -1)
        return self.o_proj(o)


class LlamaMLP(nn.Module):
    def __init__(self, shape: LlamaShape, quantized: bool, device=None, dtype=torch.bfloat16):
        super().__init__()
        ps = shape.proj_shapes()
        for n in ("gate_proj", "up_proj", "down_proj"):
            setattr(self, n, _linear(*ps[n], quantized, device, dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class LlamaBlock(nn.Module):
    """One decoder layer; ``quantized`` selects W8A8Linear or nn.Linear projections."""

    def __init__(self, shape: LlamaShape, quantized: bool = True, device=None,
                 dtype=torch.bfloat16):
        super().__init__()
        self.shape = shape
        self.input_layernorm = RMSNorm(shape.hidden, shape.eps, device, dtype)
        self.self_attn = LlamaAttention(shape, quantized, device, dtype)
        self.post_attention_layernorm = RMSNorm(shape.hidden, shape.eps, device, dtype)
        self.mlp = LlamaMLP(shape, quantized, device, dtype)

    def projection(self, name: str) -> nn.Module:
        parent = self.self_attn if name in ("q_proj", "k_proj", "v_proj", "o_proj") else self.mlp
        return getattr(parent, name)

    def base_projection(self, name: str) -> nn.Module:
        m = self.projection(name)
        return m.base_layer if isinstance(m, LoRALinear) else m

    gradient_checkpointing = False
    # Stacked int8 weights / scales of the projection groups ("qkv", "o", "gate_up",
    # "down" + ".wq" / ".sw"), set when the block is bound to a weight segment.
    fused_weights: dict | None = None
    use_fused = True
    # W8A8 projections of this block type (the fused path covers all of them)
    FUSABLE = PROJECTIONS
    FUSED_GROUPS = (("qkv", ("q_proj", "k_proj", "v_proj")), ("o", ("o_proj",)),
                    ("gate_up", ("gate_proj", "up_proj")), ("down", ("down_proj",)))

    def _can_fuse(self) -> bool:
        if not (self.use_fused and self.fused_weights is not None):
            return False
        if self.gradient_checkpointing or self.self_attn.attn_impl not in ("sdpa", "tcgen05"):
            return False
        for name in self.FUSABLE:
            m = self.projection(name)
            if getattr(self.base_projection(name), "wgrad_acc", None) is not None:
                return False  # trainable projections take the per-projection path
            if isinstance(m, LoRALinear) and name in ("o_proj", "gate_proj", "up_proj",
                                                      "down_proj"):
                return False
        return True

    def forward(self, h: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        if h.is_cuda and self._can_fuse():
            return self._forward_fused(h, cos, sin)
        residual = h
        h = self.input_layernorm(h)
        if self.gradient_checkpointing and torch.is_grad_enabled():
            # attention is re-run in backward instead of keeping its activations,
            # as the reference adapter does (src/lema/adapters/_llama.py:239-243)
            from torch.utils.checkpoint import checkpoint
            h = checkpoint(self.self_attn, h, cos, sin, use_reentrant=False)
        else:
            h = self.self_attn(h, cos, sin)
        h = residual + h
        residual = h
        h = self.post_attention_layernorm(h)
        h = self.mlp(h)
        return residual + h


    @torch.no_grad()
    def build_fused_weights(self) -> None:
        """Stacks this block's own W8A8 projections into the group tensors of the
        fused path (a copy; streamed blocks get views of their segment instead)."""
        def cat(names, what):
            return torch.cat([getattr(self.base_projection(n), what) for n in names], dim=0)
        self.fused_weights = {}
        for group, names in self.FUSED_GROUPS:
            self.fused_weights[group + ".wq"] = cat(names, "weight").contiguous()
            self.fused_weights[group + ".sw"] = cat(names, "weight_scale").contiguous()

    def _forward_fused(self, h, cos, sin):
        """The same layer through the fused producers: RMSNorm -> quantise (one
        kernel), one stacked q/k/v W8A8 GEMM, one kernel adding the LoRA outputs,
        rotating q/k and laying v out contiguously, SDPA,
        o_proj, residual, RMSNorm -> quantise, stacked gate/up GEMM, SwiGLU ->
        quantise (one kernel), down GEMM, residual."""
        return self._mlp_fused(self._attention_fused(h, cos, sin))

    def _attention_fused(self, h, cos, sin):
        """h + attention(input_layernorm(h)) through the fused producers."""
        from . import ops
        sh = self.shape
        B, S, H = h.shape
        d = sh.head_dim
        nq, nk = sh.heads * d, sh.kv_heads * d
        fw = self.fused_weights
        x2d = h.reshape(-1, H)
        hn, xq, sx = ops.RMSNormQuantFn.apply(x2d, self.input_layernorm.weight, sh.eps)
        q, k, v = ops.QKVFn.apply(hn, xq, sx, fw["qkv.wq"], fw["qkv.sw"], nq, nk)
        att = self.self_attn
        lora = []
        for name in ("q_proj", "k_proj", "v_proj"):
            m = getattr(att, name)
            lora.append((hn @ m.lora_A.transpose(0, 1) @ m.lora_B.transpose(0, 1)) * m.scaling
                        if isinstance(m, LoRALinear) else None)
        qr, kr, vc = ops.RopeQKVFn.apply(q, k, v, *lora, cos.reshape(-1, d), sin.reshape(-1, d),
                                         S, sh.heads, sh.kv_heads, d)
        qv = qr.view(B, S, sh.heads, d).transpose(1, 2)
        kv = kr.view(B, S, sh.kv_heads, d).transpose(1, 2)
        vv = vc.view(B, S, sh.kv_heads, d).transpose(1, 2)
        if att.attn_impl == "tcgen05":  # exact at any length: no query chunks needed
            return h + att.o_proj(_tc_attention(qr, kr, vc, B, S, sh)).view(B, S, H)
        gqa = sh.heads != sh.kv_heads
        if att.attn_chunk and S > att.attn_chunk:
            o = _chunked_causal_attention(qv, kv, vv, d ** -0.5, att.attn_chunk, gqa)
        else:
            o = F.scaled_dot_product_attention(qv, kv, vv, is_causal=True, scale=d ** -0.5,
                                               enable_gqa=gqa)
        o2d = o.transpose(1, 2).reshape(B * S, nq)
        return h + att.o_proj(o2d).view(B, S, H)

    def _mlp_fused(self, h2):
        """h2 + mlp(post_attention_layernorm(h2)): RMSNorm -> quantise, stacked
        gate/up GEMM, SwiGLU -> quantise, down GEMM."""
        from . import ops
        sh = self.shape
        B, S, H = h2.shape
        fw = self.fused_weights
        hn2, xq2, sx2 = ops.RMSNormQuantFn.apply(h2.reshape(-1, H),
                                                 self.post_attention_layernorm.weight, sh.eps)
        y = ops.MLPFn.apply(hn2, xq2, sx2, fw["gate_up.wq"], fw["gate_up.sw"], fw["down.wq"],
                            fw["down.sw"])
        return h2 + y.view(B, S, H)


def apply_lora(block: LlamaBlock, rank: int, alpha: float,
               targets: tuple[str, ...] = ("q_proj", "v_proj"),
               params: dict[str, tuple[nn.Parameter, nn.Parameter]] | None = None,
               dtype: torch.dtype = torch.bfloat16) -> dict[str, tuple[nn.Parameter, nn.Parameter]]:
    """Wraps the target projections with LoRALinear (reusing ``params`` when given,
    as the reference LoRAManager keeps one (A, B) pair per layer and module,
    src/lema/_lora.py:38-49). Returns name -> (A, B)."""
    out = {}
    for name in targets:
        parent = block.self_attn if name in ("q_proj", "k_proj", "v_proj", "o_proj") else block.mlp
        cur = getattr(parent, name)
        base = cur.base_layer if isinstance(cur, LoRALinear) else cur
        a, b = (params or {}).get(name, (None, None))
        w = LoRALinear(base, rank, alpha, a, b, dtype=dtype)
        setattr(parent, name, w)
        out[name] = (w.lora_A, w.lora_B)
    return out


class LlamaHead(nn.Module):
    """Final RMSNorm + lm_head (bf16 nn.Linear; not a W8A8 projection)."""

    def __init__(self, shape: LlamaShape, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.norm = RMSNorm(shape.hidden, shape.eps, device, dtype)
        self.lm_head = nn.Linear(shape.hidden, shape.vocab, bias=False, device=device, dtype=dtype)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        return self.lm_head(self.norm(h))
