"""nn.Module drop-ins for the projections of a streamed decoder layer.

``W8A8Linear`` replaces the ``nn.Linear`` base layers that HF
``LlamaDecoderLayer`` / ``MistralDecoderLayer`` create (reference
src/lema/adapters/_llama.py:80) and the adapters call
(src/lema/adapters/_llama.py:245-250). It subclasses ``nn.Linear`` so the
reference's LoRA injection, which wraps modules by ``isinstance(child,
nn.Linear)`` and reads ``in_features`` / ``out_features``
(src/lema/_lora.py:51-57), keeps working on it unchanged.

``LoRALinear`` is the same computation as the reference's ``LoRAWrapper``
(src/lema/_lora.py:13-26): ``base(x) + (x @ A^T @ B^T) * alpha / r``, with A
kaiming-uniform(a=sqrt(5)) and B zero at init (src/lema/_lora.py:38-49).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import ops


class W8A8Linear(nn.Linear):
    """Frozen W8A8 projection: int8 per-output-channel weights + fp32 scales.

    Parameters / buffers (names kept so name-based weight binding still works):
      weight        int8 [out_features, in_features] (frozen nn.Parameter)
      weight_scale  fp32 [out_features]
      bias          bf16 [out_features] or None

    ``forward(x)`` takes [..., in_features] in any float dtype, computes in bf16
    through the sm_100a kernels and returns the input dtype.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 device: torch.device | str | None = None):
        nn.Module.__init__(self)
        self.in_features = in_features
        self.out_features = out_features
        ldw = ops.pad_to(max(in_features, 1), 16)
        store = torch.zeros(out_features, ldw, dtype=torch.int8, device=device)
        self.weight = nn.Parameter(store[:, :in_features], requires_grad=False)
        self.register_buffer("weight_scale",
                             torch.ones(out_features, dtype=torch.float32, device=device))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16, device=device))
        else:
            self.register_parameter("bias", None)

    @classmethod
    def from_float(cls, linear: nn.Linear, device: torch.device | str | None = None
                   ) -> "W8A8Linear":
        """Quantises an nn.Linear's weight per output channel on the GPU."""
        dev = torch.device(device) if device is not None else linear.weight.device
        if dev.type != "cuda":
            raise RuntimeError("W8A8Linear.from_float quantises on a CUDA device")
        m = cls(linear.in_features, linear.out_features, bias=linear.bias is not None, device=dev)
        m.load_float_weight(linear.weight.detach().to(dev))
        if linear.bias is not None:
            m.bias.data.copy_(linear.bias.detach().to(dev, torch.bfloat16))
        return m

    @classmethod
    def from_conv1d(cls, conv: nn.Module, device: torch.device | str | None = None
                    ) -> "W8A8Linear":
        """Quantises a GPT-2 ``Conv1D`` (transformers.pytorch_utils; weight stored
        [in, out], y = x W + b) per output channel: its weight is transposed to the
        nn.Linear orientation [out, in] first (the pack-time transpose the GPT-2
        adapter's weights need, src/lema/adapters/_gpt2.py:33-49). The bias
        Parameter object is kept, so a name-based weight binding that copies
        into it keeps working."""
        dev = torch.device(device) if device is not None else conv.weight.device
        if dev.type != "cuda":
            raise RuntimeError("W8A8Linear.from_conv1d quantises on a CUDA device")
        in_f, out_f = conv.weight.shape
        m = cls(in_f, out_f, bias=False, device=dev)
        m.requantize_(conv.weight.detach().to(dev).t())
        if getattr(conv, "bias", None) is not None:
            m.bias = conv.bias
        return m

    @torch.no_grad()
    def requantize_(self, w: torch.Tensor) -> None:
        """Quantises a float weight [out, in] (any strides; e.g. a slice of a
        streamed flat buffer, or a transposed Conv1D weight) per output channel
        into this module's own int8 weight and scales, in place (K1)."""
        if tuple(w.shape) != (self.out_features, self.in_features):
            raise ValueError(f"weight of shape {tuple(w.shape)} for a "
                             f"[{self.out_features}, {self.in_features}] projection")
        if w.dtype not in (torch.bfloat16, torch.float32):
            w = w.to(torch.bfloat16)
        q = self.weight.data
        if q.stride(1) != 1 or q.stride(0) % 16 or q.data_ptr() % 16:
            ldw = ops.pad_to(max(self.in_features, 1), 16)
            q = torch.zeros(self.out_features, ldw, dtype=torch.int8, device=w.device)
            q = q[:, :self.in_features]
            self.weight.data = q
        if self.weight_scale.stride(0) != 1:
            self.weight_scale = torch.empty(self.out_features, dtype=torch.float32,
                                            device=w.device)
        ops.quantize_rows(w, out=q, scale=self.weight_scale)

    @torch.no_grad()
    def load_float_weight(self, w: torch.Tensor) -> None:
        """Re-quantises from a float weight [out, in] (e.g. after an optimizer step)."""
        wq, sw = ops.quantize_weight(w)
        self.weight.data = wq
        self.weight_scale = sw

    def bind(self, wq: torch.Tensor, sw: torch.Tensor, bias: torch.Tensor | None = None) -> None:
        """Points the module at int8 weights / scales living elsewhere (a streamed
        VRAM slot) without copying."""
        if wq.shape != (self.out_features, self.in_features) or wq.dtype != torch.int8:
            raise ValueError(f"bad weight view {tuple(wq.shape)} {wq.dtype}")
        self.weight.data = wq
        self.weight_scale = sw
        if bias is not None:
            self.bias.data = bias

    # Selective full fine-tuning: when ``wgrad_acc`` (fp32 [out, in]) is set, the
    # backward also adds the weight gradient dy^T . x into it.
    wgrad_acc: torch.Tensor | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.wgrad_acc is not None and torch.is_grad_enabled() and self.bias is None:
            return ops.w8a8_linear_trainable(x, self.weight, self.weight_scale, self)
        return ops.w8a8_linear(x, self.weight, self.weight_scale, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, w8a8")


class LoRALinear(nn.Module):
    """``base(x) + (x @ A^T @ B^T) * (alpha / r)`` around a (W8A8) base layer."""

    def __init__(self, base_layer: nn.Module, rank: int, alpha: float,
                 lora_A: nn.Parameter | None = None, lora_B: nn.Parameter | None = None,
                 dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.base_layer = base_layer
        self.rank = rank
        self.alpha = alpha
        self.scaling = alpha / rank
        dev = next(iter(base_layer.buffers()), base_layer.weight).device
        if lora_A is None:
            a = torch.zeros(rank, base_layer.in_features, device=dev, dtype=dtype)
            nn.init.kaiming_uniform_(a, a=math.sqrt(5))
            lora_A = nn.Parameter(a)
        if lora_B is None:
            lora_B = nn.Parameter(torch.zeros(base_layer.out_features, rank, device=dev, dtype=dtype))
        self.lora_A = lora_A
        self.lora_B = lora_B

    @property
    def in_features(self) -> int:
        return self.base_layer.in_features

    @property
    def out_features(self) -> int:
        return self.base_layer.out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        result = self.base_layer(x)
        lora_out = (x @ self.lora_A.transpose(0, 1) @ self.lora_B.transpose(0, 1)) * self.scaling
        return result + lora_out
