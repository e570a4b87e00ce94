"""The B200 W8A8 path behind the reference's ``backend="cpp"`` toggle.

The reference chooses its native memory manager with ``LemaConfig.backend``
(src/lema/_config.py:30): ``_tensorstore.py`` imports
``lema._csrc._lema_cpp`` (src/lema/_tensorstore.py:14-18) and, for ``"cpp"``,
streams layer weights through ``_lema_cpp.LemaMemoryManager``
(src/lema/_tensorstore.py:103-126). After ``enable()``, a model built with
``backend="cpp"`` on a CUDA device runs this library's path instead:

1. ``lema._csrc._lema_cpp`` is ``lema_b200._csrc._lema_cpp``: the same manager
   methods over the C ABI, so the weight segments stream through the native
   copy engine here;
2. the decoder layers' projections are ``W8A8Linear``. The adapter's
   name-based weight mapping (src/lema/adapters/_llama.py:118-151,
   src/lema/adapters/_gpt2.py:106-127) keeps each projection's offset into
   the streamed flat buffer, but its entry now quantises that slice of the
   buffer per output channel (K1, on the device) into the module's own int8
   weight and scales, where the reference copies bf16 values into an
   ``nn.Linear`` (src/lema/adapters/_llama.py:95-100). GPT-2's ``Conv1D``
   weights, stored [in, out], are transposed at that point. Fused MoE experts
   (Mixtral, LFM2: 3-D ``gate_up_proj`` / ``down_proj``) become
   ``W8A8Experts``, two grouped W8A8 GEMMs over the routed tokens, whose two
   mapping entries re-quantise each streamed copy the same way;
3. ``LemaTrainer.train_step`` keeps every streamed layer's input for the
   backward's recompute (src/lema/_trainer.py:109-111, 146-149). Those
   boundary activations now leave HBM: once a layer's no-grad forward is done,
   its input is copied to pinned host memory on a D2H stream (K5,
   ``lema_ckpt_save``) and its device storage is released; when the backward
   reaches that layer, the input was already brought back on an H2D stream
   while the layer after it was being recomputed.

``backend="python"`` and ``"auto"`` models are left exactly as the reference
builds them. Nothing here changes the reference's files: ``enable()`` wraps
``LemaModel.__init__`` and ``LemaModel.get_trainer`` and ``disable()`` puts
them back.
"""
from __future__ import annotations

import importlib
import sys

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as N
from .modules import W8A8Linear
from .moe import W8A8Experts

# Projections of each reference adapter's decoder layers that become W8A8
# (src/lema/adapters/_llama.py:41-57, _mistral.py, _mixtral.py attention,
# _gpt2.py:33-49, _lfm2.py:48-75: LFM2's attention q/k/v/out_proj, its short
# convolution's in_proj/out_proj and the dense layers' w1/w2/w3). Mixtral's and
# LFM2's experts are fused 3-D parameters: a decoder layer's ``experts`` module
# becomes W8A8Experts (grouped W8A8 GEMMs) instead. LFM2's depthwise
# convolution is a Conv1d and stays in the model dtype.
PROJECTIONS = {
    "LlamaAdapter": ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"),
    "MistralAdapter": ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                       "down_proj"),
    "MixtralAdapter": ("q_proj", "k_proj", "v_proj", "o_proj"),
    "GPT2Adapter": ("c_attn", "c_proj", "c_fc"),
    "Lfm2Adapter": ("q_proj", "k_proj", "v_proj", "out_proj", "in_proj", "w1", "w2", "w3"),
}

_saved: dict[str, object] = {}


def install_backend() -> None:
    """Makes ``lema._csrc._lema_cpp`` resolve to this library's manager (also
    when the reference's own extension was built and already imported)."""
    from ._csrc import _lema_cpp as shim
    sys.modules["lema._csrc._lema_cpp"] = shim
    pkg = importlib.import_module("lema._csrc")
    pkg._lema_cpp = shim
    ts = importlib.import_module("lema._tensorstore")
    ts._lema_cpp = shim
    ts.HAS_CPP_BACKEND = True


def enable() -> None:
    """Puts this library's path behind ``backend="cpp"`` for every ``LemaModel``
    built from now on (models already built are not changed)."""
    install_backend()
    model_mod = importlib.import_module("lema._model")
    cls = model_mod.LemaModel
    if "init" in _saved:
        return
    init, get_trainer = cls.__init__, cls.get_trainer
    _saved.update(init=init, get_trainer=get_trainer, cls=cls)

    def __init__(self, config):
        init(self, config)
        if self.config.backend == "cpp" and str(self.config.device).startswith("cuda"):
            attach_w8a8(self.adapter, self.full_ft_manager)

    def get_trainer_(self, *args, **kwargs):
        trainer = get_trainer(self, *args, **kwargs)
        if getattr(self.adapter, "_lema_b200_w8a8", None) is not None:
            attach_offload(trainer, self.config.device)
        return trainer

    cls.__init__ = __init__
    cls.get_trainer = get_trainer_


def disable() -> None:
    """Undoes ``enable()`` for models built afterwards."""
    if "init" not in _saved:
        return
    cls = _saved.pop("cls")
    cls.__init__ = _saved.pop("init")
    cls.get_trainer = _saved.pop("get_trainer")


# ---------------------------------------------------------------------------
# W8A8 projections bound to the streamed flat buffer
# ---------------------------------------------------------------------------

class _ExpertsPart:
    """One fused expert parameter (``gate_up_proj`` or ``down_proj``) of a
    W8A8Experts module, as the target of a mapping entry."""

    def __init__(self, experts, part: str):
        self.experts = experts
        self.part = part

    def requantize_(self, w: torch.Tensor) -> None:
        if self.part == "gate_up_proj":
            self.experts.requantize_gate_up_(w)
        else:
            self.experts.requantize_down_(w)


class _QuantizingSlot:
    """Takes a projection weight's place in the adapter's mapping
    (``(param, offset, numel, shape)`` entries): the adapter's
    ``param.data.copy_(flat_buffer[offset:offset + numel].view(shape))`` then
    quantises that view of the streamed buffer into the W8A8 module instead of
    copying it."""

    def __init__(self, module: W8A8Linear, transpose: bool):
        self.module = module
        self.transpose = transpose

    @property
    def data(self) -> "_QuantizingSlot":
        return self

    def copy_(self, src: torch.Tensor, non_blocking: bool = False) -> "_QuantizingSlot":
        self.module.requantize_(src.t() if self.transpose else src)
        return self


def _is_conv1d(m: nn.Module) -> bool:
    return type(m).__name__ == "Conv1D" and hasattr(m, "nf")


def _full_ft_names(full_ft) -> set[str]:
    """Parameter names (in the layer module) that selective full fine-tuning
    trains in any layer: those projections stay in the model dtype."""
    names: set[str] = set()
    for per_layer in getattr(full_ft, "module_name_to_key", {}).values():
        names.update(per_layer)
    return names


def _is_fused_experts(m: nn.Module) -> bool:
    """HF's fused-experts modules (MixtralExperts, Lfm2MoeExperts): 3-D
    gate_up_proj [E, 2I, H] and down_proj [E, H, I], SiLU gating."""
    gu, dn = getattr(m, "gate_up_proj", None), getattr(m, "down_proj", None)
    act = getattr(m, "act_fn", None)
    silu = act is F.silu or type(act).__name__ in ("SiLU", "SiLUActivation")
    return (isinstance(gu, nn.Parameter) and isinstance(dn, nn.Parameter) and gu.dim() == 3
            and dn.dim() == 3 and silu)


def _convert_experts(mapping, index, parent: nn.Module, cname: str, child: nn.Module,
                     full: str, keep: set[str]) -> None:
    """Replaces fused bf16 experts by grouped W8A8 experts (lema_grouped_w8a8_gemm)
    quantised from the weights just streamed; the two mapping entries then
    re-quantise each new streamed copy."""
    if f"{full}.gate_up_proj" in keep or f"{full}.down_proj" in keep:
        return
    entries = []
    for part in ("gate_up_proj", "down_proj"):
        i = index.get(id(getattr(child, part)))
        if i is None:
            raise N.LemaError(N.LEMA_ERR_UNSUPPORTED,
                              f"{full}.{part} is not in the adapter's weight mapping", "integrate")
        entries.append((part, i))
    experts = W8A8Experts.from_fused(child.gate_up_proj.detach(), child.down_proj.detach())
    for part, i in entries:
        _, off, numel, shape = mapping[i]
        mapping[i] = (_QuantizingSlot(_ExpertsPart(experts, part), False), off, numel, shape)
    setattr(parent, cname, experts)


def _convert(adapter, module: nn.Module, names: tuple[str, ...], keep: set[str]) -> None:
    mapping = adapter.param_mappings[id(module)]
    index = {id(param): i for i, (param, _, _, _) in enumerate(mapping)}
    for prefix, parent in list(module.named_modules()):
        for cname, child in list(parent.named_children()):
            if cname == "experts" and _is_fused_experts(child):
                _convert_experts(mapping, index, parent, cname, child,
                                 f"{prefix}.{cname}" if prefix else cname, keep)
                continue
            if cname not in names:
                continue
            wrapped = hasattr(child, "base_layer")
            base = child.base_layer if wrapped else child
            if isinstance(base, W8A8Linear):
                continue
            full = f"{prefix}.{cname}" if prefix else cname
            if f"{full}.weight" in keep or f"{full}.base_layer.weight" in keep:
                continue
            if _is_conv1d(base):
                q, transpose = W8A8Linear.from_conv1d(base), True
            elif isinstance(base, nn.Linear):
                q, transpose = W8A8Linear.from_float(base), False
                if base.bias is not None:
                    q.bias = base.bias  # the mapping keeps copying the streamed bias into it
            else:
                continue
            i = index.get(id(base.weight))
            if i is None:
                raise N.LemaError(N.LEMA_ERR_UNSUPPORTED,
                                  f"{full}.weight is not in the adapter's weight mapping",
                                  "integrate")
            _, off, numel, shape = mapping[i]
            mapping[i] = (_QuantizingSlot(q, transpose), off, numel, shape)
            setattr(child if wrapped else parent, "base_layer" if wrapped else cname, q)
    module._lema_b200_w8a8 = True


def attach_w8a8(adapter, full_ft=None) -> None:
    """Makes the decoder layers this adapter constructs from a CUDA flat buffer
    run W8A8 projections (see the module docstring)."""
    names = PROJECTIONS.get(type(adapter).__name__)
    if names is None:
        raise N.LemaError(N.LEMA_ERR_UNSUPPORTED,
                          f"no W8A8 projection list for {type(adapter).__name__}", "integrate")
    blocks = {m["id"] for m in adapter.get_layer_metadata() if m.get("type") == "block"}
    keep = _full_ft_names(full_ft) if full_ft is not None else set()
    construct = adapter.construct_layer_module

    def construct_layer_module(layer_id, flat_buffer=None, lora_manager=None,
                               full_ft_manager=None):
        module = construct(layer_id, flat_buffer, lora_manager, full_ft_manager)
        if (layer_id in blocks and flat_buffer is not None and flat_buffer.is_cuda
                and not getattr(module, "_lema_b200_w8a8", False)):
            # first use of this pooled module: the reference has just copied the
            # layer's weights into its projections; quantise them and route the
            # mapping's later copies into the quantiser
            _convert(adapter, module, names, keep)
        return module

    adapter.construct_layer_module = construct_layer_module
    adapter._lema_b200_w8a8 = names


# ---------------------------------------------------------------------------
# Boundary-activation offload under the reference's trainer
# ---------------------------------------------------------------------------

def _ev(e: torch.cuda.Event) -> int:
    return e.cuda_event


class _Offloaded:
    __slots__ = ("storage", "nbytes", "host", "saved", "restored")

    def __init__(self, storage, nbytes, host, saved):
        self.storage = storage
        self.nbytes = nbytes
        self.host = host
        self.saved = saved
        self.restored = None


class BoundaryOffload:
    """Keeps the reference trainer's boundary activations in pinned host memory
    between its forward and backward passes.

    The trainer holds each layer's input in a list (src/lema/_trainer.py:
    109-111) and passes it back to ``adapter.forward_layer`` for the recompute
    (:146-149). Wrapped around ``forward_layer``: after a no-grad forward the
    input (a float CUDA tensor that owns its whole storage) is copied to a
    pinned slot on the D2H stream and its storage is resized to zero, which
    frees the device memory for every alias, the trainer's list entry
    included; the caching allocator keeps the block until the copy has read it
    (``record_stream``). In the backward, layer by layer in reverse order, the
    input about to be recomputed is waited for and the one before it is
    restored on the H2D stream, so its copy overlaps this layer's recompute and
    backward. Inputs are matched by storage, last in first out, as the
    trainer's reverse loop consumes them."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.d2h = torch.cuda.Stream(self.device)
        self.h2d = torch.cuda.Stream(self.device)
        self.slots: list[torch.Tensor] = []
        self.stack: list[_Offloaded] = []
        self.active = False
        self.bytes_out = 0
        self.bytes_in = 0

    @staticmethod
    def _eligible(x) -> bool:
        return (isinstance(x, torch.Tensor) and x.is_cuda and x.is_floating_point()
                and x.numel() > 0 and x.is_contiguous() and x.storage_offset() == 0
                and x.untyped_storage().nbytes() == x.numel() * x.element_size())

    def _slot(self, i: int, nbytes: int) -> torch.Tensor:
        while len(self.slots) <= i:
            self.slots.append(torch.empty(0, dtype=torch.uint8))
        if self.slots[i].numel() < nbytes:
            self.slots[i] = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        return self.slots[i]

    def after_forward(self, x) -> None:
        if not self._eligible(x):
            return
        cur = torch.cuda.current_stream(self.device)
        nbytes = x.numel() * x.element_size()
        host = self._slot(len(self.stack), nbytes)
        ready, saved = torch.cuda.Event(), torch.cuda.Event()
        ready.record(cur)
        N.call("lema_ckpt_save", x.data_ptr(), host.data_ptr(), nbytes, 0, self.d2h.cuda_stream,
               _ev(ready), _ev(saved))
        x.record_stream(self.d2h)
        storage = x.untyped_storage()
        storage.resize_(0)
        self.stack.append(_Offloaded(storage, nbytes, host, saved))
        self.bytes_out += nbytes

    def _restore(self, e: _Offloaded) -> None:
        cur = torch.cuda.current_stream(self.device)
        e.storage.resize_(e.nbytes)  # device memory from the compute stream's pool
        alloc = torch.cuda.Event()
        alloc.record(cur)
        self.h2d.wait_event(e.saved)
        e.restored = torch.cuda.Event()
        N.call("lema_ckpt_restore", e.host.data_ptr(), e.storage.data_ptr(), e.nbytes,
               self.h2d.cuda_stream, _ev(alloc), _ev(e.restored))
        view = torch.empty(0, dtype=torch.uint8, device=self.device).set_(e.storage)
        view.record_stream(self.h2d)
        self.bytes_in += e.nbytes

    def before_recompute(self, x) -> None:
        if not self.stack or not isinstance(x, torch.Tensor):
            return
        e = self.stack[-1]
        if x.untyped_storage()._cdata != e.storage._cdata:
            return  # not an offloaded input (the token ids of the embedding layer)
        self.stack.pop()
        if e.restored is None:
            self._restore(e)
        torch.cuda.current_stream(self.device).wait_event(e.restored)
        if self.stack:
            self._restore(self.stack[-1])

    def reset(self) -> None:
        self.stack.clear()
        self.active = False


def attach_offload(trainer, device) -> BoundaryOffload:
    """Wraps the trainer's adapter ``forward_layer`` and ``train_step`` so the
    boundary activations of each training step live in pinned host memory."""
    off = BoundaryOffload(device)
    adapter = trainer.adapter
    forward_layer = adapter.forward_layer

    def forward_layer_(module, inputs, **kwargs):
        if not off.active:
            return forward_layer(module, inputs, **kwargs)
        x = inputs[0] if isinstance(inputs, tuple) else inputs
        if torch.is_grad_enabled():
            off.before_recompute(x)
            return forward_layer(module, inputs, **kwargs)
        y = forward_layer(module, inputs, **kwargs)
        off.after_forward(x)
        return y

    train_step = trainer.train_step

    def train_step_(*args, **kwargs):
        off.active = True
        try:
            return train_step(*args, **kwargs)
        finally:
            off.reset()

    adapter.forward_layer = forward_layer_
    trainer.train_step = train_step_
    trainer.boundary_offload = off
    return off
