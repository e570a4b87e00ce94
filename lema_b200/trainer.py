"""Layer-streamed LoRA training over W8A8 decoder blocks.

``StreamedLoraTrainer.train_step`` follows ``LemaTrainer.train_step``
(src/lema/_trainer.py:75-194) step for step, on the B200 data path:

* forward, no grad (reference :93-116): block i's int8 segment is uploaded
  from pinned RAM into one of two VRAM slots by the native manager's copy
  stream while block i-1 computes; the block's W8A8 projections are bound to
  views of the slot (no parameter copy, unlike src/lema/adapters/_llama.py:
  95-100); the block's input is saved to a pinned host slot on a D2H stream
  (``ckpt_mode`` 0, the default; 1 saves through the SM store kernel). The
  reference keeps it in VRAM (:109-111): ``ckpt_mode=2`` does that for every
  layer, and ``ckpt_mode=None`` for as many layers as fit ``ckpt_hbm_budget``
  bytes (by default a quarter of the memory free when the trainer is built),
  offloading only the rest;
* head + loss (reference :151-162): final RMSNorm, bf16 lm_head, shifted
  cross entropy, backward to the last hidden state;
* backward in reverse (reference :125-173): the saved input is restored on the
  H2D stream, the block is re-run with grad and back-propagated; the two
  blocks still resident at the turnaround are reused without re-upload; each
  finished layer's LoRA gradients start their data-parallel all-reduce
  (NCCL) while the next layer computes;
* selective full fine-tuning (reference :169-181, src/lema/_full_ft.py) of
  chosen projections of chosen layers, see ``full_ft.SelectiveFullFT``: each
  selected layer is clipped and stepped on a side stream as soon as its own
  backward is done (the reference does the same per-layer arithmetic after
  the whole backward);
* optimizer (reference :183-187): every ``grad_accum`` micro-steps (the loss
  is divided by ``grad_accum`` as at reference :156), clip_grad_norm_(1.0) and
  AdamW over the LoRA parameters; with data parallelism the LoRA gradients
  are averaged over ranks on that micro-step.

Every cross-stream dependency is a CUDA event; the host never blocks on a
transfer. The embedding and the head stay resident in HBM (they are frozen and
small next to 180 GB); the 32 blocks stream.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .llama import LlamaBlock, LlamaHead, LlamaShape, apply_lora, rope_cos_sin
from .tensorstore import ActivationCheckpointStore, WeightSegments


class LoraGradReducer:
    """Averages LoRA gradients over a process group, one flat fp32 bucket per
    layer, launched asynchronously as each layer's backward finishes."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self._pending: list[tuple[object, torch.Tensor, list[torch.Tensor]]] = []

    def launch(self, grads: list[torch.Tensor]):
        """Starts the all-reduce of one bucket; returns its entry (None when there
        is nothing to reduce)."""
        if self.world == 1 or not grads:
            return None
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        work = self.dist.all_reduce(flat, op=self.dist.ReduceOp.SUM, group=self.group,
                                    async_op=True)
        entry = (work, flat, grads)
        self._pending.append(entry)
        return entry

    def finish(self, entry=None) -> None:
        """Makes the current stream wait for the bucket(s) and writes the averages
        back into the gradients: one entry, or every pending one."""
        entries = list(self._pending) if entry is None else [entry]
        cur = torch.cuda.current_stream() if torch.cuda.is_available() else None
        for e in entries:
            work, flat, grads = e
            work.wait()
            if cur is not None and flat.is_cuda:
                flat.record_stream(cur)
            flat.div_(self.world)
            off = 0
            for g in grads:
                n = g.numel()
                g.copy_(flat[off:off + n].view_as(g))
                off += n
            self._pending.remove(e)


class StreamedLoraTrainer:
    def __init__(self, shape: LlamaShape, device, batch: int, seq: int, lora_rank: int = 16,
                 lora_alpha: float = 32.0, targets: tuple[str, ...] = ("q_proj", "v_proj"),
                 lr: float = 1e-4, weight_decay: float = 0.01, seed: int = 0,
                 ckpt_mode: int | None = 0, ckpt_hbm_budget: int | None = None,
                 resident_layers: int = 0, grad_accum: int = 1,
                 gradient_checkpointing: bool = False, attn_chunk: int = 0,
                 full_ft_layers: tuple[int, ...] = (),
                 full_ft_modules: tuple[str, ...] = ("q_proj", "k_proj", "v_proj", "o_proj"),
                 group=None, weight_shard: bool = False, vram_slots: int = 2,
                 weights: str | None = None, attn_impl: str = "sdpa"):
        self.shape = shape
        self.device = torch.device(device)
        self.batch, self.seq = batch, seq
        self.L = shape.layers
        self.targets = targets
        dev = self.device
        g = torch.Generator(device=dev).manual_seed(seed)
        # resident frozen embedding + head (HF init: normal(0, 0.02), norm weights 1)
        self.embed = nn.Embedding(shape.vocab, shape.hidden, device=dev, dtype=torch.bfloat16)
        self.embed.weight.requires_grad_(False)
        with torch.no_grad():
            self.embed.weight.normal_(0.0, 0.02, generator=g)
        self.head = LlamaHead(shape, device=dev)
        with torch.no_grad():
            self.head.lm_head.weight.normal_(0.0, 0.02, generator=g)
        for p in self.head.parameters():
            p.requires_grad_(False)
        # int8 segments of every block in pinned RAM (quantised once, on the device)
        from .moe import MixtralBlock, MixtralShape
        moe = isinstance(shape, MixtralShape)
        block_cls = MixtralBlock if moe else LlamaBlock
        shard_group = None
        if weight_shard:
            # opt-in: each rank uploads 1/world of every segment, NCCL all-gathers
            # the rest over NVLink (beyond the gradient-all-reduce-only default)
            import torch.distributed as dist
            if not dist.is_initialized() or dist.get_world_size(group) < 2:
                raise ValueError("weight_shard needs an initialised process group of >= 2 ranks")
            if full_ft_layers or resident_layers:
                raise ValueError("weight_shard streams every layer and keeps no full segment "
                                 "in RAM: no resident layers, no selective full fine-tuning")
            shard_group = group if group is not None else dist.group.WORLD
        self.ws = WeightSegments(shape, self.L, dev, shard_group=shard_group,
                                 num_slots=vram_slots)
        self.nslots = self.ws.num_slots
        true_weights = {}
        if weights is not None:
            self._load_weights(weights, block_cls, full_ft_layers, full_ft_modules,
                               true_weights)
        for b in range(self.L if weights is None else 0):
            tensors = {}
            for name in block_cls.FUSABLE:
                o, i = shape.proj_shapes()[name]
                w = torch.empty(o, i, device=dev, dtype=torch.bfloat16).normal_(0.0, 0.02,
                                                                                 generator=g)
                if b in full_ft_layers and name in full_ft_modules:
                    true_weights[(b, name)] = w
                wq, sw = ops.quantize_weight(w)
                tensors[name + ".wq"] = wq
                tensors[name + ".sw"] = sw
            ones = torch.ones(shape.hidden, device=dev, dtype=torch.bfloat16)
            tensors["input_layernorm"] = ones
            tensors["post_attention_layernorm"] = ones
            self.ws.pack_block(b, tensors, commit=False)
            if moe:
                self._pack_experts(b, g)
            self.ws.commit(b)
        torch.cuda.synchronize(dev)
        self.ws.drop_staging()
        # optional HBM-resident copies of the first `resident_layers` segments
        self.resident = [self.ws.ram[b].to(dev) for b in range(min(resident_layers, self.L))]
        self.weight_shard = weight_shard
        # two block modules, bound per layer (the reference's module pool)
        self.blocks = [block_cls(shape, quantized=True, device=dev) for _ in range(2)]
        for blk in self.blocks:
            for p in blk.parameters():  # frozen base: norms, router (LoRA is added below)
                p.requires_grad_(False)
            if targets:
                apply_lora(blk, lora_rank, lora_alpha, targets)
            blk.gradient_checkpointing = gradient_checkpointing
            blk.self_attn.attn_chunk = attn_chunk
            blk.self_attn.attn_impl = attn_impl
        # LoRA parameters per layer, reference init (A kaiming-uniform, B zeros)
        self.lora: list[dict[str, tuple[nn.Parameter, nn.Parameter]]] = []
        for _ in range(self.L):
            layer = {}
            for name in targets:
                o, i = shape.proj_shapes()[name]
                a = torch.zeros(lora_rank, i, device=dev, dtype=torch.bfloat16)
                nn.init.kaiming_uniform_(a, a=math.sqrt(5), generator=g)
                layer[name] = (nn.Parameter(a),
                               nn.Parameter(torch.zeros(o, lora_rank, device=dev,
                                                        dtype=torch.bfloat16)))
            self.lora.append(layer)
        self.params = [p for layer in self.lora for ab in layer.values() for p in ab]
        self.opt = (torch.optim.AdamW(self.params, lr=lr, weight_decay=weight_decay, fused=True)
                    if self.params else None)
        self.full_ft = None
        if true_weights:
            from .full_ft import SelectiveFullFT
            self.full_ft = SelectiveFullFT(self.ws, sorted({b for b, _ in true_weights}),
                                           full_ft_modules, true_weights, dev, lr, weight_decay)
            del true_weights
        per_layer = batch * seq * shape.hidden * 2  # one bf16 boundary activation
        if ckpt_mode is None:  # keep what fits the HBM budget, offload the rest
            budget = (ckpt_hbm_budget if ckpt_hbm_budget is not None
                      else torch.cuda.mem_get_info(dev)[0] // 4)
            mode = 0
        else:
            budget = ckpt_hbm_budget or 0
            mode = ckpt_mode
        self.ckpt = ActivationCheckpointStore(self.L, (batch, seq, shape.hidden), dev,
                                              mode=mode, h2d_stream=self.ws.h2d_stream,
                                              device_slots=int(budget // per_layer))
        self.cos, self.sin = rope_cos_sin(shape, seq, dev, torch.bfloat16)
        self.reducer = LoraGradReducer(group)
        # device-side failures (a bounded wait in a kernel that ran out) are
        # moved to pinned host memory at the end of each step and raised at the
        # start of the first step after that step's kernels ran, without a sync
        from ._native import DeviceErrorWatch
        self.errors = DeviceErrorWatch()
        self.slot_layer = [-1] * self.nslots
        self.grad_accum = max(1, int(grad_accum))
        self.micro_step = 0
        self.global_step = 0

    # ---- weights -----------------------------------------------------------
    @torch.no_grad()
    def _load_weights(self, path: str, block_cls, full_ft_layers, full_ft_modules,
                      true_weights: dict) -> None:
        """Fills the segments, embedding and head from a checkpoint: an int8
        segment file (straight copy) or a Hugging Face safetensors checkpoint
        (quantised block by block on the device)."""
        from . import checkpoint as ckp
        dev = self.device
        if ckp.is_segment_file(path):
            if full_ft_layers:
                raise ValueError("selective full fine-tuning needs the bf16 weights: load a "
                                 "Hugging Face checkpoint, not an int8 segment file")
            ck = ckp.load_segments(path, self.ws)
        else:
            ck = ckp.HFCheckpoint(path)
            for b in range(self.L):
                keep = tuple(full_ft_modules) if b in full_ft_layers else ()
                kept = ckp.pack_block_from_hf(self.ws, b, ck, block_cls.FUSABLE, dev, keep)
                for name, w in kept.items():
                    true_weights[(b, name)] = w
        self.embed.weight.copy_(ck.get("model.embed_tokens.weight").to(dev, torch.bfloat16))
        self.head.norm.weight.copy_(ck.get("model.norm.weight").to(dev, torch.bfloat16))
        lm = "lm_head.weight" if "lm_head.weight" in ck else "model.embed_tokens.weight"
        self.head.lm_head.weight.copy_(ck.get(lm).to(dev, torch.bfloat16))

    def save_segments(self, path: str) -> None:
        """Writes the quantised segments, embedding and head as an int8 segment
        file that ``weights=path`` loads without re-quantising."""
        from . import checkpoint as ckp
        torch.cuda.synchronize(self.device)
        ckp.save_segments(path, self.ws, self.embed.weight, self.head.norm.weight,
                          self.head.lm_head.weight)

    @torch.no_grad()
    def _pack_experts(self, b: int, g: torch.Generator) -> None:
        """Random-init experts of a MoE block (N(0, 0.02), as HF initialises
        MixtralExperts), quantised per output channel one expert at a time, and a
        router drawn N(0, 1/hidden) so that its logits on RMS-normalised inputs are
        ~N(0, 1)."""
        sh, dev, ws = self.shape, self.device, self.ws
        ram = ws.staging(b)
        for e in range(sh.experts):
            for name, (o, i) in (("gate_up", (2 * sh.intermediate, sh.hidden)),
                                 ("down", (sh.hidden, sh.intermediate))):
                w = torch.empty(o, i, device=dev, dtype=torch.bfloat16).normal_(0.0, 0.02,
                                                                                 generator=g)
                wq, sw = ops.quantize_weight(w)
                ws._view(ram, f"experts.{name}.wq")[e].copy_(wq)
                ws._view(ram, f"experts.{name}.sw")[e].copy_(sw)
        router = torch.empty(sh.experts, sh.hidden, device=dev, dtype=torch.bfloat16)
        router.normal_(0.0, sh.hidden ** -0.5, generator=g)
        ws._view(ram, "router").copy_(router)

    def _ensure(self, layer: int) -> None:
        """Starts the upload of ``layer`` into its slot unless it is already there."""
        slot = layer % self.nslots
        if layer < len(self.resident) or self.slot_layer[slot] == layer:
            return
        self.ws.upload(layer, slot)
        self.slot_layer[slot] = layer

    def _bind(self, layer: int) -> LlamaBlock:
        slot = layer % self.nslots
        blk = self.blocks[layer % 2]
        if layer < len(self.resident):
            self._bind_resident(blk, layer)
        else:
            self.ws.acquire(slot)
            self.ws.bind(blk, slot)
        for name, (a, b) in self.lora[layer].items():
            m = blk.projection(name)
            m.lora_A = a
            m.lora_B = b
        if self.full_ft is not None:
            self.full_ft.attach(layer, blk)
        return blk

    def _bind_resident(self, blk: LlamaBlock, layer: int) -> None:
        self.ws.bind_buffer(blk, self.resident[layer])

    def _release(self, layer: int) -> None:
        if layer >= len(self.resident):
            self.ws.release(layer % self.nslots)

    # ---- one step ------------------------------------------------------------
    def train_step(self, ids: torch.Tensor, labels: torch.Tensor | None = None) -> torch.Tensor:
        """One optimizer step on a [batch, seq] micro-batch of token ids (device or
        pinned host). Returns the loss as a 0-d device tensor."""
        self.errors.check()
        dev = self.device
        ids = ids.to(dev, non_blocking=True)
        labels = ids if labels is None else labels.to(dev, non_blocking=True)
        L = self.L
        # forward (no grad), saving each block's input to pinned host
        ahead = self.nslots - 1  # uploads run this many layers ahead of compute
        with torch.no_grad():
            h = self.embed(ids)
            for k in range(min(ahead, L)):
                self._ensure(k)
            for i in range(L):
                if i + ahead < L:
                    self._ensure(i + ahead)
                blk = self._bind(i)
                self.ckpt.save(i, h)
                h = blk(h, self.cos, self.sin)
                self._release(i)
        # the last block's input comes back while the head and the loss run
        self.ckpt.restore_async(L - 1)
        # head + loss
        h = h.detach().requires_grad_(True)
        logits = self.head(h)
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]),
                               labels[:, 1:].reshape(-1))
        # the reference divides by the accumulation count (src/lema/_trainer.py:156)
        (loss / self.grad_accum).backward()
        self.micro_step += 1
        stepping = self.micro_step % self.grad_accum == 0
        grad = h.grad
        del logits, h
        # backward in reverse: restore, re-forward with grad, backward
        for k in range(1, ahead):
            if L - 1 - k >= 0:
                self._ensure(L - 1 - k)
        for i in range(L - 1, -1, -1):
            if i - ahead >= 0:
                self._ensure(i - ahead)
            if i - 1 >= 0:
                self.ckpt.restore_async(i - 1)
            blk = self._bind(i)
            x = self.ckpt.wait(i).requires_grad_(True)
            out = blk(x, self.cos, self.sin)
            out.backward(grad)
            grad = x.grad
            del out, x
            self._release(i)
            if stepping:
                self.reducer.launch([p.grad for ab in self.lora[i].values() for p in ab])
                if self.full_ft is not None and i in self.full_ft.layers:
                    entry = self.reducer.launch(self.full_ft.layer_grads(i))
                    self.full_ft.step_layer_async(i, entry, self.reducer)
        if stepping:
            self.reducer.finish()
            if self.opt is not None:
                torch.nn.utils.clip_grad_norm_(self.params, 1.0)
                self.opt.step()
                self.opt.zero_grad(set_to_none=False)
            if self.full_ft is not None:
                self.full_ft.finish()
                # the selected layers' int8 segments changed: drop stale copies
                for s in range(self.nslots):
                    if self.slot_layer[s] in self.full_ft.layers:
                        self.slot_layer[s] = -1
                for b in self.full_ft.layers:
                    if b < len(self.resident):
                        self.resident[b].copy_(self.ws.ram[b])
            self.global_step += 1
        self.errors.arm(torch.cuda.current_stream(dev).cuda_stream)
        return loss.detach()

    def check_device_errors(self) -> None:
        """Raises LemaError if a kernel of an earlier step recorded a failure
        (the check ``train_step`` makes before each step)."""
        self.errors.check()

    def close(self) -> None:
        self.ws.close()
