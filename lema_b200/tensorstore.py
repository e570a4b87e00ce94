"""Pinned-host streams of the streamed trainer: boundary-activation checkpoints
(A5) and int8 weight segments (A7).

``ActivationCheckpointStore`` replaces the VRAM-resident
``boundary_activations`` list of ``LemaTrainer.train_step``
(src/lema/_trainer.py:109-111 save, :146-148 restore): each layer's input is
copied into a pinned host slot on a D2H copy stream right after it is produced
(``lema_ckpt_save``, copy engine or SM store kernel), overlapping the next
layer's compute and weight upload; in backward it is copied back on the H2D
stream ahead of the layer's re-forward (``lema_ckpt_restore``). Ordering is by
CUDA events only — the host never blocks.

``WeightSegments`` holds every block's int8 weights, fp32 scales and bf16
norm weights as one 128-byte-aligned segment per block in pinned host memory
(the RAM side of the reference's ``_TransferEngine``, src/lema/_tensorstore.py:
213-302) and streams segments into two VRAM slots through the native memory
manager (``lema_mm_*``), binding W8A8Linear weights as views of the slot
instead of copying them into parameters (src/lema/adapters/_llama.py:95-100).
A Mixtral block's segment holds its attention projections the same way plus
the grouped expert tensors (int8 gate_up [E, 2I, H], down [E, H, I], their
scales) and the bf16 router weight, bound into the block's experts module.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _native as N
from .llama import LlamaBlock, LlamaShape


def _ev_ptr(ev: torch.cuda.Event | None):
    return None if ev is None else C.c_void_p(ev.cuda_event)


class ActivationCheckpointStore:
    """``num`` checkpoint slots of ``shape`` (bf16 by default): slots
    [0, device_slots) stay in device memory, the others go to pinned host slots.

    ``mode`` 0 saves the host slots through the copy engine, 1 through the SM
    store kernel (``lema_ckpt_save``); mode 2 keeps every boundary tensor in
    device memory (the reference's ``boundary_activations`` list,
    src/lema/_trainer.py:109-111): no host slots, no copies."""

    DEVICE = 2

    def __init__(self, num: int, shape: tuple[int, ...], device: torch.device,
                 dtype: torch.dtype = torch.bfloat16, mode: int = 0,
                 h2d_stream: torch.cuda.Stream | None = None, device_slots: int = 0):
        if mode not in (0, 1, self.DEVICE):
            raise ValueError(f"checkpoint mode must be 0, 1 or 2, not {mode}")
        self.device = torch.device(device)
        self.shape = tuple(shape)
        self.dtype = dtype
        self.device_slots = num if mode == self.DEVICE else max(0, min(int(device_slots), num))
        if self.device_slots == num:
            mode = self.DEVICE
        self.mode = mode
        self.host_slots = num - self.device_slots
        self._kept: dict[int, torch.Tensor] = {}
        if mode == self.DEVICE:
            self.host = None
            self.nbytes = 0  # bytes moved per host slot and direction
            self._dev_buf: dict[int, torch.Tensor] = {}
            return
        self.host = torch.empty((num, *shape), dtype=dtype).pin_memory()
        self.nbytes = self.host[0].numel() * self.host.element_size()
        self.d2h = torch.cuda.Stream(device=self.device)
        self.h2d = h2d_stream if h2d_stream is not None else torch.cuda.Stream(device=self.device)
        self.saved = [torch.cuda.Event() for _ in range(num)]
        self.restored = [torch.cuda.Event() for _ in range(num)]
        self._dev_buf: dict[int, torch.Tensor] = {}

    def save(self, i: int, t: torch.Tensor) -> None:
        """Copies device tensor ``t`` into slot i once the current stream has produced it."""
        if tuple(t.shape) != self.shape or t.dtype != self.dtype:
            raise ValueError(f"checkpoint slot holds {self.shape} {self.dtype}, got "
                             f"{tuple(t.shape)} {t.dtype}")
        t = t.detach()
        if i < self.device_slots:
            self._kept[i] = t
            return
        if not t.is_contiguous():
            t = t.contiguous()
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        N.call("lema_ckpt_save", t.data_ptr(), self.host[i].data_ptr(), self.nbytes, self.mode,
               self.d2h.cuda_stream, _ev_ptr(ready), _ev_ptr(self.saved[i]))
        t.record_stream(self.d2h)  # the caching allocator keeps t alive until the copy ends

    def restore_async(self, i: int) -> torch.Tensor:
        """Starts the H2D copy of slot i into a device buffer and returns the buffer;
        call ``wait(i)`` on the consuming stream before reading it."""
        if i < self.device_slots:
            self._dev_buf[i] = self._kept.pop(i)
            return self._dev_buf[i]
        buf = torch.empty(self.shape, dtype=self.dtype, device=self.device)
        # buf's memory may still be read by earlier work on the allocating stream:
        # the copy stream starts only after that point.
        self.h2d.wait_stream(torch.cuda.current_stream(self.device))
        N.call("lema_ckpt_restore", self.host[i].data_ptr(), buf.data_ptr(), self.nbytes,
               self.h2d.cuda_stream, _ev_ptr(self.saved[i]), _ev_ptr(self.restored[i]))
        buf.record_stream(self.h2d)
        self._dev_buf[i] = buf
        return buf

    def wait(self, i: int, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        if i < self.device_slots:
            return self._dev_buf.pop(i)
        s = stream or torch.cuda.current_stream(self.device)
        s.wait_event(self.restored[i])
        return self._dev_buf.pop(i)

    @property
    def moved_bytes(self) -> int:
        """Bytes copied per step and direction (the host slots)."""
        return self.nbytes * self.host_slots

    def restore(self, i: int) -> torch.Tensor:
        self.restore_async(i)
        return self.wait(i)


@dataclass
class _Seg:
    offset: int
    nbytes: int
    shape: tuple[int, ...]
    dtype: torch.dtype


def shard_layout(seg_bytes: int, world: int, align: int = 128) -> tuple[int, int]:
    """(padded segment bytes, bytes per rank) when a segment is split into
    ``world`` equal, ``align``-aligned chunks for sharded streaming."""
    chunk = -(-seg_bytes // (world * align)) * align
    return chunk * world, chunk


class WeightSegments:
    """All blocks' int8 segments in pinned RAM + ``num_slots`` (default two) VRAM
    slots fed by the native manager's H2D copy stream.

    Sharded streaming (``shard_group`` given, opt-in): rank r of W keeps only
    chunk r of every (padded) segment in pinned RAM and uploads it into its
    place in the slot; an in-place NCCL all-gather over NVLink, issued on a side
    stream behind the upload, fills in the other W-1 chunks. Each rank then moves
    1/W of the segment bytes over PCIe (the host's memory and PCIe root are
    shared by the ranks) and ~(W-1)/W of them over NVLink. The default is the
    unsharded form: every rank streams its own full copy of each segment."""

    ALIGN = 128

    def __init__(self, shape: LlamaShape, num_blocks: int, device: torch.device,
                 shard_group=None, num_slots: int = 2):
        from .moe import MixtralBlock, MixtralShape
        self.moe = isinstance(shape, MixtralShape)
        block_cls = MixtralBlock if self.moe else LlamaBlock
        self.GROUPS = block_cls.FUSED_GROUPS
        self.shape = shape
        self.device = torch.device(device)
        self.num_blocks = num_blocks
        self.layout: dict[str, _Seg] = {}
        off = 0

        def add(name, shp, dtype):
            nonlocal off
            nb = int(torch.Size(shp).numel()) * torch.empty((), dtype=dtype).element_size()
            self.layout[name] = _Seg(off, nb, tuple(shp), dtype)
            off = (off + nb + self.ALIGN - 1) // self.ALIGN * self.ALIGN

        # Projections that read the same input are stacked (q|k|v, gate|up) so the
        # block can run them as one GEMM; each projection is a row range of its group.
        self.sub: dict[str, tuple[str, int, int]] = {}
        ps = shape.proj_shapes()
        for group, names in self.GROUPS:
            rows = sum(ps[n][0] for n in names)
            add(group + ".wq", (rows, ps[names[0]][1]), torch.int8)
            add(group + ".sw", (rows,), torch.float32)
            r0 = 0
            for n in names:
                r1 = r0 + ps[n][0]
                self.sub[n + ".wq"] = (group + ".wq", r0, r1)
                self.sub[n + ".sw"] = (group + ".sw", r0, r1)
                r0 = r1
        if self.moe:
            E, I, H = shape.experts, shape.intermediate, shape.hidden
            add("experts.gate_up.wq", (E, 2 * I, H), torch.int8)
            add("experts.gate_up.sw", (E, 2 * I), torch.float32)
            add("experts.down.wq", (E, H, I), torch.int8)
            add("experts.down.sw", (E, H), torch.float32)
            add("router", (E, H), torch.bfloat16)
        add("input_layernorm", (shape.hidden,), torch.bfloat16)
        add("post_attention_layernorm", (shape.hidden,), torch.bfloat16)
        self.seg_bytes = off
        self.group = shard_group
        if shard_group is not None:
            import torch.distributed as dist
            self._dist = dist
            self.rank = dist.get_rank(shard_group)
            self.world = dist.get_world_size(shard_group)
            self.slot_bytes, self.chunk = shard_layout(self.seg_bytes, self.world, self.ALIGN)
            self.gather_stream = torch.cuda.Stream(self.device)
        else:
            self.rank, self.world = 0, 1
            self.slot_bytes = self.chunk = self.seg_bytes
        # pinned RAM: every block's full segment, or this rank's chunk of it
        self.ram = torch.empty(num_blocks, self.chunk, dtype=torch.uint8, pin_memory=True)
        self.num_slots = max(2, int(num_slots))
        self.vram = [torch.empty(self.slot_bytes, dtype=torch.uint8, device=self.device)
                     for _ in range(self.num_slots)]
        self._staging: torch.Tensor | None = None
        self.mm = C.c_void_p()
        dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        N.call("lema_mm_create", num_blocks + 2, self.chunk, dev_index, C.byref(self.mm))
        for b in range(num_blocks):
            N.call("lema_mm_register_ram_buffer", self.mm, b, self.ram[b].data_ptr(),
                   self.chunk)
        for s in range(self.num_slots):  # the upload lands at this rank's chunk of the slot
            N.call("lema_mm_register_vram_slot", self.mm, s,
                   self.vram[s].data_ptr() + self.rank * self.chunk, self.chunk)
        sp = C.c_void_p()
        N.call("lema_mm_copy_stream", self.mm, C.byref(sp))
        self.h2d_stream = torch.cuda.ExternalStream(sp.value, device=self.device)
        self._pending: dict[int, int] = {}
        self._gathers: dict[int, object] = {}

    @property
    def sharded(self) -> bool:
        return self.group is not None

    def close(self) -> None:
        if self.mm:
            N.call("lema_mm_destroy", self.mm)
            self.mm = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- filling RAM (pack time) -------------------------------------------
    def _view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        if name in self.sub:
            group, r0, r1 = self.sub[name]
            return self._view(buf, group)[r0:r1]
        seg = self.layout[name]
        raw = buf[seg.offset: seg.offset + seg.nbytes]
        return raw.view(seg.dtype).view(seg.shape)

    def staging(self, b: int) -> torch.Tensor:
        """A full-segment buffer to write block b into: the pinned segment itself,
        or (sharded) a device buffer whose chunk ``commit`` keeps."""
        if not self.sharded:
            return self.ram[b]
        if self._staging is None:
            self._staging = torch.zeros(self.slot_bytes, dtype=torch.uint8, device=self.device)
        return self._staging

    def drop_staging(self) -> None:
        """Frees the device staging buffer once every block is packed."""
        self._staging = None

    def commit(self, b: int) -> None:
        """Sharded: copies this rank's chunk of the staging buffer into RAM."""
        if self.sharded:
            c0 = self.rank * self.chunk
            self.ram[b].copy_(self._staging[c0:c0 + self.chunk])

    def pack_block(self, b: int, tensors: dict[str, torch.Tensor], commit: bool = True) -> None:
        """Writes one block's quantised tensors (device or host) into its segment."""
        buf = self.staging(b)
        for name, t in tensors.items():
            v = self._view(buf, name)
            v.copy_(t.detach().reshape(v.shape))
        if commit:
            self.commit(b)

    # ---- streaming -----------------------------------------------------------
    def upload(self, b: int, slot: int) -> None:
        """Starts the H2D of block b's segment (or this rank's chunk of it) into
        VRAM slot ``slot`` (the copy stream first waits until compute released
        that slot); sharded, the slot's all-gather follows on the gather stream."""
        ev = C.c_int64(-1)
        N.call("lema_mm_async_transfer_to_vram", self.mm, b, slot, 0, C.byref(ev))
        if not self.sharded:
            self._pending[slot] = ev.value
            return
        gs = self.gather_stream
        N.call("lema_mm_stream_wait_transfer", self.mm, ev.value, gs.cuda_stream)
        with torch.cuda.stream(gs):
            full = self.vram[slot]
            mine = full[self.rank * self.chunk:(self.rank + 1) * self.chunk]
            self._gathers[slot] = self._dist.all_gather_into_tensor(full, mine, group=self.group,
                                                                    async_op=True)

    def acquire(self, slot: int, stream: torch.cuda.Stream | None = None) -> None:
        """Makes the compute stream wait (on the device) for slot's upload (and,
        sharded, its all-gather)."""
        s = stream or torch.cuda.current_stream(self.device)
        if self.sharded:
            work = self._gathers.pop(slot, None)
            if work is not None:
                with torch.cuda.stream(s):
                    work.wait()
            return
        ev = self._pending.pop(slot, -1)
        if ev >= 0:
            N.call("lema_mm_stream_wait_transfer", self.mm, ev, s.cuda_stream)

    def release(self, slot: int, stream: torch.cuda.Stream | None = None) -> None:
        """Records that compute on ``stream`` is done reading ``slot``."""
        s = stream or torch.cuda.current_stream(self.device)
        N.call("lema_mm_release_vram_slot", self.mm, slot, s.cuda_stream)

    def bind(self, block: LlamaBlock, slot: int) -> None:
        """Binds a block's W8A8 projections and norms to views of VRAM slot ``slot``."""
        self.bind_buffer(block, self.vram[slot])

    def bind_buffer(self, block: LlamaBlock, buf: torch.Tensor) -> None:
        """Binds a block to views of any device copy of a segment; also gives the
        block the stacked group weights for its fused path."""
        block.fused_weights = {g + k: self._view(buf, g + k) for g, _ in self.GROUPS
                               for k in (".wq", ".sw")}
        for name in block.FUSABLE:
            block.base_projection(name).bind(self._view(buf, name + ".wq"),
                                             self._view(buf, name + ".sw"))
        if self.moe:
            ex = block.mlp.experts
            ex.wq_gate_up = self._view(buf, "experts.gate_up.wq")
            ex.sw_gate_up = self._view(buf, "experts.gate_up.sw")
            ex.wq_down = self._view(buf, "experts.down.wq")
            ex.sw_down = self._view(buf, "experts.down.sw")
            block.mlp.gate.weight.data = self._view(buf, "router")
        block.input_layernorm.weight.data = self._view(buf, "input_layernorm")
        block.post_attention_layernorm.weight.data = self._view(buf, "post_attention_layernorm")
