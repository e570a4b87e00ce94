"""Drop-in for ``lema._csrc._lema_cpp`` (the reference's pybind module,
src/lema/_csrc/memory_manager.cpp:204-217) over the C ABI's ``lema_mm_*``.

``LemaMemoryManager(num_layers_hint, max_layer_size)`` keeps the same 11 methods
and semantics as the reference class (src/lema/_csrc/memory_manager.h:25-55):
buffers are registered as torch tensors (references are held, as the
reference holds ``torch::Tensor``s), ``async_transfer_to_vram`` returns an event
id from a ring of 1024, invalid event ids are no-ops, unknown job ids count as
complete, and unregistered buffers raise ``RuntimeError`` (``LemaError`` is a
``RuntimeError``). ``_TransferEngine`` (src/lema/_tensorstore.py:103-126, 278-302)
uses it unchanged when it imports this module as ``_lema_cpp``.

Additions: ``wait_vram_transfer_timeout`` (bounded wait, raises on timeout),
``wait_for_prefetch_timeout``, ``stream_wait_transfer`` (the compute stream waits
on the device instead of the host blocking) and ``release_vram_slot`` (the next
transfer into a slot waits until compute has finished reading it). A job
callable that raises does not take the worker thread down: the error is kept
and re-raised by ``wait_for_prefetch``.
"""
from __future__ import annotations

import ctypes as C
import threading

import torch

from .. import _native as N


class LemaMemoryManager:
    def __init__(self, num_layers_hint: int, max_layer_size: int, device: int | None = None):
        if device is None:
            device = torch.cuda.current_device() if torch.cuda.is_available() else -1
        self._h = C.c_void_p()
        N.call("lema_mm_create", int(num_layers_hint), int(max_layer_size), int(device),
               C.byref(self._h))
        self.device = device
        self._ram: dict[int, torch.Tensor] = {}
        self._vram: dict[int, torch.Tensor] = {}
        self._jobs: dict[int, tuple] = {}
        self._lock = threading.Lock()

    def __del__(self):
        try:
            if self._h:
                N.call("lema_mm_destroy", self._h)
                self._h = C.c_void_p()
        except Exception:
            pass

    # ---- registration -------------------------------------------------------
    def register_ram_buffer(self, layer_id: int, buf: torch.Tensor) -> None:
        self._ram[layer_id] = buf
        N.call("lema_mm_register_ram_buffer", self._h, int(layer_id), buf.data_ptr(),
               buf.numel() * buf.element_size())

    def register_vram_slot(self, slot: int, buf: torch.Tensor) -> None:
        self._vram[slot] = buf
        N.call("lema_mm_register_vram_slot", self._h, int(slot), buf.data_ptr(),
               buf.numel() * buf.element_size())

    # ---- packing ------------------------------------------------------------
    def pack_layer_to_ram(self, layer_id: int, src_tensors: list[torch.Tensor]) -> None:
        ts = [t.contiguous() for t in src_tensors]
        ptrs = (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
        sizes = (C.c_size_t * len(ts))(*[t.numel() * t.element_size() for t in ts])
        N.call("lema_mm_pack_layer_to_ram", self._h, int(layer_id), ptrs, sizes, len(ts))

    # ---- transfers ----------------------------------------------------------
    def async_transfer_to_vram(self, layer_id: int, vram_slot: int) -> int:
        ev = C.c_int64(-1)
        N.call("lema_mm_async_transfer_to_vram", self._h, int(layer_id), int(vram_slot), 0,
               C.byref(ev))
        return ev.value

    def wait_vram_transfer(self, event_id: int) -> None:
        N.call("lema_mm_wait_vram_transfer", self._h, int(event_id))

    def wait_vram_transfer_timeout(self, event_id: int, timeout_ms: int) -> None:
        N.call("lema_mm_wait_vram_transfer_timeout", self._h, int(event_id), int(timeout_ms))

    def is_transfer_complete(self, event_id: int) -> bool:
        out = C.c_int32(0)
        N.call("lema_mm_is_transfer_complete", self._h, int(event_id), C.byref(out))
        return bool(out.value)

    def stream_wait_transfer(self, event_id: int, stream: torch.cuda.Stream | None = None) -> None:
        s = stream or torch.cuda.current_stream()
        N.call("lema_mm_stream_wait_transfer", self._h, int(event_id), s.cuda_stream)

    def release_vram_slot(self, vram_slot: int, stream: torch.cuda.Stream | None = None) -> None:
        s = stream or torch.cuda.current_stream()
        N.call("lema_mm_release_vram_slot", self._h, int(vram_slot), s.cuda_stream)

    def synchronize_all(self) -> None:
        N.call("lema_mm_synchronize_all", self._h)

    # ---- prefetch jobs ------------------------------------------------------
    def submit_prefetch_job(self, task) -> int:
        state = {"error": None}

        def run(_user):
            try:
                task()
            except BaseException as e:  # keep the worker alive; surfaced by wait
                state["error"] = e

        cb = N.JOB_FN(run)
        jid = C.c_int64(0)
        N.call("lema_mm_submit_prefetch_job", self._h, cb, None, C.byref(jid))
        with self._lock:
            self._jobs[jid.value] = (cb, state)
        return jid.value

    def is_prefetch_complete(self, job_id: int) -> bool:
        out = C.c_int32(0)
        N.call("lema_mm_is_prefetch_complete", self._h, int(job_id), C.byref(out))
        return bool(out.value)

    def _finish_job(self, job_id: int) -> None:
        with self._lock:
            entry = self._jobs.pop(job_id, None)
        if entry is not None and entry[1]["error"] is not None:
            raise entry[1]["error"]

    def wait_for_prefetch(self, job_id: int) -> None:
        N.call("lema_mm_wait_for_prefetch", self._h, int(job_id))
        self._finish_job(job_id)

    def wait_for_prefetch_timeout(self, job_id: int, timeout_ms: int) -> None:
        N.call("lema_mm_wait_for_prefetch_timeout", self._h, int(job_id), int(timeout_ms))
        self._finish_job(job_id)

    def is_layer_in_ram(self, layer_id: int) -> bool:
        out = C.c_int32(0)
        N.call("lema_mm_is_layer_in_ram", self._h, int(layer_id), C.byref(out))
        return bool(out.value)
