"""The drop-in LemaMemoryManager (lema_b200._csrc._lema_cpp) keeps the
reference's method names and semantics (src/lema/_csrc/memory_manager.cpp:
51-199). CPU tests use a host-only manager (no device); GPU tests move bytes."""
import threading
import time

import pytest
import torch

from lema_b200._csrc._lema_cpp import LemaMemoryManager
from lema_b200._native import LemaError


def test_method_names_match_the_reference_pybind_module():
    names = ["register_ram_buffer", "register_vram_slot", "pack_layer_to_ram",
             "async_transfer_to_vram", "wait_vram_transfer", "is_transfer_complete",
             "submit_prefetch_job", "is_prefetch_complete", "wait_for_prefetch",
             "is_layer_in_ram", "synchronize_all"]
    for n in names:
        assert callable(getattr(LemaMemoryManager, n))


def test_pack_and_status_host_only():
    mm = LemaMemoryManager(4, 1 << 16, device=-1)
    buf = torch.zeros(64, dtype=torch.float32)
    assert not mm.is_layer_in_ram(1000)
    mm.register_ram_buffer(1000, buf)
    assert mm.is_layer_in_ram(1000)
    a = torch.arange(10, dtype=torch.float32)
    b = torch.arange(5, dtype=torch.int64)
    mm.pack_layer_to_ram(1000, [a, b])
    assert torch.equal(buf[:10], a)
    assert torch.equal(buf[10:20].view(torch.int64), b)
    with pytest.raises(RuntimeError, match="not registered"):
        mm.pack_layer_to_ram(3, [a])
    with pytest.raises(RuntimeError, match="overflow"):
        mm.pack_layer_to_ram(1000, [torch.zeros(100)])
    # invalid event ids are no-ops / complete, as in the reference
    mm.wait_vram_transfer(-1)
    assert mm.is_transfer_complete(5000)
    mm.synchronize_all()


def test_prefetch_jobs_run_on_workers_and_report_errors():
    mm = LemaMemoryManager(2, 16, device=-1)
    seen = []
    gate = threading.Event()

    def job():
        gate.wait(5)
        seen.append(threading.current_thread().name)

    jid = mm.submit_prefetch_job(job)
    assert not mm.is_prefetch_complete(jid)
    with pytest.raises(LemaError):
        mm.wait_for_prefetch_timeout(jid, 30)
    gate.set()
    mm.wait_for_prefetch(jid)
    assert mm.is_prefetch_complete(jid) and len(seen) == 1

    def bad():
        raise ValueError("disk read failed")

    jid = mm.submit_prefetch_job(bad)
    with pytest.raises(ValueError, match="disk read failed"):
        mm.wait_for_prefetch(jid)
    # the pool survives a failing job
    jid = mm.submit_prefetch_job(lambda: seen.append("again"))
    mm.wait_for_prefetch(jid)
    assert seen[-1] == "again"
    assert mm.is_prefetch_complete(987654)


@pytest.mark.gpu
def test_transfer_roundtrip_and_device_side_wait(cuda_device):
    mm = LemaMemoryManager(4, 1 << 22)
    ram = torch.arange(1 << 20, dtype=torch.int32).pin_memory()
    vram = torch.zeros(1 << 20, dtype=torch.int32, device=cuda_device)
    mm.register_ram_buffer(1000, ram)
    mm.register_vram_slot(0, vram)
    ev = mm.async_transfer_to_vram(1000, 0)
    mm.wait_vram_transfer(ev)
    assert mm.is_transfer_complete(ev)
    assert torch.equal(vram.cpu(), ram)
    # second transfer: compute waits on the device, then releases the slot
    ram2 = (torch.arange(1 << 20, dtype=torch.int32) * 3).pin_memory()
    mm.register_ram_buffer(1001, ram2)
    ev = mm.async_transfer_to_vram(1001, 0)
    mm.stream_wait_transfer(ev)
    total = vram.sum(dtype=torch.int64)
    mm.release_vram_slot(0)
    assert int(total) == int(ram2.sum(dtype=torch.int64))
    # a slot that compute still reads is not overwritten before the release
    slow = torch.randn(4096, 4096, device=cuda_device)
    for _ in range(20):
        slow = slow @ slow.T / 4096.0
    before = vram.clone()
    mm.release_vram_slot(0)
    ev = mm.async_transfer_to_vram(1000, 0)
    mm.wait_vram_transfer_timeout(ev, 10_000)
    torch.cuda.synchronize()
    assert torch.equal(before.cpu(), ram2) and torch.equal(vram.cpu(), ram)
    with pytest.raises(RuntimeError, match="Invalid VRAM slot"):
        mm.async_transfer_to_vram(1000, 7)
    mm.synchronize_all()
