"""Host placement of a rank's process next to its GPU.

The streamed trainer pins gigabytes of host memory per rank (weight segments,
activation slots) and pulls them over the GPU's PCIe link every step. Pinned
pages are placed on the NUMA node of the thread that first touches them, so a
rank whose process runs on the other socket streams its weights across the
inter-socket link. ``bind_to_gpu_cpus`` restricts the calling process to the
CPUs NVML reports as local to the GPU (read-only NVML queries; no GPU setting is
changed), before anything is pinned.
"""
from __future__ import annotations

import os

import torch


def gpu_local_cpus(device) -> list[int] | None:
    """CPUs local to ``device`` that this process may run on, or None when NVML
    or the PCI identity of the device is unavailable."""
    try:
        import pynvml
    except ImportError:
        return None
    try:
        props = torch.cuda.get_device_properties(torch.device(device))
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = ((os.cpu_count() or 64) + 63) // 64
            masks = list(pynvml.nvmlDeviceGetCpuAffinity(handle, words))
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        return None
    allowed = os.sched_getaffinity(0)
    cpus = [w * 64 + b for w, m in enumerate(masks) for b in range(64)
            if (int(m) >> b) & 1 and (w * 64 + b) in allowed]
    return cpus or None


def bind_to_gpu_cpus(device) -> list[int] | None:
    """Restricts this process to the CPUs local to ``device``; returns them (None
    and no change when they cannot be determined)."""
    cpus = gpu_local_cpus(device)
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus
