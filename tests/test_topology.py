"""Host placement helper: without a GPU (or NVML) it reports nothing and leaves
the process's CPU affinity unchanged."""
import os

import torch

from lema_b200.topology import bind_to_gpu_cpus, gpu_local_cpus


def test_no_gpu_no_binding():
    if torch.cuda.is_available():
        return
    before = os.sched_getaffinity(0)
    assert gpu_local_cpus("cuda:0") is None
    assert bind_to_gpu_cpus("cuda:0") is None
    assert os.sched_getaffinity(0) == before
