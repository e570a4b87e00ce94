"""Data parallelism on real GPUs: a 2-rank streamed LoRA step (NCCL gradient
all-reduce) equals one rank accumulating the same two micro-batches. Needs 2
GPUs; runs the ranks as a torchrun child process."""
import os
import subprocess
import sys

import pytest
import torch
from torch.nn.attention import SDPBackend, sdpa_kernel

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_step_equals_accumulation(cuda_device, tmp_path):
    out = tmp_path / "dp.pt"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29561",
           os.path.join(HERE, "dp_gpu_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    dp = torch.load(out)

    sys.path.insert(0, HERE)
    from dp_gpu_worker import SMALL, micro_batch
    from lema_b200.trainer import StreamedLoraTrainer
    tr = StreamedLoraTrainer(SMALL, cuda_device, batch=2, seq=64, lr=1e-3, seed=21, grad_accum=2)
    with sdpa_kernel(SDPBackend.MATH):
        l0 = float(tr.train_step(micro_batch(0, cuda_device)))
        l1 = float(tr.train_step(micro_batch(1, cuda_device)))
    assert abs(l0 - dp["losses"][0]) <= 1e-3 * abs(l0)
    assert abs(l1 - dp["losses"][1]) <= 1e-3 * abs(l1)
    # first AdamW step moves each parameter by about lr * sign(grad): compare
    # elementwise, allowing a few sign flips where the gradient is ~0
    total = mismatched = 0
    for a, b in zip(dp["params"], [p.detach().cpu() for p in tr.params]):
        d = (a.float() - b.float()).abs()
        total += d.numel()
        mismatched += int((d > 2e-4).sum())
    tr.close()
    assert mismatched <= 0.01 * total, (mismatched, total)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_weight_stream_equals_own_segments(cuda_device, tmp_path):
    """Sharded streaming (half of every segment over each rank's PCIe link, the
    other half all-gathered over NVLink) gives the same 2-rank steps, bit for
    bit, as every rank streaming its own segments — dense and MoE blocks."""
    out = tmp_path / "shard.pt"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29563",
           os.path.join(HERE, "shard_gpu_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    rep = torch.load(out)
    for name, v in rep.items():
        assert v["chunk_bytes"] * 2 >= v["segment_bytes"] > v["chunk_bytes"], (name, v)
    assert all(v["stream_bytes_equal"] for v in rep.values()), rep
    assert all(v["same"] for v in rep.values()), rep


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_full_ft_step_equals_accumulation(cuda_device, tmp_path):
    """Selective full fine-tuning under data parallelism (each selected layer's
    accumulators all-reduced as their own bucket, then clipped and stepped on the
    side stream) moves the true weights as one rank accumulating both
    micro-batches does."""
    out = tmp_path / "dpft.pt"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29565",
           os.path.join(HERE, "dp_ft_gpu_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    dp = torch.load(out)
    sys.path.insert(0, HERE)
    from dp_ft_gpu_worker import FT_LAYERS
    from dp_gpu_worker import SMALL, micro_batch
    from lema_b200.trainer import StreamedLoraTrainer
    tr = StreamedLoraTrainer(SMALL, cuda_device, batch=2, seq=64, targets=(), lr=1e-3,
                             seed=31, full_ft_layers=FT_LAYERS, grad_accum=2)
    with sdpa_kernel(SDPBackend.MATH):
        tr.train_step(micro_batch(0, cuda_device))
        tr.train_step(micro_batch(1, cuda_device))
    total = moved = mismatched = 0
    for key, w in tr.full_ft.true.items():
        a, b = dp[key].float(), w.float()
        total += a.numel()
        mismatched += int(((a - b).abs() > 1e-6 + 2 ** -7 * b.abs()).sum())
        moved += int((a != 0).sum())
    tr.close()
    assert moved > 0
    # the first AdamW step moves each weight by about lr * sign(grad): a few
    # elements whose gradient is ~0 may go the other way
    assert mismatched <= 0.01 * total, (mismatched, total)
