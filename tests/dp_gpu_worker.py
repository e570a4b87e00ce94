"""torchrun worker for tests/test_dp_gpu.py: one data-parallel LoRA step of the
streamed trainer on a small model, each rank on its own micro-batch; rank 0
saves the loss and the updated LoRA parameters."""
import datetime
import os
import sys

import torch
import torch.distributed as dist
from torch.nn.attention import SDPBackend, sdpa_kernel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from lema_b200.llama import LlamaShape  # noqa: E402
from lema_b200.trainer import StreamedLoraTrainer  # noqa: E402

SMALL = LlamaShape(hidden=256, heads=4, kv_heads=4, intermediate=688, vocab=512, layers=4)


def micro_batch(i, dev):
    g = torch.Generator(device=dev).manual_seed(500 + i)
    return torch.randint(0, SMALL.vocab, (2, 64), device=dev, generator=g)


def main(out_path):
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank = dist.get_rank()
    tr = StreamedLoraTrainer(SMALL, dev, batch=2, seq=64, lr=1e-3, seed=21)
    with sdpa_kernel(SDPBackend.MATH):
        loss = tr.train_step(micro_batch(rank, dev))
    losses = [torch.zeros(1, device=dev) for _ in range(dist.get_world_size())]
    dist.all_gather(losses, loss.float().reshape(1))
    if rank == 0:
        torch.save({"losses": [float(x) for x in losses],
                    "params": [p.detach().cpu() for p in tr.params]}, out_path)
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
