"""torchrun worker for tests/test_dp_gpu.py: one data-parallel step of selective
full fine-tuning (q/k/v/o of the last two layers), each rank on its own
micro-batch; rank 0 saves the updated bf16 true weights."""
import datetime
import os
import sys

import torch
import torch.distributed as dist
from torch.nn.attention import SDPBackend, sdpa_kernel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from lema_b200.trainer import StreamedLoraTrainer  # noqa: E402
from dp_gpu_worker import SMALL, micro_batch  # noqa: E402

FT_LAYERS = (2, 3)


def main(out_path):
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank = dist.get_rank()
    tr = StreamedLoraTrainer(SMALL, dev, batch=2, seq=64, targets=(), lr=1e-3, seed=31,
                             full_ft_layers=FT_LAYERS)
    with sdpa_kernel(SDPBackend.MATH):
        tr.train_step(micro_batch(rank, dev))
    if rank == 0:
        torch.save({k: v.clone() for k, v in tr.full_ft.true.items()}, out_path)
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
