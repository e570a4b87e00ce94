"""torchrun worker for tests/test_dp_gpu.py: the data-parallel streamed LoRA step
with sharded weight streaming (each rank uploads half of every segment, NCCL
all-gathers the other half) against the same step with every rank streaming
its own full segments; dense (Llama-shaped) and MoE (Mixtral-shaped) blocks.
Rank 0 writes whether losses and LoRA parameters matched bit for bit."""
import datetime
import os
import sys

import torch
import torch.distributed as dist
from torch.nn.attention import SDPBackend, sdpa_kernel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from lema_b200.llama import LlamaShape  # noqa: E402
from lema_b200.moe import MixtralShape  # noqa: E402
from lema_b200.trainer import StreamedLoraTrainer  # noqa: E402

SHAPES = {
    "dense": LlamaShape(hidden=256, heads=4, kv_heads=4, intermediate=688, vocab=512, layers=4),
    "moe": MixtralShape(hidden=256, heads=4, kv_heads=2, intermediate=512, vocab=512, layers=3,
                        experts=4, top_k=2),
}


def run(shape, dev, rank, shard):
    tr = StreamedLoraTrainer(shape, dev, batch=2, seq=64, lr=1e-3, seed=21, weight_shard=shard)
    g = torch.Generator(device=dev).manual_seed(700 + rank)
    ids = torch.randint(0, shape.vocab, (2, 64), device=dev, generator=g)
    with sdpa_kernel(SDPBackend.MATH):
        losses = [float(tr.train_step(ids)) for _ in range(2)]
    params = [p.detach().clone() for p in tr.params]
    chunk = tr.ws.chunk
    tr.close()
    return losses, params, chunk


def main(out_path):
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank = dist.get_rank()
    report = {}
    for name, shape in SHAPES.items():
        l_own, p_own, c_own = run(shape, dev, rank, False)
        l_sh, p_sh, c_sh = run(shape, dev, rank, True)
        same = l_own == l_sh and all(torch.equal(a.view(torch.int16), b.view(torch.int16))
                                     for a, b in zip(p_own, p_sh))
        flag = torch.tensor([1.0 if same else 0.0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        report[name] = {"same": bool(flag.item() == 1.0), "losses": l_sh,
                        "chunk_bytes": c_sh, "segment_bytes": c_own}
    if rank == 0:
        torch.save(report, out_path)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
