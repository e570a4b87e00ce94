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


def stream_check(shape, dev, rank):
    """Streaming alone: the same random segments packed sharded and unsharded;
    after upload (+ all-gather) every slot byte equals the unsharded segment."""
    from lema_b200.tensorstore import WeightSegments
    blocks = 3
    g = torch.Generator(device="cpu").manual_seed(5)
    own = WeightSegments(shape, blocks, dev)
    sh = WeightSegments(shape, blocks, dev, shard_group=dist.group.WORLD)
    segs = [torch.randint(0, 256, (own.seg_bytes,), generator=g, dtype=torch.uint8)
            for _ in range(blocks)]
    for b in range(blocks):
        own.ram[b].copy_(segs[b])
        buf = sh.staging(b)
        buf.zero_()
        buf[:sh.seg_bytes].copy_(segs[b].to(dev))
        sh.commit(b)
    sh.drop_staging()
    ok = True
    for b in range(blocks):
        slot = b % sh.num_slots
        sh.upload(b, slot)
        sh.acquire(slot)
        torch.cuda.synchronize(dev)
        ok &= bool(torch.equal(sh.vram[slot][:sh.seg_bytes].cpu(), segs[b]))
        sh.release(slot)
    torch.cuda.synchronize(dev)
    own.close()
    sh.close()
    return ok


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
        streams = stream_check(shape, dev, rank)
        flag = torch.tensor([1.0 if same else 0.0, 1.0 if streams else 0.0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        diff = max(float((a.float() - b.float()).abs().max()) for a, b in zip(p_own, p_sh))
        report[name] = {"same": bool(flag[0].item() == 1.0),
                        "stream_bytes_equal": bool(flag[1].item() == 1.0),
                        "losses": l_sh, "losses_own": l_own, "max_param_diff": diff,
                        "chunk_bytes": c_sh, "segment_bytes": c_own}
    if rank == 0:
        torch.save(report, out_path)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
