"""Data-parallel host logic on CPU with the gloo backend (world size 2).

1. LoraGradReducer averages each layer's LoRA gradient bucket over the ranks
   and writes the average back into the gradients.
2. Two ranks, each running a decoder block (oracle W8A8 projections, LoRA on
   q/v) forward + backward on its own micro-batch and then the reducer, end with
   the same LoRA gradients as one process accumulating both micro-batches with
   the loss divided by 2 (the reference's accumulation rule,
   src/lema/_trainer.py:156) — the equivalence the GPU data-parallel step relies on.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            init_method=f"tcp://127.0.0.1:{port}")


def _reducer_worker(rank, world, port, out_dir):
    from lema_b200.trainer import LoraGradReducer
    _init(rank, world, port)
    try:
        grads = [torch.full((3, 4), float(rank + 1), dtype=torch.bfloat16),
                 torch.arange(6, dtype=torch.bfloat16).reshape(2, 3) * (rank + 1)]
        red = LoraGradReducer()
        red.launch(grads)
        red.finish()
        torch.save(grads, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_reducer_averages_over_gloo_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_reducer_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    g0 = torch.load(tmp_path / "r0.pt")
    g1 = torch.load(tmp_path / "r1.pt")
    for a, b in zip(g0, g1):
        assert torch.equal(a, b)
    assert torch.equal(g0[0], torch.full((3, 4), 1.5, dtype=torch.bfloat16))
    assert torch.equal(g0[1], (torch.arange(6, dtype=torch.float32).reshape(2, 3) * 1.5)
                       .to(torch.bfloat16))


def _block(seed=0):
    from lema_b200.llama import LlamaBlock, LlamaShape, apply_lora
    from oracle.torch_ref import swap_linears
    shape = LlamaShape(hidden=64, heads=4, kv_heads=4, intermediate=160, vocab=64, layers=1)
    g = torch.Generator().manual_seed(seed)
    blk = LlamaBlock(shape, quantized=False, device="cpu")
    with torch.no_grad():
        for name, p in blk.named_parameters():
            p.copy_((1.0 if "layernorm" in name else 0.0) + 0.05 * torch.randn(p.shape, generator=g))
    lora = apply_lora(blk, 4, 8.0)
    with torch.no_grad():
        for a, b in lora.values():
            a.copy_(0.1 * torch.randn(a.shape, generator=g))
            b.copy_(0.05 * torch.randn(b.shape, generator=g))
    swap_linears(blk)
    blk.self_attn.attn_impl = "eager"
    return shape, blk, lora


def _micro_batch(i):
    g = torch.Generator().manual_seed(100 + i)
    return (torch.randn(1, 16, 64, generator=g).to(torch.bfloat16),
            torch.randn(1, 16, 64, generator=g).to(torch.bfloat16))


def _loss_grads(blk, lora, shape, x, w, scale):
    from lema_b200.llama import rope_cos_sin
    cos, sin = rope_cos_sin(shape, x.shape[1], "cpu", torch.bfloat16)
    y = blk(x, cos, sin)
    loss = (y.float() * w.float()).sum() * scale
    loss.backward()


def _dp_worker(rank, world, port, out_dir):
    from lema_b200.trainer import LoraGradReducer
    _init(rank, world, port)
    try:
        shape, blk, lora = _block()
        x, w = _micro_batch(rank)
        _loss_grads(blk, lora, shape, x, w, 1.0)
        grads = [p.grad for ab in lora.values() for p in ab]
        red = LoraGradReducer()
        red.launch(grads)
        red.finish()
        torch.save([g.clone() for g in grads], os.path.join(out_dir, f"dp{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_dp_grads_equal_single_process_accumulation(tmp_path):
    port = _free_port()
    mp.start_processes(_dp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    dp0 = torch.load(tmp_path / "dp0.pt")
    dp1 = torch.load(tmp_path / "dp1.pt")
    shape, blk, lora = _block()
    for i in range(2):
        x, w = _micro_batch(i)
        _loss_grads(blk, lora, shape, x, w, 0.5)
    acc = [p.grad for ab in lora.values() for p in ab]
    for a, b, ref in zip(dp0, dp1, acc):
        assert torch.equal(a, b), "all ranks hold the same averaged gradient"
        rms = ref.float().pow(2).mean().sqrt().item() + 1e-30
        rel = (a.float() - ref.float()).pow(2).mean().sqrt().item() / rms
        # bf16 gradients: fp32 rank average vs bf16 accumulation of two halves
        assert rel <= 1e-2, rel


def _lonely_worker(rank, port, out_dir):
    import datetime
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                init_method=f"tcp://127.0.0.1:{port}",
                                timeout=datetime.timedelta(seconds=3))
        msg = "joined"
    except Exception as e:  # the missing rank surfaces as an error, not a hang
        msg = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "lonely.txt"), "w") as f:
        f.write(msg)


def test_missing_rank_fails_fast_on_the_host(tmp_path):
    """A data-parallel job whose second rank never starts ends rank 0's
    rendezvous with an error after the process-group timeout (host-side
    failure detection; no GPU involved)."""
    import time
    port = _free_port()
    t0 = time.time()
    mp.start_processes(_lonely_worker, args=(port, str(tmp_path)), nprocs=1, join=True,
                       start_method="spawn")
    assert (tmp_path / "lonely.txt").read_text().startswith("error")
    assert time.time() - t0 < 60


def test_shard_layout_covers_the_segment():
    from lema_b200.tensorstore import shard_layout
    for seg in (1, 127, 128, 202_375_168 + 65_536, 1_451_229_312):
        for world in (1, 2, 3, 4, 8):
            padded, chunk = shard_layout(seg, world)
            assert chunk % 128 == 0 and padded == chunk * world
            assert padded >= seg and padded - seg < world * 128
