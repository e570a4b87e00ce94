"""GPU tests of the layer-streamed trainer on Mixtral-shaped MoE blocks (GQA
attention + grouped W8A8 experts, LoRA on q/v): the fused attention half
equals the per-projection path, streaming equals HBM residency bit for bit,
and the loss goes down."""
import pytest
import torch
from torch.nn.attention import SDPBackend, sdpa_kernel

from lema_b200.llama import apply_lora, rope_cos_sin
from lema_b200.moe import MixtralBlock, MixtralShape
from lema_b200.trainer import StreamedLoraTrainer

pytestmark = pytest.mark.gpu

TINY = MixtralShape(hidden=256, heads=4, kv_heads=2, intermediate=512, vocab=512, layers=3,
                    experts=4, top_k=2)


def _ids(seed, batch, seq, vocab, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq), device=dev, generator=g)


def _rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return ((a - b).pow(2).mean().sqrt() / (b.pow(2).mean().sqrt() + 1e-30)).item()


def test_mixtral_block_fused_attention_matches_per_projection(cuda_device):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(3)
    blk = MixtralBlock(TINY, quantized=True, device=dev)
    with torch.no_grad():
        for name in blk.FUSABLE:
            m = blk.base_projection(name)
            m.load_float_weight(torch.randn(m.out_features, m.in_features, device=dev,
                                            generator=g) * 0.02)
        E, I, H = TINY.experts, TINY.intermediate, TINY.hidden
        blk.mlp.experts.load_float(torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.02,
                                   torch.randn(E, H, I, device=dev, generator=g) * 0.02)
        blk.mlp.gate.weight.copy_(torch.randn(E, H, device=dev, generator=g) / H ** 0.5)
    lora = apply_lora(blk, 8, 16.0)
    with torch.no_grad():
        for a, b in lora.values():
            b.copy_(torch.randn(b.shape, device=dev, generator=g) * 0.02)
    blk.build_fused_weights()
    cos, sin = rope_cos_sin(TINY, 64, dev, torch.bfloat16)
    x = torch.randn(2, 64, TINY.hidden, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.randn(2, 64, TINY.hidden, device=dev, generator=g).to(torch.bfloat16)
    out = {}
    for fused in (True, False):
        blk.use_fused = fused
        assert blk._can_fuse() == fused
        for a, b in lora.values():
            a.grad = b.grad = None
        xr = x.clone().requires_grad_(True)
        y = blk(xr, cos, sin)
        y.backward(dy)
        out[fused] = (y, xr.grad, [p.grad.clone() for ab in lora.values() for p in ab])
    (y1, dx1, g1), (y0, dx0, g0) = out[True], out[False]
    assert _rel(y1, y0) <= 1e-2
    assert _rel(dx1, dx0) <= 2e-2
    for a, b in zip(g1, g0):
        assert _rel(a, b) <= 5e-2


def test_mixtral_streamed_equals_hbm_resident(cuda_device):
    """Streaming the 3 MoE segments through two VRAM slots or keeping them
    resident runs the same kernels on the same bytes: identical LoRA parameters
    after two steps (top-2 combines are two-term sums, so the index_add order
    does not matter)."""
    ids = _ids(11, 2, 64, TINY.vocab, cuda_device)
    results = []
    for resident in (0, TINY.layers):
        tr = StreamedLoraTrainer(TINY, cuda_device, batch=2, seq=64, lr=1e-3, seed=9,
                                 resident_layers=resident)
        with sdpa_kernel(SDPBackend.MATH):
            losses = [float(tr.train_step(ids)) for _ in range(2)]
        results.append((losses, [p.detach().clone() for p in tr.params]))
        tr.close()
    (l0, p0), (l1, p1) = results
    assert l0 == l1
    for a, b in zip(p0, p1):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_mixtral_trainer_loss_decreases(cuda_device):
    tr = StreamedLoraTrainer(TINY, cuda_device, batch=2, seq=64, lr=1e-2, seed=0)
    assert tr.ws.moe and tr.blocks[0].__class__ is MixtralBlock
    ids = _ids(1, 2, 64, TINY.vocab, cuda_device)
    losses = [float(tr.train_step(ids)) for _ in range(8)]
    tr.close()
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0] - 0.05, losses
