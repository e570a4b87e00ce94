"""Selective full fine-tuning of W8A8 projections (row A9) on the GPU."""
import numpy as np
import pytest
import torch
from torch.nn.attention import SDPBackend, sdpa_kernel

from lema_b200.llama import LlamaShape
from lema_b200.trainer import StreamedLoraTrainer

pytestmark = pytest.mark.gpu

SMALL = LlamaShape(hidden=256, heads=4, kv_heads=4, intermediate=688, vocab=512, layers=4)


def _ids(seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randint(0, SMALL.vocab, (2, 64), device=dev, generator=g)


def test_full_ft_learns(cuda_device):
    tr = StreamedLoraTrainer(SMALL, cuda_device, batch=2, seq=64, targets=(), lr=3e-3, seed=0,
                             full_ft_layers=(2, 3))
    ids = _ids(1, cuda_device)
    losses = [float(tr.train_step(ids)) for _ in range(6)]
    tr.close()
    assert losses[-1] < losses[0] - 0.05, losses


def test_full_ft_step_requantises_and_matches_reference_adamw(cuda_device):
    from oracle import oracle as O
    from oracle.torch_ref import adamw_step_ref
    tr = StreamedLoraTrainer(SMALL, cuda_device, batch=2, seq=64, targets=(), lr=1e-3,
                             weight_decay=0.01, seed=5, full_ft_layers=(2, 3))
    ft = tr.full_ft
    before = {k: O.torch_bf16_to_bits(w).copy() for k, w in ft.true.items()}  # not a view
    grads = {}
    orig = ft.step_layer

    def capture(layer):
        for n in ft.modules:
            grads[(layer, n)] = ft.acc[(layer, n)].detach().cpu().numpy().copy()
        return orig(layer)
    ft.step_layer = capture
    with sdpa_kernel(SDPBackend.MATH):
        tr.train_step(_ids(2, cuda_device))
    for key, w0 in before.items():
        g = grads[key]
        assert np.abs(g).max() > 0, key
        ref_w, ref_m, ref_v = adamw_step_ref(w0, g, np.zeros_like(g), np.zeros_like(g), 1,
                                             1e-3, 0.01)
        got = O.torch_bf16_to_bits(ft.true[key])
        # The fp32 update may differ in its last bits between the device (fused
        # multiply-adds in addcmul / addcdiv) and numpy: allow one bf16 ulp of the
        # result, or, where w + update nearly cancels and the result is tiny, an
        # absolute 2^-20 * lr (a few fp32 ulps of an update of size ~lr).
        gf, rf = O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(ref_w)
        ulp = np.ldexp(np.float32(1.0), np.frexp(np.abs(rf))[1] - 8)
        bound = np.maximum(ulp, np.float32(2.0 ** -20 * 1e-3))
        excess = np.abs(gf - rf) - bound
        assert excess.max() <= 0, (key, float(excess.max()))
        diff = np.abs(got.astype(np.int32) - ref_w.astype(np.int32))
        assert np.mean(diff == 0) > 0.99, (key, float(np.mean(diff == 0)))
        np.testing.assert_allclose(ft.m[key].numpy(), ref_m, rtol=1e-6, atol=1e-12)
        # the streamed segment now holds the quantised new weight
        layer, name = key
        wq_ref, sw_ref = O.c_quantize_rows(got)
        seg = tr.ws.ram[layer]
        np.testing.assert_array_equal(tr.ws._view(seg, name + ".wq").numpy(), wq_ref)
        np.testing.assert_array_equal(tr.ws._view(seg, name + ".sw").numpy(), sw_ref)
    tr.close()


def test_full_ft_weight_gradient_is_dy_t_x(cuda_device):
    """The accumulated fp32 gradient of a trainable projection equals dy^T . x of
    the activations that flowed through it (captured with hooks)."""
    tr = StreamedLoraTrainer(SMALL, cuda_device, batch=2, seq=64, targets=(), lr=0.0,
                             seed=6, full_ft_layers=(3,), full_ft_modules=("o_proj",))
    seen = {}
    blk = tr.blocks[3 % 2]
    mod = blk.base_projection("o_proj")

    def fwd_hook(m, inp, out):
        if torch.is_grad_enabled() and m.wgrad_acc is not None:
            seen["x"] = inp[0].detach().reshape(-1, inp[0].shape[-1]).float()
            out.register_hook(lambda g: seen.__setitem__("dy", g.reshape(-1, g.shape[-1]).float()))
    mod.register_forward_hook(fwd_hook)
    ft = tr.full_ft
    orig = ft.step_layer
    acc = {}

    def capture(layer):
        acc[layer] = ft.acc[(layer, "o_proj")].clone()
        return orig(layer)
    ft.step_layer = capture
    orig_clip = ft.clip_layer_
    ft.clip_layer_ = lambda layer, max_norm=1.0: orig_clip(layer, 1e30)
    tr.train_step(_ids(3, cuda_device))
    ref = (seen["dy"].double().t() @ seen["x"].double()).float()
    got = acc[3]
    rel = (got - ref).pow(2).mean().sqrt() / ref.pow(2).mean().sqrt()
    assert rel < 1e-5, float(rel)
    tr.close()


@pytest.mark.parametrize("shape,step,wd", [((64, 4096), 3, 0.01), ((37, 11008), 1, 0.01),
                                           ((5, 100), 7, 0.0), ((3, 4104), 2, 0.1),
                                           ((0, 64), 1, 0.01)])
def test_fused_adamw_requant_bitexact(cuda_device, shape, step, wd):
    """lema_adamw_requant_rows against the numpy restatement of the reference's
    AdamW step (bit for bit: each fp32 operation rounded once in the same
    order), the int8 rows against the quantisation contract of the new weight,
    and the accumulator cleared. Vector path (cols % 8 == 0) and scalar path."""
    from oracle import oracle as O
    from oracle.torch_ref import adamw_step_ref
    from lema_b200 import ops
    g0 = torch.Generator().manual_seed(shape[1] + step)
    w = (torch.randn(*shape, generator=g0) * 0.02).to(torch.bfloat16)
    g = torch.randn(*shape, generator=g0) * 1e-3
    m = torch.randn(*shape, generator=g0) * 1e-4
    v = torch.rand(*shape, generator=g0) * 1e-6
    lr = 1e-3
    ref_w, ref_m, ref_v = adamw_step_ref(O.torch_bf16_to_bits(w), g.numpy(), m.numpy(),
                                         v.numpy(), step, lr, wd)
    dev = cuda_device
    wd_, gd, md, vd = w.to(dev), g.to(dev), m.to(dev), v.to(dev)
    wq, sw = ops.adamw_requant_rows(wd_, gd, md, vd, step, lr, wd)
    np.testing.assert_array_equal(O.torch_bf16_to_bits(wd_.cpu()), ref_w)
    np.testing.assert_array_equal(md.cpu().numpy(), ref_m)
    np.testing.assert_array_equal(vd.cpu().numpy(), ref_v)
    assert not gd.any()
    if shape[0]:
        wq_ref, sw_ref = O.c_quantize_rows(ref_w)
        np.testing.assert_array_equal(wq.cpu().numpy(), wq_ref)
        np.testing.assert_array_equal(sw.cpu().numpy(), sw_ref)
