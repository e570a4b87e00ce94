"""The tcgen05 causal attention against an fp32 restatement of the torch op it
replaces (scaled_dot_product_attention(q, k, v, is_causal=True, scale=d**-0.5,
enable_gqa=...)) on the same bf16 inputs. The bar is set by torch's own bf16
SDPA: the kernel's error against the fp32 result stays within twice SDPA's
(plus a floor of one bf16 ulp at the output's scale), and its log-sum-exp
matches the fp32 one to 1e-3 (log2 units)."""
import math

import pytest
import torch
import torch.nn.functional as F

from lema_b200 import ops

pytestmark = pytest.mark.gpu

D = 128


def _inputs(B, S, H, Hkv, seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B * S, H * D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B * S, Hkv * D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B * S, Hkv * D, generator=g).to(torch.bfloat16).to(dev)
    return q, k, v


def _heads(t, B, S, n):
    return t.view(B, S, n, D).transpose(1, 2)


def _ref_fp32(q, k, v, B, S, H, Hkv):
    """fp32 causal attention and the log2-domain log-sum-exp of the scaled scores."""
    qh, kh, vh = (_heads(t.float(), B, S, n) for t, n in ((q, H), (k, Hkv), (v, Hkv)))
    kh = kh.repeat_interleave(H // Hkv, dim=1)
    vh = vh.repeat_interleave(H // Hkv, dim=1)
    s = (qh @ kh.transpose(-1, -2)) * D ** -0.5
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse2 = torch.logsumexp(s, dim=-1) / math.log(2.0)
    o = torch.softmax(s, dim=-1) @ vh
    return o, lse2


# The forward runs one query tile per CTA while B * H * (pairs of tiles) is below the SM
# count (every shape up to (1, 640, 2, 1) here) and pairs of tiles above it:
# (1, 2048, 20, 4) has 160 pairs, (1, 640, 64, 8) 192 pairs of five tiles, whose last
# pair has no second tile.
SHAPES = [(1, 128, 1, 1), (2, 256, 4, 2), (1, 200, 2, 2), (2, 512, 8, 2), (1, 2048, 4, 1),
          (3, 77, 2, 1), (1, 640, 2, 1), (1, 2048, 20, 4), (1, 640, 64, 8)]


@pytest.mark.parametrize("B,S,H,Hkv", SHAPES)
def test_forward_matches_fp32_within_sdpa_error(cuda_device, B, S, H, Hkv):
    q, k, v = _inputs(B, S, H, Hkv, B * 1000 + S + H, cuda_device)
    o, lse = ops.attention_fwd(q, k, v, B, S, H, Hkv, D ** -0.5)
    torch.cuda.synchronize()
    o_ref, lse_ref = _ref_fp32(q, k, v, B, S, H, Hkv)
    o_sdpa = F.scaled_dot_product_attention(_heads(q, B, S, H), _heads(k, B, S, Hkv),
                                            _heads(v, B, S, Hkv), is_causal=True,
                                            scale=D ** -0.5, enable_gqa=H != Hkv)
    got = _heads(o, B, S, H).float()
    err = (got - o_ref).abs().max().item()
    err_sdpa = (o_sdpa.float() - o_ref).abs().max().item()
    floor = 2 ** -8 * o_ref.abs().max().item()
    assert err <= 2 * err_sdpa + floor, (err, err_sdpa)
    assert torch.isfinite(got).all()
    assert (lse - lse_ref).abs().max().item() <= 1e-3


BWD_SHAPES = [(1, 128, 1, 1), (2, 256, 4, 2), (1, 200, 2, 2), (2, 512, 8, 2), (1, 2048, 4, 1),
              (3, 77, 2, 1), (1, 640, 2, 1)]


@pytest.mark.parametrize("B,S,H,Hkv", BWD_SHAPES)
def test_backward_matches_fp32_within_sdpa_error(cuda_device, B, S, H, Hkv):
    """dq, dk, dv against fp32 autograd of the same op; the bar is twice torch
    bf16 SDPA's own error on the same gradients plus one bf16 ulp at scale."""
    q, k, v = _inputs(B, S, H, Hkv, 7 * S + H, cuda_device)
    g = torch.Generator(device="cpu").manual_seed(S + 3)
    do = torch.randn(B * S, H * D, generator=g).to(torch.bfloat16).to(cuda_device)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = ops.AttentionFn.apply(qg, kg, vg, B, S, H, Hkv, D ** -0.5)
    o.backward(do)
    torch.cuda.synchronize()

    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    o_ref, _ = _ref_fp32(qf, kf, vf, B, S, H, Hkv)
    o_ref.transpose(1, 2).reshape(B * S, H * D).backward(do.float())

    qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
    o_s = F.scaled_dot_product_attention(_heads(qs, B, S, H), _heads(ks, B, S, Hkv),
                                         _heads(vs, B, S, Hkv), is_causal=True,
                                         scale=D ** -0.5, enable_gqa=H != Hkv)
    o_s.transpose(1, 2).reshape(B * S, H * D).backward(do)
    for name, got, ref, sd in (("dq", qg.grad, qf.grad, qs.grad), ("dk", kg.grad, kf.grad, ks.grad),
                               ("dv", vg.grad, vf.grad, vs.grad)):
        assert torch.isfinite(got).all(), name
        err = (got.float() - ref).abs().max().item()
        err_sdpa = (sd.float() - ref).abs().max().item()
        floor = 2 ** -8 * ref.abs().max().item()
        assert err <= 2 * err_sdpa + floor, (name, err, err_sdpa)


@pytest.mark.parametrize("moe", [False, True])
def test_trainer_step_with_tcgen05_attention_matches_sdpa(cuda_device, moe):
    """The streamed LoRA trainer with attn_impl='tcgen05' against the same trainer
    on torch SDPA (head_dim 128, GQA, a ragged 200-token sequence): same loss to
    2e-3 relative and LoRA gradients to 3e-2 relative (Frobenius), the spread
    two bf16 attention implementations leave after the W8A8 quantisers."""
    from lema_b200.llama import LlamaShape
    from lema_b200.moe import MixtralShape
    from lema_b200.trainer import StreamedLoraTrainer
    shape = (MixtralShape(hidden=256, heads=2, kv_heads=1, intermediate=256, vocab=512,
                          layers=2, experts=4, top_k=2) if moe else
             LlamaShape(hidden=256, heads=2, kv_heads=1, intermediate=512, vocab=512, layers=2))
    g = torch.Generator(device="cpu").manual_seed(9)
    ids = torch.randint(0, shape.vocab, (2, 200), generator=g).to(cuda_device)
    out = {}
    for impl in ("sdpa", "tcgen05"):
        tr = StreamedLoraTrainer(shape, cuda_device, batch=2, seq=200, seed=3, grad_accum=2,
                                 attn_impl=impl)
        loss = float(tr.train_step(ids))  # first micro-step: gradients stay in .grad
        grads = [p.grad.detach().float().clone() for p in tr.params]
        tr.close()
        out[impl] = (loss, grads)
    (l_ref, g_ref), (l_tc, g_tc) = out["sdpa"], out["tcgen05"]
    assert abs(l_tc - l_ref) <= 2e-3 * abs(l_ref), (l_tc, l_ref)
    for a, b in zip(g_tc, g_ref):
        rel = ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
        assert rel <= 3e-2, rel


@pytest.mark.parametrize("B,S,H,Hkv", [(2, 256, 4, 2), (1, 200, 8, 2)])
def test_backward_gqa_without_head_split(cuda_device, B, S, H, Hkv):
    """The GQA backward with one CTA per kv head (no workspace: the group's
    query heads accumulate in TMEM) against the split one and the fp32 autograd
    reference, at the same bar."""
    q, k, v = _inputs(B, S, H, Hkv, 5 * S + H, cuda_device)
    g = torch.Generator(device="cpu").manual_seed(S + 1)
    do = torch.randn(B * S, H * D, generator=g).to(torch.bfloat16).to(cuda_device)
    o, lse = ops.attention_fwd(q, k, v, B, S, H, Hkv, D ** -0.5)
    grouped = ops.attention_bwd(q, k, v, o, lse, do, B, S, H, Hkv, D ** -0.5, split_heads=False)
    split = ops.attention_bwd(q, k, v, o, lse, do, B, S, H, Hkv, D ** -0.5)
    torch.cuda.synchronize()
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    o_ref, _ = _ref_fp32(qf, kf, vf, B, S, H, Hkv)
    o_ref.transpose(1, 2).reshape(B * S, H * D).backward(do.float())
    for name, a, b_, ref in zip(("dq", "dk", "dv"), grouped, split, (qf.grad, kf.grad, vf.grad)):
        floor = 2 ** -8 * ref.abs().max().item()
        scale = ref.abs().max().item()
        for got in (a, b_):
            assert torch.isfinite(got).all(), name
            assert (got.float() - ref).abs().max().item() <= 2e-2 * scale + floor, name
        # the two orders of summing the group's heads agree to bf16 rounding
        assert (a.float() - b_.float()).abs().max().item() <= 2 ** -7 * scale, name
