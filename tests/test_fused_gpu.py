"""The fused producers of the block's fast path against numpy restatements of
the torch/HF math they replace: RoPE bit-exact; SwiGLU within one bf16 ulp and
RMSNorm within two (the device's rsqrt / exp differ from the host's in the last
fp32 bit, which can move a bf16 rounding), with the int8 rows then bit-exact against the
quantiser applied to the device's own bf16 output; backward kernels against
fp64 formulas at bf16 tolerance."""
import numpy as np
import pytest
import torch

from lema_b200 import ops

pytestmark = pytest.mark.gpu


def bits(t):
    from oracle.oracle import torch_bf16_to_bits
    return torch_bf16_to_bits(t)


def _ulp_check(got_bits, ref_bits, frac_exact=0.999, max_ulp=1):
    d = np.abs(got_bits.astype(np.int32) - ref_bits.astype(np.int32))
    assert d.max() <= max_ulp, d.max()
    assert (d == 0).mean() >= frac_exact, (d == 0).mean()


@pytest.mark.parametrize("M,H", [(512, 4096), (37, 11008), (5, 64)])
def test_rmsnorm_quant(cuda_device, oracle, M, H):
    g = torch.Generator().manual_seed(M + H)
    x = (torch.randn(M, H, generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    hn, xq, sx, rstd = ops.rmsnorm_quant(x.to(cuda_device), w.to(cuda_device), 1e-5)
    # two stacked bf16 roundings (x*rstd, then g*.): a last-bit rstd difference
    # can move the result by up to 2 ulps
    _ulp_check(bits(hn), oracle.np_rmsnorm(bits(x), bits(w), 1e-5), max_ulp=2)
    q_ref, s_ref = oracle.c_quantize_rows(bits(hn))
    np.testing.assert_array_equal(xq.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sx.cpu().numpy(), s_ref)


def test_rmsnorm_bwd(cuda_device):
    g = torch.Generator().manual_seed(3)
    M, H = 64, 4096
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    dhn = torch.randn(M, H, generator=g).to(torch.bfloat16)
    _, _, _, rstd = ops.rmsnorm_quant(x.to(cuda_device), w.to(cuda_device), 1e-5, want_q=False)
    dx = ops.rmsnorm_bwd(x.to(cuda_device), w.to(cuda_device), rstd, dhn.to(cuda_device))
    xd = x.double().requires_grad_(True)
    y = w.double() * (xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-5))
    y.backward(dhn.double())
    ref = xd.grad
    err = (dx.double().cpu() - ref).abs()
    assert (err <= 2 ** -7 * ref.abs() + 2 ** -9 * ref.pow(2).mean().sqrt()).all(), err.max()


@pytest.mark.parametrize("hq,hk", [(32, 32), (32, 8)])
def test_rope_forward_bitexact_and_backward(cuda_device, oracle, hq, hk):
    from lema_b200.llama import LlamaShape, rope_cos_sin
    d, S, B = 128, 96, 2
    shape = LlamaShape(hidden=hq * d, heads=hq, kv_heads=hk)
    cos, sin = rope_cos_sin(shape, S, cuda_device, torch.bfloat16)
    cos, sin = cos[0], sin[0]
    g = torch.Generator().manual_seed(hq + hk)
    qkv = torch.randn(B * S, (hq + 2 * hk) * d, generator=g).to(torch.bfloat16).to(cuda_device)
    q, k = qkv[:, : hq * d], qkv[:, hq * d:(hq + hk) * d]  # strided rows, as the QKV GEMM gives
    qo, ko = ops.rope(q, k, cos, sin, S, hq, hk, d, 0)
    cb, sb = bits(cos), bits(sin)
    np.testing.assert_array_equal(bits(qo), oracle.np_rope(bits(q.contiguous()), cb, sb, S, hq, d))
    np.testing.assert_array_equal(bits(ko), oracle.np_rope(bits(k.contiguous()), cb, sb, S, hk, d))
    # backward = transposed rotation: <rope(x), y> == <x, rope_bwd(y)> in fp64
    dq = torch.randn(B * S, hq * d, generator=g).to(torch.bfloat16).to(cuda_device)
    dk = torch.randn(B * S, hk * d, generator=g).to(torch.bfloat16).to(cuda_device)
    gq, gk = ops.rope(dq, dk, cos, sin, S, hq, hk, d, 1)
    c = cos.double().repeat(B, 1)[:, None, :].cpu()
    s_ = sin.double().repeat(B, 1)[:, None, :].cpu()

    def rot_t(y, h):
        y = y.double().cpu().view(-1, h, d)
        a, b = y[..., : d // 2], y[..., d // 2:]
        # transpose of x -> x*c + rotate_half(x)*s
        return (y * c + torch.cat([b * s_[..., d // 2:], -a * s_[..., : d // 2]], -1)).view(-1, h * d)
    for got, ref in ((gq, rot_t(dq, hq)), (gk, rot_t(dk, hk))):
        err = (got.double().cpu() - ref).abs()
        assert (err <= 2 ** -8 * ref.abs() + 1e-6).all(), err.max()


@pytest.mark.parametrize("M,I", [(256, 11008), (9, 128)])
def test_swiglu_quant_and_bwd(cuda_device, oracle, M, I):
    g = torch.Generator().manual_seed(M + I)
    gu = (torch.randn(M, 2 * I, generator=g) * 2).to(torch.bfloat16)
    mq, sm, m = ops.swiglu_quant(gu.to(cuda_device), want_m=True)
    _ulp_check(bits(m), oracle.np_swiglu(bits(gu)))
    q_ref, s_ref = oracle.c_quantize_rows(bits(m))
    np.testing.assert_array_equal(mq.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sm.cpu().numpy(), s_ref)
    dm = torch.randn(M, I, generator=g).to(torch.bfloat16)
    dgu = ops.swiglu_bwd(gu.to(cuda_device), dm.to(cuda_device)).double().cpu()
    gd = gu.double()
    gate, up = gd[:, :I].requires_grad_(True), gd[:, I:].requires_grad_(True)
    (torch.nn.functional.silu(gate) * up).backward(dm.double())
    ref = torch.cat([gate.grad, up.grad], 1)
    err = (dgu - ref).abs()
    assert (err <= 2 ** -7 * ref.abs() + 1e-5).all(), err.max()


def test_rope_qkv_with_lora_addends(cuda_device, oracle):
    """q/k/v of a stacked projection plus LoRA addends: rotate(bf16(q + lq)),
    rotate(bf16(k)), bf16(v + lv) made contiguous — bit-exact against torch's
    composition of the same bf16 ops."""
    from lema_b200.llama import LlamaShape, apply_rope, rope_cos_sin
    d, S, B, hq, hk = 128, 64, 2, 32, 8
    shape = LlamaShape(hidden=hq * d, heads=hq, kv_heads=hk)
    cos, sin = rope_cos_sin(shape, S, cuda_device, torch.bfloat16)
    g = torch.Generator(device=cuda_device).manual_seed(4)
    qkv = torch.randn(B * S, (hq + 2 * hk) * d, device=cuda_device, generator=g).to(torch.bfloat16)
    q, k, v = qkv[:, :hq * d], qkv[:, hq * d:(hq + hk) * d], qkv[:, (hq + hk) * d:]
    lq = torch.randn(B * S, hq * d, device=cuda_device, generator=g).to(torch.bfloat16) * 0.1
    lv = torch.randn(B * S, hk * d, device=cuda_device, generator=g).to(torch.bfloat16) * 0.1
    qo, ko, vo = ops.rope_qkv(q, k, v, lq, None, lv, cos[0], sin[0], S, hq, hk, d)
    qt = (q + lq).view(B, S, hq, d).transpose(1, 2)
    kt = k.reshape(B, S, hk, d).transpose(1, 2)
    qr, kr = apply_rope(qt, kt, cos, sin)
    assert torch.equal(qo.view(torch.int16), qr.transpose(1, 2).reshape(B * S, -1).view(torch.int16))
    assert torch.equal(ko.view(torch.int16), kr.transpose(1, 2).reshape(B * S, -1).view(torch.int16))
    assert torch.equal(vo.view(torch.int16), (v + lv).view(torch.int16))
