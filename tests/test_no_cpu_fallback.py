"""The product path has no CPU fallback: every public op refuses tensors that
are not on a CUDA device with an error before any work, so a CPU run can never
pass silently on a host implementation. (The oracle under oracle/ is the only
CPU implementation, and it is test infrastructure.)"""
import pytest
import torch

from lema_b200 import ops


def _cases():
    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    wq = torch.zeros(8, 16, dtype=torch.int8)
    sw = torch.ones(8)
    g = torch.ones(16, dtype=torch.bfloat16)
    f32 = torch.zeros(8, 16)
    yield "quantize_rows", lambda: ops.quantize_rows(x)
    yield "quantize_weight", lambda: ops.quantize_weight(x)
    yield "w8a8_linear", lambda: ops.w8a8_linear(x, wq, sw)
    yield "w8a8_dgrad", lambda: ops.w8a8_dgrad(torch.zeros(4, 8, dtype=torch.bfloat16), wq, sw)
    yield "rmsnorm_quant", lambda: ops.rmsnorm_quant(x, g, 1e-5)
    yield "swiglu_quant", lambda: ops.swiglu_quant(torch.zeros(4, 32, dtype=torch.bfloat16))
    yield "adamw_requant_rows", lambda: ops.adamw_requant_rows(
        torch.zeros(8, 16, dtype=torch.bfloat16), f32, f32.clone(), f32.clone(), 1, 1e-3, 0.0)
    q = torch.zeros(128, 128, dtype=torch.bfloat16)
    yield "attention_fwd", lambda: ops.attention_fwd(q, q, q, 1, 128, 1, 1, 128 ** -0.5)


@pytest.mark.parametrize("name,call", list(_cases()), ids=[n for n, _ in _cases()])
def test_op_refuses_cpu_tensors(name, call):
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        call()
