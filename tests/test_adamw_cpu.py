"""Host side of the fused AdamW + re-quantisation step: the fp32 coefficients
that ``ops.adamw_requant_rows`` passes to the kernel, applied in the kernel's
per-element order (each fp32 operation rounded once), reproduce the numpy
restatement of the reference's AdamW step (src/lema/_full_ft.py:204-229) bit
for bit. No GPU: the element order is emulated with numpy fp32 operations."""
import numpy as np
import pytest

from lema_b200 import ops


def _kernel_order(w_bits, g, m, v, coef):
    from oracle import oracle as O
    decay, beta1, c1, beta2, c2, sqrt_bc2, step_size, eps = (np.float32(c) for c in coef)
    w = O.bf16_bits_to_f32(w_bits) * decay
    m = m * beta1 + g * c1
    v = v * beta2 + (g * g) * c2
    d = np.sqrt(v) / sqrt_bc2 + eps
    w = w + step_size * (m / d)
    return O.f32_to_bf16_bits(w.astype(np.float32)), m.astype(np.float32), v.astype(np.float32)


@pytest.mark.parametrize("step,lr,wd", [(1, 1e-3, 0.01), (3, 1e-4, 0.0), (250, 3e-3, 0.1)])
def test_coefficients_and_order_match_reference_restatement(step, lr, wd):
    from oracle import oracle as O
    from oracle.torch_ref import adamw_step_ref
    rng = np.random.default_rng(step)
    w = O.f32_to_bf16_bits((rng.standard_normal((7, 96)) * 0.02).astype(np.float32))
    g = (rng.standard_normal((7, 96)) * 1e-3).astype(np.float32)
    m = (rng.standard_normal((7, 96)) * 1e-4).astype(np.float32)
    v = (rng.random((7, 96)) * 1e-6).astype(np.float32)
    coef = ops.adamw_coefficients(step, lr, wd)
    assert all(float(np.float32(c)) == c for c in coef)  # exact fp32 values
    got = _kernel_order(w, g, m, v, coef)
    ref = adamw_step_ref(w, g, m, v, step, lr, wd)
    for a, b in zip(got, ref):
        np.testing.assert_array_equal(a, b)
    # the int8 rows of the new weight follow the quantisation contract
    q, s = O.c_quantize_rows(got[0])
    qn, sn = O.np_quantize_rows(got[0])
    np.testing.assert_array_equal(q, qn)
    np.testing.assert_array_equal(s, sn)


def test_no_weight_decay_is_a_unit_multiply():
    assert ops.adamw_coefficients(5, 1e-3, 0.0)[0] == 1.0
