"""CPU tests of the oracle itself: the C and numpy restatements agree with each
other and with exact rational arithmetic on hand-picked known answers, and the
committed golden fixture still reproduces."""
from fractions import Fraction
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).parent / "golden"


def _exact_quant_row(vals):
    """Exact rational restatement: s = fp32(amax / 127), q = round_half_even(x / s)."""
    xs = np.asarray(vals, dtype=np.float32)
    amax = float(np.max(np.abs(xs))) if len(xs) else 0.0
    s = np.float32(amax) / np.float32(127.0) if amax > 0 else np.float32(1.0)
    out = []
    for v in xs:
        r = Fraction(float(v)) / Fraction(float(s))
        fl = r.numerator // r.denominator
        frac = r - fl
        if frac > Fraction(1, 2) or (frac == Fraction(1, 2) and fl % 2 == 1):
            fl += 1
        q_exact = max(-127, min(127, fl))
        out.append(q_exact)
    return out, s


def _to_bits(rows):
    t = torch.tensor(rows, dtype=torch.float32).to(torch.bfloat16)
    from oracle.oracle import torch_bf16_to_bits
    return torch_bf16_to_bits(t)


KNOWN_ROWS = [
    [127.0, -63.5, 0.5, -0.5, 1.5, 2.5, -2.5, 126.5],  # s = 1: ties go to even
    [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],          # zero row: s = 1, q = 0
    [254.0, 1.0, -1.0, 3.0, -254.0, 2.0, 0.0, 6.0],    # s = 2
    [1.0, 0.5, -0.5, 0.25, 0.125, -1.0, 0.75, 0.0],    # s = fp32(1/127)
    [-3.0, 1e-3, 2e-3, -1e-3, 0.0, 3.0, 1.5, -1.5],
]


def test_known_answers_exact(oracle):
    bits = _to_bits(KNOWN_ROWS)
    qc, sc = oracle.c_quantize_rows(bits)
    qn, sn = oracle.np_quantize_rows(bits)
    f = oracle.bf16_bits_to_f32(bits)
    for r in range(len(KNOWN_ROWS)):
        q_exact, s_exact = _exact_quant_row(f[r])
        assert sc[r] == s_exact and sn[r] == s_exact
        assert list(qc[r]) == q_exact, (r, list(qc[r]), q_exact)
        assert list(qn[r]) == q_exact
    # spot values of the first row: ties to even
    assert list(qc[0][:7]) == [127, -64, 0, 0, 2, 2, -2]
    assert sc[1] == 1.0 and not qc[1].any()
    assert sc[2] == 2.0 and list(qc[2]) == [127, 0, 0, 2, -127, 1, 0, 3]


@pytest.mark.parametrize("shape", [(7, 33), (64, 4096), (3, 11008), (1, 1), (5, 0)])
def test_c_matches_numpy_quantiser(oracle, shape):
    g = torch.Generator().manual_seed(shape[0] * 1000 + shape[1])
    x = torch.randn(*shape, generator=g) * 3.0
    if shape[1] > 4:
        x[:, : shape[1] // 50 + 1] *= 20.0
    if shape[0] > 2:
        x[1] = 0.0
    bits = oracle.torch_bf16_to_bits(x.to(torch.bfloat16))
    qc, sc = oracle.c_quantize_rows(bits)
    qn, sn = oracle.np_quantize_rows(bits)
    np.testing.assert_array_equal(qc, qn)
    np.testing.assert_array_equal(sc, sn)
    xf = x.float().numpy()
    qc32, sc32 = oracle.c_quantize_rows_f32(xf)
    qn32, sn32 = oracle.np_quantize_rows_f32(xf)
    np.testing.assert_array_equal(qc32, qn32)
    np.testing.assert_array_equal(sc32, sn32)


def test_gemm_epilogue_dequant_agree(oracle):
    rng = np.random.default_rng(1)
    a = rng.integers(-127, 128, size=(37, 300), dtype=np.int8)
    b = rng.integers(-127, 128, size=(45, 300), dtype=np.int8)
    acc_c = oracle.c_int8_gemm(a, b)
    np.testing.assert_array_equal(acc_c, oracle.np_int8_gemm(a, b))
    rs, cs = oracle.c_int8_gemm_checksums(a, b)
    np.testing.assert_array_equal(rs, acc_c.astype(np.int64).sum(1))
    np.testing.assert_array_equal(cs, acc_c.astype(np.int64).sum(0))
    sx = rng.random(37, dtype=np.float32) * 0.1 + 1e-3
    sw = rng.random(45, dtype=np.float32) * 1e-3 + 1e-5
    bias = oracle.f32_to_bf16_bits(rng.standard_normal(45).astype(np.float32))
    for bb in (None, bias):
        np.testing.assert_array_equal(oracle.c_epilogue(acc_c, sx, sw, bb),
                                      oracle.np_epilogue(acc_c, sx, sw, bb))
    np.testing.assert_array_equal(oracle.c_dequant_transpose(b, sw),
                                  oracle.np_dequant_transpose(b, sw))


def test_int8_dgrad_restatement(oracle):
    """The int8-dy dgrad chain (C) agrees with the same chain in numpy, and with
    unit scales it is the exact integer product."""
    rng = np.random.default_rng(4)
    dy = oracle.f32_to_bf16_bits(rng.standard_normal((21, 90)).astype(np.float32))
    wq = rng.integers(-127, 128, size=(90, 33), dtype=np.int8)
    sw = rng.random(90, dtype=np.float32) * 1e-3 + 1e-5
    out = oracle.dgrad_int8_ref(dy, wq, sw)
    g = (oracle.bf16_bits_to_f32(dy) * sw[None, :]).astype(np.float32)
    dq, sd = oracle.np_quantize_rows_f32(g)
    np.testing.assert_array_equal(out["dq"], dq)
    np.testing.assert_array_equal(out["sd"], sd)
    acc = oracle.np_int8_gemm(dq, np.ascontiguousarray(wq.T))
    np.testing.assert_array_equal(out["acc"], acc)
    np.testing.assert_array_equal(out["dx"],
                                  oracle.np_epilogue(acc, sd, np.ones(33, np.float32), None))
    # dx approximates dy . (wq * sw) to the quantiser's resolution
    exact = oracle.bf16_bits_to_f32(dy).astype(np.float64) @ (wq * sw[:, None]).astype(np.float64)
    got = oracle.bf16_bits_to_f32(out["dx"]).astype(np.float64)
    rel = np.sqrt(np.mean((got - exact) ** 2) / np.mean(exact ** 2))
    assert rel < 2e-2, rel


def test_bf16_gemm_reference_close_to_torch(oracle):
    g = torch.Generator().manual_seed(3)
    a = torch.randn(19, 70, generator=g).to(torch.bfloat16)
    b = torch.randn(23, 70, generator=g).to(torch.bfloat16)
    y, yf = oracle.c_bf16_gemm_tn(oracle.torch_bf16_to_bits(a), oracle.torch_bf16_to_bits(b))
    ref = (a.double() @ b.double().T).float().numpy()
    np.testing.assert_allclose(yf, ref, rtol=1e-6, atol=1e-6)


def test_golden_fixture_reproduces(oracle):
    """tests/golden/w8a8_cfg1_slice.npz was written by tests/golden/make_golden.py;
    the oracle must still reproduce it bit for bit."""
    path = GOLDEN / "w8a8_cfg1_slice.npz"
    d = np.load(path)
    out = oracle.w8a8_linear_ref(d["x"], d["w"], d["bias"])
    for k in ("xq", "sx", "wq", "sw", "acc", "y"):
        np.testing.assert_array_equal(out[k], d[k], err_msg=k)


def test_cfg1_inputs_seeded():
    from oracle.oracle import cfg1_inputs
    x1, w1, b1 = cfg1_inputs(seed=0, M=8, K=64, N=16)
    x2, w2, b2 = cfg1_inputs(seed=0, M=8, K=64, N=16)
    assert torch.equal(x1.view(torch.int16), x2.view(torch.int16))
    assert torch.equal(w1.view(torch.int16), w2.view(torch.int16))
    assert x1.dtype == torch.bfloat16 and w1.shape == (16, 64) and not b1.any()


def test_adamw_restatement_pinned_to_reference(oracle):
    """tests/golden/full_ft_adamw.npz was written by tests/golden/make_golden_adamw.py
    from the reference's own clip and AdamW step (src/lema/_full_ft.py:194-229).
    The oracle's numpy restatement (which the fused kernel matches bit for bit)
    reproduces each step from the reference's state: the clip norm to 1e-6, the
    moments to 1e-6 relative (1e-10 absolute near zero; the reference's CPU
    addcmul_ may fuse its multiply-add) and every bf16 weight bit for bit."""
    from oracle.torch_ref import adamw_step_ref
    d = np.load(GOLDEN / "full_ft_adamw.npz")
    names = sorted({k.split("/")[1] for k in d.files if k.startswith("w0/")})
    w = {n: d[f"w0/{n}"] for n in names}
    m = {n: np.zeros(d[f"g1/{n}"].shape, np.float32) for n in names}
    v = {n: np.zeros(d[f"g1/{n}"].shape, np.float32) for n in names}
    for step in (1, 2, 3):
        g = {n: d[f"g{step}/{n}"].astype(np.float32) for n in names}
        total = sum(float(np.sum(g[n].astype(np.float32) ** 2, dtype=np.float32)) for n in names)
        ref_norm = float(d[f"norm{step}"])
        assert abs(np.sqrt(total) - ref_norm) <= 1e-6 * ref_norm
        if ref_norm > 1.0:
            g = {n: (g[n] * np.float32(1.0 / ref_norm)).astype(np.float32) for n in names}
        for n in names:
            nw, nm, nv = adamw_step_ref(w[n], g[n], m[n], v[n], step, 1e-3, 0.01)
            # one rounding apart where the reference's multiply-add is fused
            np.testing.assert_allclose(nm, d[f"m{step}/{n}"], rtol=1e-6, atol=1e-10)
            np.testing.assert_allclose(nv, d[f"v{step}/{n}"], rtol=1e-6, atol=1e-14)
            ref_w = d[f"w{step}/{n}"]
            np.testing.assert_array_equal(nw, ref_w, err_msg=f"step {step} {n}")
            # the next step starts from the reference's state
            w[n], m[n], v[n] = ref_w, d[f"m{step}/{n}"], d[f"v{step}/{n}"]
