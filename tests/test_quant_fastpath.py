"""CPU check of the quantiser's fast element form (lema_b200/csrc/quant_core.cuh)
against the operator contract:

    p = x * RN(1/s) exactly (inside fma); t = RN(p + 1.5*2^23) = 1.5*2^23 + rint(p);
    d = RN(p - (t - 1.5*2^23))
    |d| <= 0.4999  ->  q = low byte of t's bits (two's complement) = rint(p)
    otherwise      ->  q = clamp(rint(RN(x / s)), -127, 127)  (exact division)

The fused products are emulated exactly in float64 (a product of two fp32 values
has at most 48 significant bits, and p - rint(p) is then exact too); t is
formed as the integer rint(p), which is what the fp32 sum rounds to when
|p| < 2^22.

The fast result must equal the contract wherever it is taken: over every bf16
value |x| <= amax for a spread of bf16 row maxima (the activations are bf16, so
amax and x are bf16 values), and over fp32 inputs placed within a few ulps of
the rounding ties."""
import numpy as np

MAGIC = np.float32(12582912.0)
GUARD = np.float32(0.4999)


def _fast(x: np.ndarray, s: np.float32):
    inv = np.float32(1.0) / s
    p = x.astype(np.float64) * np.float64(inv)        # exact
    r = np.rint(p)                                     # half to even
    d = (p - r).astype(np.float32)                     # one rounding of the exact distance
    ok = np.abs(d) <= GUARD
    t = (r + np.float64(MAGIC)).astype(np.float32)     # exact: |r| <= 2^22
    q = (t.view(np.uint32) & 0xFF).astype(np.uint8).view(np.int8).astype(np.int32)
    return q, ok


def _contract(x: np.ndarray, s: np.float32) -> np.ndarray:
    return np.clip(np.rint(x / s), -127, 127).astype(np.int32)


def _all_finite_bf16() -> np.ndarray:
    bits = np.arange(1 << 16, dtype=np.uint32) << 16
    v = bits.view(np.float32)
    return v[np.isfinite(v)]


def _row_scale(amax: np.float32) -> np.float32:
    return np.float32(amax) / np.float32(127.0) if amax > 0 else np.float32(1.0)


def test_fast_form_matches_contract_on_bf16_rows():
    allv = _all_finite_bf16()
    pos = np.unique(np.abs(allv[allv != 0]))
    rng = np.random.default_rng(0)
    # row maxima: random bf16 magnitudes across the normal range plus the edges
    # where 1/s is near overflow or s near the normal/subnormal boundary
    picks = list(rng.choice(pos[(pos > 1e-30) & (pos < 1e30)], 120, replace=False))
    picks += [np.float32(v) for v in (1.0, 127.0, 254.0, 0.5, 2.0 ** -100, 2.0 ** 100,
                                      3.0e38, 1.5e-36)]
    taken = total = 0
    with np.errstate(over="ignore", invalid="ignore"):
        for amax in picks:
            amax = np.float32(amax)
            s = _row_scale(amax)
            if not (s >= np.float32(1.17549435e-38)):
                continue  # subnormal scale: the kernel takes the exact division for the row
            x = allv[np.abs(allv) <= amax]
            q, ok = _fast(x, s)
            want = _contract(x, s)
            assert np.array_equal(q[ok], want[ok]), amax
            taken += int(ok.sum())
            total += x.size
    assert total > 1_000_000
    assert taken >= 0.99 * total  # the exact division is the rare path


def test_fast_form_near_ties_fp32():
    rng = np.random.default_rng(1)
    scales = (rng.uniform(1e-3, 1e3, 2000).astype(np.float32))
    k = rng.integers(-127, 127, 2000).astype(np.float32)
    out_taken = 0
    for delta in range(-6, 7):
        x = ((k + np.float32(0.5)) * scales).astype(np.float32)
        x = np.nextafter(x, np.float32(np.inf) if delta > 0 else np.float32(-np.inf))
        for _ in range(abs(delta) - 1):
            x = np.nextafter(x, np.float32(np.inf) if delta > 0 else np.float32(-np.inf))
        for i in range(0, x.size, 500):
            xs, ss = x[i:i + 500], scales[i:i + 500]
            for xv, sv in zip(xs, ss):
                q, ok = _fast(np.array([xv], np.float32), sv)
                if ok[0]:
                    out_taken += 1
                    assert q[0] == _contract(np.array([xv], np.float32), sv)[0], (xv, sv)
    # points this close to a tie must almost all be sent to the exact division
    assert out_taken < 0.05 * 13 * 2000


def test_fast_form_nan_goes_to_exact_path():
    q, ok = _fast(np.array([np.nan, 1.0], np.float32), np.float32(0.5))
    assert not ok[0] and ok[1] and q[1] == 2
