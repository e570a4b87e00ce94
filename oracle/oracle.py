"""CPU oracle for the W8A8 hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module; it is the checker, never the thing measured or
shipped. Two independent restatements of the operator contract written in
include/lema_b200.h live here:

* ``c_*``  functions: ctypes wrappers over oracle/w8a8_oracle.c
  (built by oracle/Makefile into oracle/_build/liboracle.so);
* ``np_*`` functions: a vectorised numpy restatement.

Tests check the two against each other and against hand-derived known
answers (tests/golden/). Parity status: the reference has no quantised linear
(README.md:143-145), so the quantiser / int8 GEMM / epilogue / dgrad rules
are UNPINNED against reference outputs; the unquantised layer math they plug
into is pinned by fixtures generated from the reference's own Python path
(tests/golden/make_golden.py).

bf16 arrays are carried as numpy uint16 (the raw bit pattern).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "_build" / "liboracle.so"

_lib = None


def build() -> Path:
    """Compiles the C oracle with the committed Makefile (gcc)."""
    src = ORACLE_DIR / "w8a8_oracle.c"
    if LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    r = subprocess.run(["make", "-C", str(ORACLE_DIR)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        p = C.c_void_p
        i = C.c_int64
        L.oracle_quantize_rows_bf16.argtypes = [p, i, i, i, p, i, p]
        L.oracle_quantize_rows_f32.argtypes = [p, i, i, i, p, i, p]
        L.oracle_int8_gemm.argtypes = [p, i, p, i, i, i, i, p, i]
        L.oracle_epilogue.argtypes = [p, i, p, p, p, i, i, p, i]
        L.oracle_dequant_transpose.argtypes = [p, i, p, i, i, p, i]
        L.oracle_bf16_gemm_tn.argtypes = [p, i, p, i, i, i, i, p, i, p]
        L.oracle_int8_gemm_checksums.argtypes = [p, i, p, i, i, i, i, p, p]
        L.oracle_set_threads.argtypes = [C.c_int]
        for f in ("oracle_quantize_rows_bf16", "oracle_quantize_rows_f32", "oracle_int8_gemm",
                  "oracle_epilogue", "oracle_dequant_transpose", "oracle_bf16_gemm_tn",
                  "oracle_int8_gemm_checksums", "oracle_set_threads"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------------------
# bf16 helpers (numpy)
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def torch_bf16_to_bits(t) -> np.ndarray:
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bits_to_torch_bf16(h: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(h).view(np.int16)).view(torch.bfloat16)


# ---------------------------------------------------------------------------
# C restatement
# ---------------------------------------------------------------------------

def c_quantize_rows(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x bf16 bits [R, C] -> (q int8 [R, C], scale fp32 [R])."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    R, Cc = x.shape
    q = np.empty((R, Cc), dtype=np.int8)
    s = np.empty(R, dtype=np.float32)
    lib().oracle_quantize_rows_bf16(_p(x), R, Cc, Cc, _p(q), Cc, _p(s))
    return q, s


def c_quantize_rows_f32(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, Cc = x.shape
    q = np.empty((R, Cc), dtype=np.int8)
    s = np.empty(R, dtype=np.float32)
    lib().oracle_quantize_rows_f32(_p(x), R, Cc, Cc, _p(q), Cc, _p(s))
    return q, s


def c_int8_gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    M, K = a.shape
    Nn = b.shape[0]
    acc = np.empty((M, Nn), dtype=np.int32)
    lib().oracle_int8_gemm(_p(a), K, _p(b), K, M, Nn, K, _p(acc), Nn)
    return acc


def c_epilogue(acc: np.ndarray, sx: np.ndarray, sw: np.ndarray,
               bias_bits: np.ndarray | None) -> np.ndarray:
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    M, Nn = acc.shape
    sx = np.ascontiguousarray(sx, dtype=np.float32)
    sw = np.ascontiguousarray(sw, dtype=np.float32)
    b = None if bias_bits is None else np.ascontiguousarray(bias_bits, dtype=np.uint16)
    y = np.empty((M, Nn), dtype=np.uint16)
    lib().oracle_epilogue(_p(acc), Nn, _p(sx), _p(sw), _p(b), M, Nn, _p(y), Nn)
    return y


def c_dequant_transpose(wq: np.ndarray, sw: np.ndarray) -> np.ndarray:
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    Nn, K = wq.shape
    out = np.empty((K, Nn), dtype=np.uint16)
    lib().oracle_dequant_transpose(_p(wq), K, _p(np.ascontiguousarray(sw, dtype=np.float32)),
                                   Nn, K, _p(out), Nn)
    return out


def c_bf16_gemm_tn(a_bits: np.ndarray, b_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(y bf16 bits, y fp32) of a . b^T accumulated in double."""
    a = np.ascontiguousarray(a_bits, dtype=np.uint16)
    b = np.ascontiguousarray(b_bits, dtype=np.uint16)
    M, K = a.shape
    Nn = b.shape[0]
    y = np.empty((M, Nn), dtype=np.uint16)
    yf = np.empty((M, Nn), dtype=np.float32)
    lib().oracle_bf16_gemm_tn(_p(a), K, _p(b), K, M, Nn, K, _p(y), Nn, _p(yf))
    return y, yf


def c_int8_gemm_checksums(a: np.ndarray, b: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Exact int64 row sums and column sums of a . b^T without forming it."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    M, K = a.shape
    Nn = b.shape[0]
    rs = np.empty(M, dtype=np.int64)
    cs = np.empty(Nn, dtype=np.int64)
    lib().oracle_int8_gemm_checksums(_p(a), K, _p(b), K, M, Nn, K, _p(rs), _p(cs))
    return rs, cs


# ---------------------------------------------------------------------------
# numpy restatement (independent of the C code)
# ---------------------------------------------------------------------------

def np_quantize_rows_f32(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32)
    amax = amax.astype(np.float32)
    s = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.rint(x / s[:, None]).astype(np.float32)  # numpy rint: ties to even
    q = np.clip(r, -127, 127).astype(np.int8)
    return q, s


def np_quantize_rows(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    return np_quantize_rows_f32(bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16)))


def np_int8_gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.astype(np.int32) @ b.astype(np.int32).T).astype(np.int32)


def np_epilogue(acc: np.ndarray, sx: np.ndarray, sw: np.ndarray,
                bias_bits: np.ndarray | None) -> np.ndarray:
    f = (acc.astype(np.float32) * sx.astype(np.float32)[:, None]).astype(np.float32)
    f = (f * sw.astype(np.float32)[None, :]).astype(np.float32)
    if bias_bits is not None:
        f = (f + bf16_bits_to_f32(bias_bits)[None, :]).astype(np.float32)
    return f32_to_bf16_bits(f)


def np_dequant_transpose(wq: np.ndarray, sw: np.ndarray) -> np.ndarray:
    f = (wq.astype(np.float32) * sw.astype(np.float32)[:, None]).astype(np.float32)
    return np.ascontiguousarray(f32_to_bf16_bits(f).T)


def w8a8_linear_ref(x_bits: np.ndarray, w_bits: np.ndarray, bias_bits: np.ndarray | None = None):
    """Full forward restated: quantise x per token and W per channel, int8 GEMM,
    epilogue. Returns dict with xq, sx, wq, sw, acc, y (bf16 bits)."""
    xq, sx = c_quantize_rows(x_bits)
    wq, sw = c_quantize_rows(w_bits)
    acc = c_int8_gemm(xq, wq)
    y = c_epilogue(acc, sx, sw, bias_bits)
    return {"xq": xq, "sx": sx, "wq": wq, "sw": sw, "acc": acc, "y": y}


def dgrad_int8_ref(dy_bits: np.ndarray, wq: np.ndarray, sw: np.ndarray):
    """The optional int8-dy variant of the frozen-base backward (straight-through
    estimator of src/lema/adapters/_llama.py:245-250 through both quantisers):
    g[m, n] = fp32(dy[m, n]) * sw[n] (one fp32 rounding), g quantised per row by
    the contract (dq, sd), acc = dq . wq in s32, dx = bf16(acc * sd[m]). Returns
    dict with g, dq, sd, acc, dx (bf16 bits)."""
    sw = np.ascontiguousarray(sw, dtype=np.float32)
    g = (bf16_bits_to_f32(np.asarray(dy_bits, dtype=np.uint16)) * sw[None, :]).astype(np.float32)
    dq, sd = c_quantize_rows_f32(g)
    acc = c_int8_gemm(dq, np.ascontiguousarray(np.asarray(wq, dtype=np.int8).T))
    dx = c_epilogue(acc, sd, np.ones(acc.shape[1], np.float32), None)
    return {"g": g, "dq": dq, "sd": sd, "acc": acc, "dx": dx}


def cfg1_inputs(seed: int = 0, M: int = 512, K: int = 4096, N: int = 4096,
                outlier_frac: float = 0.01):
    """Seeded single-linear workload: X ~ N(0,1) bf16 [M,K] with 1% of channels
    scaled x20, W ~ N(0, 0.02) bf16 [N,K], zero bias. Draw order fixed: X, channel
    permutation, W."""
    import torch
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    n_out = max(1, int(round(outlier_frac * K)))
    idx = torch.randperm(K, generator=g)[:n_out]
    x[:, idx] *= 20.0
    x = x.to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(N, dtype=torch.bfloat16)
    return x, w, bias


if __name__ == "__main__":
    print(build())
    os.environ.setdefault("OMP_NUM_THREADS", "1")


# ---------------------------------------------------------------------------
# fused producers (numpy restatements of HF LlamaRMSNorm, apply_rotary_pos_emb
# and LlamaMLP's act(gate) * up, with the bf16 roundings torch applies)
# ---------------------------------------------------------------------------

def _bf(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 and back to fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def np_rmsnorm(x_bits: np.ndarray, g_bits: np.ndarray, eps: float) -> np.ndarray:
    """hn bits = bf16(g * bf16(x * rsqrt(mean(x^2) + eps))), statistics in fp32."""
    x = bf16_bits_to_f32(x_bits)
    g = bf16_bits_to_f32(g_bits)
    var = (np.sum(x.astype(np.float64) ** 2, axis=1) / x.shape[1]).astype(np.float32)
    rstd = (1.0 / np.sqrt(var.astype(np.float64) + eps)).astype(np.float32)
    xh = _bf(x * rstd[:, None])
    return f32_to_bf16_bits(g[None, :] * xh)


def np_rope(x_bits: np.ndarray, cos_bits: np.ndarray, sin_bits: np.ndarray, seq: int,
            heads: int, d: int) -> np.ndarray:
    """x [T, heads*d] bits -> bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)) bits."""
    x = bf16_bits_to_f32(x_bits).reshape(-1, heads, d)
    T = x.shape[0]
    pos = np.arange(T) % seq
    c = bf16_bits_to_f32(cos_bits)[pos][:, None, :]
    s = bf16_bits_to_f32(sin_bits)[pos][:, None, :]
    rot = np.concatenate([-x[..., d // 2:], x[..., : d // 2]], axis=-1)
    out = _bf(_bf(x * c) + _bf(rot * s))
    return f32_to_bf16_bits(out.reshape(T, heads * d))


def np_swiglu(gu_bits: np.ndarray) -> np.ndarray:
    """rows of [gate | up] bits -> bf16(bf16(silu(gate)) * up) bits."""
    gu = bf16_bits_to_f32(gu_bits)
    I = gu.shape[1] // 2
    gate, up = gu[:, :I], gu[:, I:]
    a = _bf((gate / (np.float32(1) + np.exp(-gate))).astype(np.float32))
    return f32_to_bf16_bits(a * up)
