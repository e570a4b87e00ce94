"""Torch-facing W8A8 operators over the C ABI.

These are the host-side mirror of the op the reference runs at every
projection of a streamed decoder layer: ``nn.Linear`` inside HF
``LlamaDecoderLayer`` (created at adapters/_llama.py:80, called at
adapters/_llama.py:245-250), wrapped by ``LoRAWrapper.forward``
(_lora.py:23-26). The quantised operator is defined in include/lema_b200.h:

* ``quantize_rows``      per-row symmetric int8 (per token / per output channel)
* ``w8a8_gemm``          int8 x int8 -> s32 (tcgen05) + dequant/bias/bf16 epilogue
* ``w8a8_linear``        differentiable y = x W^T (+ b) with straight-through
                         backward dx = dy . (wq * sw) through ``w8a8_dgrad``
* ``grouped_w8a8_gemm``  the same per expert over pre-sorted token ranges

All tensors must live on a CUDA device; there is no CPU fallback. Calls run
on the current torch stream of the tensors' device.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _native as N


class GemmTimer:
    """Optional timing of every int8 GEMM launch (for the bench's roofline): the
    library records a pre-created CUDA event pair around each launch on its
    stream (``lema_gemm_timer_start`` / ``lema_gemm_timer_stop``), so a timed
    step runs the same fused entry points as an untimed one."""

    enabled = False
    max_records = 1 << 16
    dropped = 0

    @classmethod
    def enable(cls, on: bool = True) -> None:
        if on:
            N.call("lema_gemm_timer_start", cls.max_records)
        elif cls.enabled:
            cls.summary()
        cls.enabled = on

    @classmethod
    def summary(cls) -> tuple[float, float, int]:
        """(total ops, total ms, launches) over the recorded GEMMs since
        ``enable()`` (synchronises; recording stops)."""
        ops_, ms = C.c_double(0.0), C.c_double(0.0)
        n, dropped = C.c_int64(0), C.c_int64(0)
        N.call("lema_gemm_timer_stop", C.byref(ops_), C.byref(ms), C.byref(n), C.byref(dropped))
        cls.enabled = False
        cls.dropped = dropped.value
        return ops_.value, ms.value, n.value


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "lema_b200 ops run only on CUDA tensors (no CPU fallback); got a tensor on "
                f"{t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    if dev is None:
        raise RuntimeError("no tensor given")
    return dev


def _rows_view(t: torch.Tensor) -> torch.Tensor:
    """2-D view with unit stride along the last dim (copies only if needed)."""
    if t.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(t.shape)}")
    if t.stride(1) != 1 or t.stride(0) < t.shape[1]:
        t = t.contiguous()
    return t


def _ld(t: torch.Tensor) -> int:
    return t.stride(0) if t.shape[0] > 1 else max(t.shape[1], t.stride(0))


def pad_to(n: int, m: int) -> int:
    return (n + m - 1) // m * m


# ---------------------------------------------------------------------------
# K1: quantisation
# ---------------------------------------------------------------------------

def quantize_rows(x: torch.Tensor, out: torch.Tensor | None = None,
                  scale: torch.Tensor | None = None, ldq: int | None = None
                  ) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row int8 quantisation of a bf16 or fp32 [R, C] tensor.

    Returns (q int8 [R, C] (a view of an [R, ldq] buffer), scale fp32 [R]).
    ``ldq`` defaults to C rounded up to 16 so the result can feed the GEMM.
    """
    dev = _require_cuda(x)
    x = _rows_view(x)
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"quantize_rows takes bf16 or fp32, got {x.dtype}")
    rows, cols = x.shape
    if ldq is None:
        ldq = pad_to(max(cols, 1), 16)
    if out is None:
        buf = torch.empty(rows, ldq, dtype=torch.int8, device=dev)
        if ldq > cols:
            buf[:, cols:].zero_()
    else:
        buf = out
        if buf.dtype != torch.int8 or buf.shape[0] != rows or buf.stride(1) != 1:
            raise ValueError("out must be int8 [rows, >=cols] with unit column stride")
        ldq = buf.stride(0) if rows > 1 else ldq
    if scale is None:
        scale = torch.empty(rows, dtype=torch.float32, device=dev)
    fn = "lema_quantize_rows" if x.dtype == torch.bfloat16 else "lema_quantize_rows_f32"
    N.call(fn, _ptr(x), rows, cols, _ld(x), _ptr(buf), ldq, _ptr(scale), _stream(dev))
    return buf[:, :cols], scale


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel int8 quantisation of an nn.Linear weight [N, K].

    Returns (wq int8 [N, K] with row stride padded to 16, sw fp32 [N]).
    """
    if w.dtype not in (torch.bfloat16, torch.float32):
        w = w.to(torch.bfloat16)
    return quantize_rows(w)


# ---------------------------------------------------------------------------
# K2+K3: int8 GEMM with fused epilogue
# ---------------------------------------------------------------------------

def w8a8_gemm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
              bias: torch.Tensor | None = None, want_y: bool = True, want_acc: bool = False,
              out: torch.Tensor | None = None):
    """y[M,N] = bf16((acc * sx[m]) * sw[n] + bias[n]), acc = xq . wq^T (exact s32).

    Returns y, or (y, acc) when ``want_acc`` (y is None if not ``want_y``).
    """
    dev = _require_cuda(xq, sx, wq, sw, bias)
    if xq.dtype != torch.int8 or wq.dtype != torch.int8:
        raise TypeError("xq and wq must be int8")
    M, K = xq.shape
    Nn, K2 = wq.shape
    if K2 != K:
        raise ValueError(f"K mismatch: {K} vs {K2}")
    if xq.stride(1) != 1 or wq.stride(1) != 1:
        raise ValueError("xq and wq need unit column stride")
    sx = sx.contiguous().float()
    sw = sw.contiguous().float()
    if bias is not None:
        bias = bias.contiguous().to(torch.bfloat16)
    y = None
    if want_y:
        y = out if out is not None else torch.empty(M, Nn, dtype=torch.bfloat16, device=dev)
    acc = torch.empty(M, Nn, dtype=torch.int32, device=dev) if want_acc else None
    N.call("lema_w8a8_gemm", _ptr(xq), _ld(xq), _ptr(sx), _ptr(wq), _ld(wq), _ptr(sw),
           _ptr(bias), _ptr(y), Nn if y is None else _ld(y), _ptr(acc), Nn, M, Nn, K,
           _stream(dev))
    if want_acc:
        return y, acc
    return y


def w8a8_linear_forward(x2d: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                        bias: torch.Tensor | None = None) -> torch.Tensor:
    """K1 + K2/K3 on a bf16 [M, K] input: the forward of one W8A8 projection."""
    dev = _require_cuda(x2d, wq, sw, bias)
    x2d = _rows_view(x2d)
    if x2d.dtype != torch.bfloat16:
        raise TypeError("w8a8 forward takes bf16 activations")
    M, K = x2d.shape
    Nn = wq.shape[0]
    if wq.shape[1] != K:
        raise ValueError(f"weight in_features {wq.shape[1]} != input features {K}")
    ldq = pad_to(max(K, 1), 16)
    xq = torch.empty(M, ldq, dtype=torch.int8, device=dev)
    sx = torch.empty(M, dtype=torch.float32, device=dev)
    y = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev)
    if bias is not None:
        bias = bias.contiguous().to(torch.bfloat16)
    N.call("lema_w8a8_linear_fwd", _ptr(x2d), _ld(x2d), _ptr(wq), _ld(wq), _ptr(sw),
           _ptr(bias), _ptr(y), Nn, _ptr(xq), ldq, _ptr(sx), M, Nn, K, _stream(dev))
    return y


# ---------------------------------------------------------------------------
# K4: backward of the frozen base
# ---------------------------------------------------------------------------

def dequant_transpose(wq: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """wdT[K, ldt] bf16 with wdT[k, n] = bf16(float(wq[n, k]) * sw[n]); returns [K, N] view."""
    dev = _require_cuda(wq, sw)
    Nn, K = wq.shape
    ldt = pad_to(max(Nn, 1), 8)
    wdT = torch.empty(K, ldt, dtype=torch.bfloat16, device=dev)
    N.call("lema_dequant_transpose", _ptr(wq), _ld(wq), _ptr(sw.contiguous().float()), Nn, K,
           _ptr(wdT), ldt, _stream(dev))
    return wdT[:, :Nn]


def quantize_rows_colscaled(x: torch.Tensor, cs: torch.Tensor
                            ) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows of fp32(x[r, c]) * cs[c] (bf16 x, fp32 cs) quantised per row:
    (q int8 [R, C] view of an [R, ldq] buffer, scale fp32 [R])."""
    dev = _require_cuda(x, cs)
    x = _rows_view(x).to(torch.bfloat16)
    rows, cols = x.shape
    ldq = pad_to(max(cols, 1), 16)
    buf = torch.empty(rows, ldq, dtype=torch.int8, device=dev)
    if ldq > cols:
        buf[:, cols:].zero_()
    scale = torch.empty(rows, dtype=torch.float32, device=dev)
    N.call("lema_quantize_rows_colscaled", _ptr(x), _ptr(cs.contiguous().float()), rows, cols,
           _ld(x), _ptr(buf), ldq, _ptr(scale), _stream(dev))
    return buf[:, :cols], scale


def transpose_i8(wq: torch.Tensor) -> torch.Tensor:
    """wqT[K, N] = wq[N, K] for int8 (a view of a [K, round_up(N, 16)] buffer)."""
    dev = _require_cuda(wq)
    wq = _rows_view(wq)
    if wq.dtype != torch.int8:
        raise TypeError("transpose_i8 takes int8")
    Nn, K = wq.shape
    ldt = pad_to(max(Nn, 1), 16)
    out = torch.zeros(K, ldt, dtype=torch.int8, device=dev)
    N.call("lema_transpose_i8", _ptr(wq), _ld(wq), Nn, K, _ptr(out), ldt, _stream(dev))
    return out[:, :Nn]


def bf16_gemm_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """y = bf16(a . b^T) with fp32 accumulation (tcgen05 kind::f16)."""
    dev = _require_cuda(a, b)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("bf16 operands required")
    a = _rows_view(a)
    b = _rows_view(b)
    M, K = a.shape
    Nn = b.shape[0]
    y = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev)
    N.call("lema_bf16_gemm_tn", _ptr(a), _ld(a), _ptr(b), _ld(b), _ptr(y), Nn, M, Nn, K,
           _stream(dev))
    return y


# Straight-through dgrad of the frozen W8A8 projections: "bf16" (the contract:
# dy . bf16(wq * sw) with fp32 accumulation) or the opt-in "int8" variant
# (dy * sw quantised per row, int8 GEMM with wq^T; looser tolerance).
_DGRAD_MODE = "bf16"


def set_dgrad_mode(mode: str) -> None:
    global _DGRAD_MODE
    if mode not in ("bf16", "int8"):
        raise ValueError(f"dgrad mode must be 'bf16' or 'int8', not {mode!r}")
    _DGRAD_MODE = mode


def dgrad_mode() -> str:
    return _DGRAD_MODE


def w8a8_dgrad_int8(dy: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """dx[M, K] ~ dy[M, N] . (wq * sw): dy * sw quantised per row to int8, int8
    GEMM with the transposed int8 weight, dx = bf16(sd[m] * acc)."""
    dev = _require_cuda(dy, wq, sw)
    dy = _rows_view(dy).to(torch.bfloat16)
    M, Nn = dy.shape
    K = wq.shape[1]
    ld = pad_to(max(Nn, 1), 16)
    wqT = torch.empty(K, ld, dtype=torch.int8, device=dev)
    dq = torch.empty(M, ld, dtype=torch.int8, device=dev)
    if ld > Nn:
        wqT[:, Nn:].zero_()
        dq[:, Nn:].zero_()
    sd = torch.empty(M, dtype=torch.float32, device=dev)
    dx = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    N.call("lema_w8a8_dgrad_int8", _ptr(dy), _ld(dy), _ptr(wq), _ld(wq),
           _ptr(sw.contiguous().float()), _ptr(dx), K, _ptr(wqT), ld, _ptr(dq), ld, _ptr(sd),
           M, Nn, K, _stream(dev))
    return dx


def w8a8_dgrad(dy: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """dx[M, K] = bf16(dy[M, N] . wdeq[N, K]), wdeq = bf16(wq * sw) (straight-through);
    the int8 variant when ``set_dgrad_mode("int8")`` is in effect."""
    if _DGRAD_MODE == "int8":
        return w8a8_dgrad_int8(dy, wq, sw)
    dev = _require_cuda(dy, wq, sw)
    dy = _rows_view(dy)
    if dy.dtype != torch.bfloat16:
        dy = dy.to(torch.bfloat16)
    if (dy.stride(0) * 2) % 16 != 0 or dy.data_ptr() % 16 != 0:
        # TMA needs 16-byte row pitch: re-lay dy out with a padded pitch.
        M0, N0 = dy.shape
        buf = torch.zeros(M0, pad_to(N0, 8), dtype=torch.bfloat16, device=dev)
        buf[:, :N0] = dy
        dy = buf[:, :N0]
    M, Nn = dy.shape
    K = wq.shape[1]
    ldt = pad_to(max(Nn, 1), 8)
    ws = torch.empty(K, ldt, dtype=torch.bfloat16, device=dev)
    dx = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    N.call("lema_w8a8_dgrad", _ptr(dy), _ld(dy), _ptr(wq), _ld(wq), _ptr(sw.contiguous().float()),
           _ptr(dx), K, _ptr(ws), ldt, M, Nn, K, _stream(dev))
    return dx


# ---------------------------------------------------------------------------
# K6: grouped W8A8 GEMM (MoE experts)
# ---------------------------------------------------------------------------

def grouped_w8a8_gemm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                      offsets: list[int], bias: torch.Tensor | None = None) -> torch.Tensor:
    """Per-expert W8A8 GEMM. xq [T, K] rows sorted by expert, wq [E, N, K], sw [E, N],
    offsets: E+1 host ints (rows of expert e are offsets[e]:offsets[e+1])."""
    dev = _require_cuda(xq, sx, wq, sw, bias)
    E, Nn, K = wq.shape
    if len(offsets) != E + 1:
        raise ValueError("offsets must have E+1 entries")
    if wq.stride(2) != 1 or wq.stride(0) != Nn * wq.stride(1):
        raise ValueError("expert weights must be stacked contiguously: [E, N, ldw]")
    T = xq.shape[0]
    y = torch.empty(T, Nn, dtype=torch.bfloat16, device=dev)
    offs = (C.c_int64 * (E + 1))(*[int(o) for o in offsets])
    if bias is not None:
        bias = bias.contiguous().to(torch.bfloat16)
    args = ("lema_grouped_w8a8_gemm", _ptr(xq), _ld(xq), _ptr(sx.contiguous().float()),
            _ptr(wq), wq.stride(1), _ptr(sw.contiguous().float()), _ptr(bias), _ptr(y), Nn,
            offs, E, Nn, K, _stream(dev))
    N.call(*args)
    return y


# ---------------------------------------------------------------------------
# Differentiable linear
# ---------------------------------------------------------------------------

class _W8A8LinearFn(torch.autograd.Function):
    """y = W8A8(x); dx = dy . (wq * sw) (STE through both quantisers); no dW (frozen base)."""

    @staticmethod
    def forward(ctx, x2d, wq, sw, bias):
        y = w8a8_linear_forward(x2d, wq, sw, bias)
        ctx.save_for_backward(wq, sw)
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        wq, sw = ctx.saved_tensors
        dx = w8a8_dgrad(dy, wq, sw) if ctx.needs_input_grad[0] else None
        dbias = None
        if ctx.has_bias and ctx.needs_input_grad[3]:
            dbias = dy.float().sum(0).to(torch.bfloat16)
        return dx, None, None, dbias


class _W8A8TrainableFn(torch.autograd.Function):
    """W8A8 forward of a trainable projection (the int8 copy of its current true
    weight); backward: straight-through dx and the fp32 weight gradient
    dW = dy^T . x, added into ``sink.wgrad_acc``."""

    @staticmethod
    def forward(ctx, x2d, wq, sw, sink):
        y = w8a8_linear_forward(x2d, wq, sw, None)
        ctx.save_for_backward(x2d, wq, sw)
        ctx.sink = sink
        return y

    @staticmethod
    def backward(ctx, dy):
        x2d, wq, sw = ctx.saved_tensors
        dx = w8a8_dgrad(dy, wq, sw) if ctx.needs_input_grad[0] else None
        ctx.sink.wgrad_acc.add_(w8a8_wgrad(dy, x2d))
        return dx, None, None, None


def w8a8_linear_trainable(x: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, sink) -> torch.Tensor:
    K = x.shape[-1]
    lead = x.shape[:-1]
    x2d = x.reshape(-1, K)
    if x2d.dtype != torch.bfloat16:
        x2d = x2d.to(torch.bfloat16)
    return _W8A8TrainableFn.apply(x2d, wq, sw, sink).reshape(*lead, wq.shape[0])


def w8a8_linear(x: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                bias: torch.Tensor | None = None) -> torch.Tensor:
    """Functional W8A8 linear over [..., K] -> [..., N] (bf16 compute, input dtype out)."""
    K = x.shape[-1]
    lead = x.shape[:-1]
    in_dtype = x.dtype
    x2d = x.reshape(-1, K)
    if x2d.dtype != torch.bfloat16:
        x2d = x2d.to(torch.bfloat16)
    y = _W8A8LinearFn.apply(x2d, wq, sw, bias)
    y = y.reshape(*lead, wq.shape[0])
    if in_dtype != torch.bfloat16 and in_dtype.is_floating_point:
        y = y.to(in_dtype)
    return y


def _offsets_array(offsets) -> tuple[C.Array, int]:
    offs = [int(o) for o in offsets]
    return (C.c_int64 * len(offs))(*offs), len(offs) - 1


def grouped_w8a8_dgrad(dy: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                       offsets: list[int]) -> torch.Tensor:
    """Per-expert straight-through dgrad: rows of expert e get dy . bf16(wq[e] * sw[e]).
    dy [T, N] bf16 sorted by expert, wq [E, N, K] int8, sw [E, N]. The int8-dy
    variant when ``set_dgrad_mode("int8")`` is in effect."""
    if _DGRAD_MODE == "int8":
        return grouped_w8a8_dgrad_int8(dy, wq, sw, offsets)
    dev = _require_cuda(dy, wq, sw)
    dy = _rows_view(dy.to(torch.bfloat16))
    E, Nn, K = wq.shape
    if wq.stride(2) != 1 or wq.stride(0) != Nn * wq.stride(1):
        raise ValueError("expert weights must be stacked contiguously: [E, N, ldw]")
    offs, E2 = _offsets_array(offsets)
    if E2 != E:
        raise ValueError("offsets must have E+1 entries")
    ldt = pad_to(max(Nn, 1), 8)
    ws = torch.empty(E, K, ldt, dtype=torch.bfloat16, device=dev)
    T = dy.shape[0]
    dx = torch.empty(T, K, dtype=torch.bfloat16, device=dev)
    N.call("lema_grouped_w8a8_dgrad", _ptr(dy), _ld(dy), _ptr(wq), wq.stride(1),
           _ptr(sw.contiguous().float()), _ptr(dx), K, _ptr(ws), ldt, offs, E, Nn, K,
           _stream(dev))
    return dx


def grouped_w8a8_dgrad_int8(dy: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                            offsets: list[int]) -> torch.Tensor:
    """Per-expert int8-dy dgrad: the rows of expert e, dy * sw[e], quantised per
    row (column-scaled quantiser), wq[e] transposed in int8, then one grouped int8
    GEMM with unit column scales: dx ~ dy . (wq[e] * sw[e]). Experts without rows
    are skipped."""
    dev = _require_cuda(dy, wq, sw)
    dy = _rows_view(dy.to(torch.bfloat16))
    E, Nn, K = wq.shape
    if wq.stride(2) != 1 or wq.stride(0) != Nn * wq.stride(1):
        raise ValueError("expert weights must be stacked contiguously: [E, N, ldw]")
    offs, E2 = _offsets_array(offsets)
    if E2 != E:
        raise ValueError("offsets must have E+1 entries")
    bounds = [int(o) for o in offsets]
    T = dy.shape[0]
    ld = pad_to(max(Nn, 1), 16)
    dq = torch.empty(T, ld, dtype=torch.int8, device=dev)
    wqT = torch.empty(E, K, ld, dtype=torch.int8, device=dev)
    if ld > Nn:
        dq[:, Nn:].zero_()
        wqT[:, :, Nn:].zero_()
    sd = torch.empty(T, dtype=torch.float32, device=dev)
    swc = sw.contiguous().float()
    stream = _stream(dev)
    lddy = _ld(dy)
    for e in range(E):
        r0, r1 = bounds[e], bounds[e + 1]
        if r1 <= r0:
            continue
        N.call("lema_quantize_rows_colscaled", dy.data_ptr() + r0 * lddy * 2,
               swc[e].data_ptr(), r1 - r0, Nn, lddy, dq.data_ptr() + r0 * ld, ld,
               sd.data_ptr() + r0 * 4, stream)
        N.call("lema_transpose_i8", wq[e].data_ptr(), wq.stride(1), Nn, K, wqT[e].data_ptr(), ld,
               stream)
    dx = torch.empty(T, K, dtype=torch.bfloat16, device=dev)
    N.call("lema_grouped_w8a8_gemm", _ptr(dq), ld, _ptr(sd), _ptr(wqT), ld, None, None,
           _ptr(dx), K, offs, E, K, Nn, stream)
    return dx


def grouped_bf16_gemm_tn(a: torch.Tensor, b: torch.Tensor, offsets: list[int]) -> torch.Tensor:
    """Rows [offsets[e], offsets[e+1]) of a times b[e]^T; a [T, K], b [E, N, K] bf16."""
    dev = _require_cuda(a, b)
    a = _rows_view(a)
    E, Nn, K = b.shape
    offs, E2 = _offsets_array(offsets)
    if E2 != E:
        raise ValueError("offsets must have E+1 entries")
    y = torch.empty(a.shape[0], Nn, dtype=torch.bfloat16, device=dev)
    N.call("lema_grouped_bf16_gemm_tn", _ptr(a), _ld(a), _ptr(b), b.stride(1), _ptr(y), Nn,
           offs, E, Nn, K, _stream(dev))
    return y


def bf16_gemm_tn_f32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 y = a . b^T (bf16 operands, fp32 accumulators returned as is)."""
    dev = _require_cuda(a, b)
    a = _rows_view(a.to(torch.bfloat16))
    b = _rows_view(b.to(torch.bfloat16))
    M, K = a.shape
    Nn = b.shape[0]
    y = torch.empty(M, Nn, dtype=torch.float32, device=dev)
    N.call("lema_bf16_gemm_tn_f32", _ptr(a), _ld(a), _ptr(b), _ld(b), _ptr(y), Nn, M, Nn, K,
           _stream(dev))
    return y


def w8a8_wgrad(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Straight-through weight gradient of a W8A8 projection: dW[N, K] = dy^T . x
    (bf16 inputs, fp32 accumulation) for dy [M, N], x [M, K]."""
    dyt = dy.to(torch.bfloat16).t().contiguous()
    xt = x.to(torch.bfloat16).t().contiguous()
    K = xt.shape[0]
    if (dyt.shape[1] * 2) % 16 != 0:  # TMA row pitch: pad the token dimension
        M8 = pad_to(dyt.shape[1], 8)
        dyt = torch.nn.functional.pad(dyt, (0, M8 - dyt.shape[1]))
        xt = torch.nn.functional.pad(xt, (0, M8 - xt.shape[1]))
    return bf16_gemm_tn_f32(dyt, xt) if K else torch.zeros(dyt.shape[0], 0, device=dy.device)


# ---------------------------------------------------------------------------
# Fused producers of the decoder block (RMSNorm -> quantise, RoPE, SwiGLU ->
# quantise) and the autograd functions of the fused block path
# ---------------------------------------------------------------------------

def rmsnorm_quant(x2d: torch.Tensor, g: torch.Tensor, eps: float, want_q: bool = True):
    """(hn bf16 [M, H], xq int8 [M, H] | None, sx fp32 [M] | None, rstd fp32 [M])."""
    dev = _require_cuda(x2d, g)
    x2d = _rows_view(x2d)
    M, H = x2d.shape
    hn = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    rstd = torch.empty(M, dtype=torch.float32, device=dev)
    xq = sx = None
    if want_q:
        xq = torch.empty(M, pad_to(H, 16), dtype=torch.int8, device=dev)[:, :H]
        sx = torch.empty(M, dtype=torch.float32, device=dev)
    N.call("lema_rmsnorm_quant", _ptr(x2d), _ld(x2d), _ptr(g.contiguous()), M, H, float(eps),
           _ptr(hn), H, _ptr(xq), (xq.stride(0) if xq is not None else 0), _ptr(sx), _ptr(rstd),
           _stream(dev))
    return hn, xq, sx, rstd


def rmsnorm_bwd(x2d, g, rstd, dhn):
    dev = _require_cuda(x2d, g, rstd, dhn)
    x2d, dhn = _rows_view(x2d), _rows_view(dhn.to(torch.bfloat16))
    M, H = x2d.shape
    dx = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    N.call("lema_rmsnorm_bwd", _ptr(x2d), _ld(x2d), _ptr(g.contiguous()), _ptr(rstd), _ptr(dhn),
           _ld(dhn), M, H, _ptr(dx), H, _stream(dev))
    return dx


def rope(q2d, k2d, cos, sin, seq: int, hq: int, hk: int, d: int, mode: int = 0):
    """Rotary embedding of q [T, hq*d] and k [T, hk*d] rows (may be strided);
    cos/sin [seq, d] bf16. Returns contiguous (q_out, k_out)."""
    dev = _require_cuda(q2d, k2d, cos, sin)
    T = q2d.shape[0]
    qo = torch.empty(T, hq * d, dtype=torch.bfloat16, device=dev)
    ko = torch.empty(T, hk * d, dtype=torch.bfloat16, device=dev)
    N.call("lema_rope", _ptr(q2d), q2d.stride(0), _ptr(k2d), k2d.stride(0),
           _ptr(cos.contiguous()), _ptr(sin.contiguous()), T, seq, hq, hk, d, _ptr(qo), _ptr(ko),
           mode, _stream(dev))
    return qo, ko


def swiglu_quant(gu: torch.Tensor, want_m: bool = False):
    """Rows of [gate | up] -> (mq int8 [M, I], sm fp32 [M], m bf16 [M, I] | None)."""
    dev = _require_cuda(gu)
    M, I2 = gu.shape
    I = I2 // 2
    mq = torch.empty(M, pad_to(I, 16), dtype=torch.int8, device=dev)[:, :I]
    sm = torch.empty(M, dtype=torch.float32, device=dev)
    m = torch.empty(M, I, dtype=torch.bfloat16, device=dev) if want_m else None
    N.call("lema_swiglu_quant", _ptr(gu), gu.stride(0), M, I, _ptr(mq), mq.stride(0), _ptr(sm),
           _ptr(m), I, _stream(dev))
    return mq, sm, m


# ---------------------------------------------------------------------------
# Selective full fine-tuning: fused AdamW step + re-quantisation
# ---------------------------------------------------------------------------

def adamw_coefficients(step: int, lr: float, wd: float, beta1: float = 0.9,
                       beta2: float = 0.999, eps: float = 1e-8) -> tuple[float, ...]:
    """The fp32 scalars of one AdamW step as the reference forms them
    (src/lema/_full_ft.py:204-229; Python doubles rounded once to fp32):
    (decay, beta1, c1, beta2, c2, sqrt_bc2, step_size, eps)."""
    import numpy as np
    b1 = 1 - beta1 ** step
    b2 = 1 - beta2 ** step
    f = np.float32
    decay = f(1 - lr * wd) if wd else f(1.0)
    return tuple(float(x) for x in (decay, f(beta1), f(1 - beta1), f(beta2), f(1 - beta2),
                                    f(math.sqrt(b2)), f(-(lr / b1)), f(eps)))


def adamw_requant_rows(w: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
                       step: int, lr: float, wd: float, zero_grad: bool = True
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """One AdamW step of a [N, K] weight in place (w bf16, g / m / v fp32 on the
    device; g cleared when ``zero_grad``) fused with the per-output-channel int8
    quantisation of the new weight: returns (wq [N, K] view of [N, round_up(K, 16)],
    sw [N])."""
    dev = _require_cuda(w, g, m, v)
    if w.dtype != torch.bfloat16 or g.dtype != torch.float32 or m.dtype != torch.float32 \
            or v.dtype != torch.float32:
        raise TypeError("adamw_requant_rows takes bf16 w and fp32 g, m, v")
    for t in (w, g, m, v):
        if t.dim() != 2 or t.stride(1) != 1:
            raise ValueError("2-D tensors with unit column stride required")
    if m.stride(0) != v.stride(0) or not (w.shape == g.shape == m.shape == v.shape):
        raise ValueError("w, g, m, v must have one shape (m and v one row stride)")
    rows, cols = w.shape
    ldq = pad_to(max(cols, 1), 16)
    q = torch.empty(rows, ldq, dtype=torch.int8, device=dev)
    if ldq > cols:
        q[:, cols:].zero_()
    sw = torch.empty(rows, dtype=torch.float32, device=dev)
    N.call("lema_adamw_requant_rows", _ptr(w), _ld(w), _ptr(g), _ld(g), _ptr(m), _ptr(v),
           _ld(m), rows, cols, *adamw_coefficients(step, lr, wd), int(zero_grad), _ptr(q), ldq,
           _ptr(sw), _stream(dev))
    return q[:, :cols], sw


def swiglu_bwd(gu: torch.Tensor, dm: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(gu, dm)
    dm = _rows_view(dm.to(torch.bfloat16))
    M, I2 = gu.shape
    dgu = torch.empty(M, I2, dtype=torch.bfloat16, device=dev)
    N.call("lema_swiglu_bwd", _ptr(gu), gu.stride(0), _ptr(dm), _ld(dm), M, I2 // 2, _ptr(dgu),
           I2, _stream(dev))
    return dgu


def gemm_from_quant(xq, sx, wq, sw) -> torch.Tensor:
    """bf16 y = W8A8 GEMM of already-quantised rows (xq, sx) with (wq, sw)."""
    dev = _require_cuda(xq, wq)
    M, K = xq.shape
    Nn = wq.shape[0]
    y = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev)
    N.call("lema_w8a8_gemm", _ptr(xq), _ld(xq), _ptr(sx), _ptr(wq), _ld(wq), _ptr(sw), None,
           _ptr(y), Nn, None, Nn, M, Nn, K, _stream(dev))
    return y


class RMSNormQuantFn(torch.autograd.Function):
    """hn = RMSNorm(x) (bf16 rounding of HF LlamaRMSNorm) plus its int8 rows."""

    @staticmethod
    def forward(ctx, x2d, g, eps):
        hn, xq, sx, rstd = rmsnorm_quant(x2d, g, eps)
        ctx.save_for_backward(x2d, g, rstd)
        ctx.mark_non_differentiable(xq, sx)
        return hn, xq, sx

    @staticmethod
    def backward(ctx, dhn, _dxq, _dsx):
        x2d, g, rstd = ctx.saved_tensors
        return rmsnorm_bwd(x2d, g, rstd, dhn), None, None


class QKVFn(torch.autograd.Function):
    """Stacked q/k/v W8A8 projection of pre-quantised rows; returns (q, k, v) views.
    Backward: one straight-through dgrad over the concatenated gradients."""

    @staticmethod
    def forward(ctx, hn, xq, sx, wq, sw, nq, nk):
        y = gemm_from_quant(xq, sx, wq, sw)
        ctx.save_for_backward(wq, sw)
        ctx.split = (nq, nk)
        return y[:, :nq], y[:, nq:nq + nk], y[:, nq + nk:]

    @staticmethod
    def backward(ctx, dq, dk, dv):
        wq, sw = ctx.saved_tensors
        nq, nk = ctx.split
        rows = next(g for g in (dq, dk, dv) if g is not None).shape[0]
        parts = []
        for g, n in ((dq, nq), (dk, nk), (dv, wq.shape[0] - nq - nk)):
            parts.append(g if g is not None else
                         torch.zeros(rows, n, dtype=torch.bfloat16, device=wq.device))
        dy = torch.cat([p.to(torch.bfloat16) for p in parts], dim=1)
        return w8a8_dgrad(dy, wq, sw), None, None, None, None, None, None


class RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q2d, k2d, cos, sin, seq, hq, hk, d):
        ctx.save_for_backward(cos, sin)
        ctx.meta = (seq, hq, hk, d)
        return rope(q2d, k2d, cos, sin, seq, hq, hk, d, 0)

    @staticmethod
    def backward(ctx, dq, dk):
        cos, sin = ctx.saved_tensors
        seq, hq, hk, d = ctx.meta
        dqi, dki = rope(dq.contiguous().to(torch.bfloat16), dk.contiguous().to(torch.bfloat16),
                        cos, sin, seq, hq, hk, d, 1)
        return dqi, dki, None, None, None, None, None, None


class MLPFn(torch.autograd.Function):
    """down(silu(gate) * up) with stacked [gate; up] W8A8 weights: gate_up GEMM on the
    pre-quantised RMSNorm rows, fused SwiGLU -> quantise, down GEMM. Backward:
    straight-through dgrads around the SwiGLU backward kernel."""

    @staticmethod
    def forward(ctx, hn, xq, sx, wq_gu, sw_gu, wq_dn, sw_dn):
        gu = gemm_from_quant(xq, sx, wq_gu, sw_gu)
        mq, sm, _ = swiglu_quant(gu)
        y = gemm_from_quant(mq, sm, wq_dn, sw_dn)
        ctx.save_for_backward(gu, wq_gu, sw_gu, wq_dn, sw_dn)
        return y

    @staticmethod
    def backward(ctx, dy):
        gu, wq_gu, sw_gu, wq_dn, sw_dn = ctx.saved_tensors
        dm = w8a8_dgrad(dy, wq_dn, sw_dn)
        dgu = swiglu_bwd(gu, dm)
        return w8a8_dgrad(dgu, wq_gu, sw_gu), None, None, None, None, None, None


def rope_qkv(q2d, k2d, v2d, q_add, k_add, v_add, cos, sin, seq, hq, hk, d):
    """Forward RoPE of q and k plus the contiguous copy of v, each after adding its
    optional LoRA output (bf16 rounding). Returns contiguous (q_out, k_out, v_out)."""
    dev = _require_cuda(q2d, k2d, v2d, cos, sin)
    T = q2d.shape[0]
    qo = torch.empty(T, hq * d, dtype=torch.bfloat16, device=dev)
    ko = torch.empty(T, hk * d, dtype=torch.bfloat16, device=dev)
    vo = torch.empty(T, hk * d, dtype=torch.bfloat16, device=dev)
    adds = [None if t is None else t.contiguous().to(torch.bfloat16) for t in (q_add, k_add, v_add)]
    N.call("lema_rope_qkv", _ptr(q2d), q2d.stride(0), _ptr(k2d), k2d.stride(0), _ptr(v2d),
           v2d.stride(0), _ptr(adds[0]), _ptr(adds[1]), _ptr(adds[2]), _ptr(cos.contiguous()),
           _ptr(sin.contiguous()), T, seq, hq, hk, d, _ptr(qo), _ptr(ko), _ptr(vo), 0,
           _stream(dev))
    return qo, ko, vo


class RopeQKVFn(torch.autograd.Function):
    """(q + lq, k + lk) rotated and v + lv made contiguous in one kernel."""

    @staticmethod
    def forward(ctx, q, k, v, lq, lk, lv, cos, sin, seq, hq, hk, d):
        ctx.save_for_backward(cos, sin)
        ctx.meta = (seq, hq, hk, d)
        ctx.has_add = (lq is not None, lk is not None, lv is not None)
        return rope_qkv(q, k, v, lq, lk, lv, cos, sin, seq, hq, hk, d)

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin = ctx.saved_tensors
        seq, hq, hk, d = ctx.meta
        dqi, dki = rope(dq.contiguous().to(torch.bfloat16), dk.contiguous().to(torch.bfloat16),
                        cos, sin, seq, hq, hk, d, 1)
        dv = dv.contiguous()
        hq_, hk_, hv_ = ctx.has_add
        return (dqi, dki, dv, dqi if hq_ else None, dki if hk_ else None, dv if hv_ else None,
                None, None, None, None, None, None)


def attention_fwd(q2d: torch.Tensor, k2d: torch.Tensor, v2d: torch.Tensor, B: int, S: int,
                  H: int, Hkv: int, scale: float):
    """Causal attention on the tcgen05 kernel: q2d [B*S, H*128], k2d / v2d
    [B*S, Hkv*128] token-major bf16 -> (o [B*S, H*128] bf16, lse [B, H, S] fp32
    log2-domain log-sum-exp of the scaled scores)."""
    dev = _require_cuda(q2d, k2d, v2d)
    q2d, k2d, v2d = (_rows_view(t) for t in (q2d, k2d, v2d))
    o = torch.empty(B * S, H * 128, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, H, S, dtype=torch.float32, device=dev)
    N.call("lema_attn_fwd", _ptr(q2d), _ld(q2d), _ptr(k2d), _ld(k2d), _ptr(v2d), _ld(v2d),
           _ptr(o), H * 128, _ptr(lse), B, S, H, Hkv, 128, float(scale), _stream(dev))
    return o, lse


def attention_bwd(q2d, k2d, v2d, o2d, lse, dout2d, B: int, S: int, H: int, Hkv: int,
                  scale: float, split_heads: bool = True):
    """(dq [B*S, H*128], dk, dv [B*S, Hkv*128]) of attention_fwd. With GQA the
    library may split dK / dV per query head through a workspace (when the kv
    heads alone would leave SMs idle); ``split_heads=False`` withholds it."""
    dev = _require_cuda(q2d, k2d, v2d, o2d, lse, dout2d)
    q2d, k2d, v2d, o2d = (_rows_view(t) for t in (q2d, k2d, v2d, o2d))
    dout2d = _rows_view(dout2d.to(torch.bfloat16))
    dq = torch.empty(B * S, H * 128, dtype=torch.bfloat16, device=dev)
    dk = torch.empty(B * S, Hkv * 128, dtype=torch.bfloat16, device=dev)
    dv = torch.empty(B * S, Hkv * 128, dtype=torch.bfloat16, device=dev)
    delta = torch.empty(B, H, S, dtype=torch.float32, device=dev)
    ws = (torch.empty(2 * B * S * H * 128, dtype=torch.float32, device=dev)
          if H != Hkv and split_heads else None)
    N.call("lema_attn_bwd", _ptr(q2d), _ld(q2d), _ptr(k2d), _ld(k2d), _ptr(v2d), _ld(v2d),
           _ptr(o2d), _ld(o2d), _ptr(dout2d), _ld(dout2d), _ptr(lse.contiguous()), _ptr(delta),
           _ptr(ws), _ptr(dq), H * 128, _ptr(dk), Hkv * 128, _ptr(dv), Hkv * 128, B, S, H, Hkv,
           128, float(scale), _stream(dev))
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    if ws is not None and B * Hkv * -(-S // 128) < n_sm:
        N.kernel_launches += 1  # the library split dK/dV per query head: the reduce kernel
    return dq, dk, dv


class AttentionFn(torch.autograd.Function):
    """Causal attention (head_dim 128, GQA) on the tcgen05 kernels over the
    token-major q [B*S, H*128], k / v [B*S, Hkv*128]; returns o [B*S, H*128]."""

    @staticmethod
    def forward(ctx, q2d, k2d, v2d, B, S, H, Hkv, scale):
        o, lse = attention_fwd(q2d, k2d, v2d, B, S, H, Hkv, scale)
        ctx.save_for_backward(q2d, k2d, v2d, o, lse)
        ctx.meta = (B, S, H, Hkv, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q2d, k2d, v2d, o, lse = ctx.saved_tensors
        dq, dk, dv = attention_bwd(q2d, k2d, v2d, o, lse, do, *ctx.meta)
        return dq, dk, dv, None, None, None, None, None
