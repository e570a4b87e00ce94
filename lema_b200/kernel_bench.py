"""Micro-benchmarks of single kernels on one GPU (CUDA events, median of the
repetitions), printing one JSON line per case.

    python -m lema_b200.kernel_bench attention [small | long]
        the tcgen05 causal attention (ops.attention_fwd / attention_bwd) beside
        torch SDPA at the training shapes; ``small`` runs B 2, S 512, H 8 and
        ``long`` B 1, S 4096, H 16, Hkv 4 only (the shapes the attention ncu
        captures use: latency, and throughput)
    python -m lema_b200.kernel_bench producers
        K1 (quantize_rows), RMSNorm -> quantise and SwiGLU -> quantise at
        M = 4096 tokens, each beside a device copy moving the same bytes; the L2
        is flushed (a 512 MB write) before every timed launch
    python -m lema_b200.kernel_bench misc [once]
        the remaining kernels of the path: the fused AdamW + re-quantisation of
        a 4096 x 4096 projection, the SM checkpoint-store kernel (32 MB into
        pinned host memory) beside the copy engine, the generic quantisers on
        unaligned rows (4096 x 4100), the device-error snapshot; ``once``
        launches each (plus a GQA attention backward for its delta and dK/dV
        reduce kernels) a single time, untimed, for an ncu capture
"""
from __future__ import annotations

import json
import statistics
import sys

import torch
import torch.nn.functional as F

from . import _native, ops

D = 128


def _time_us(fn, reps: int = 7, flush: torch.Tensor | None = None) -> float:
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    return statistics.median(ts)


def attention(which: str) -> None:
    dev = torch.device("cuda:0")
    shapes = {"small": [(2, 512, 8, 8)], "long": [(1, 4096, 16, 4)]}.get(
        which, [(8, 512, 32, 32), (8, 512, 32, 8), (1, 2048, 32, 32), (2, 4096, 32, 8)])
    for B, S, H, Hkv in shapes:
        q = torch.randn(B * S, H * D, device=dev).to(torch.bfloat16)
        k = torch.randn(B * S, Hkv * D, device=dev).to(torch.bfloat16)
        v = torch.randn(B * S, Hkv * D, device=dev).to(torch.bfloat16)
        do = torch.randn(B * S, H * D, device=dev).to(torch.bfloat16)
        o, lse = ops.attention_fwd(q, k, v, B, S, H, Hkv, D ** -0.5)
        fwd = _time_us(lambda: ops.attention_fwd(q, k, v, B, S, H, Hkv, D ** -0.5))
        bwd = _time_us(lambda: ops.attention_bwd(q, k, v, o, lse, do, B, S, H, Hkv, D ** -0.5))
        qh = q.view(B, S, H, D).transpose(1, 2)
        kh = k.view(B, S, Hkv, D).transpose(1, 2)
        vh = v.view(B, S, Hkv, D).transpose(1, 2)

        def sdpa():
            return F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=D ** -0.5,
                                                  enable_gqa=H != Hkv)
        sfwd = _time_us(sdpa)
        qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (qh, kh, vh))
        og = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True, scale=D ** -0.5,
                                            enable_gqa=H != Hkv)
        g = torch.randn_like(og)
        sbwd = _time_us(lambda: torch.autograd.grad(og, (qg, kg, vg), g, retain_graph=True))
        flops = 2 * B * H * S * S * D  # causal forward: half of two S x S x D GEMMs
        print(json.dumps({"case": f"attention B{B} S{S} H{H} Hkv{Hkv}",
                          "fwd_us": round(fwd, 1), "fwd_tflops": round(flops / fwd / 1e6, 1),
                          "bwd_us": round(bwd, 1),
                          "bwd_tflops": round(2.5 * flops / bwd / 1e6, 1),
                          "sdpa_fwd_us": round(sfwd, 1), "sdpa_bwd_us": round(sbwd, 1)}),
              flush=True)


def producers() -> None:
    dev = torch.device("cuda:0")
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)

    def copy_gbs(nbytes: int) -> float:
        src = torch.empty(nbytes // 2, dtype=torch.uint8, device=dev)
        dst = torch.empty_like(src)
        return round(nbytes / _time_us(lambda: dst.copy_(src), 9, flush) / 1e3, 1)

    def report(case: str, us: float, nbytes: int) -> None:
        print(json.dumps({"case": case, "us": round(us, 2),
                          "GBps": round(nbytes / us / 1e3, 1), "bytes": nbytes,
                          "copy_same_bytes_GBps": copy_gbs(nbytes)}), flush=True)

    M = 4096
    x = torch.randn(M, 4096, device=dev).to(torch.bfloat16)
    xq = torch.empty(M, 4096, dtype=torch.int8, device=dev)
    sx = torch.empty(M, device=dev)
    report("quantize_rows 4096 x 4096",
           _time_us(lambda: ops.quantize_rows(x, out=xq, scale=sx), 9, flush), M * 4096 * 3 + M * 4)
    w = (1 + 0.1 * torch.randn(4096, device=dev)).to(torch.bfloat16)
    report("rmsnorm_quant 4096 x 4096", _time_us(lambda: ops.rmsnorm_quant(x, w, 1e-5), 9, flush),
           M * 4096 * 5 + M * 8)
    for inter in (11008, 14336):
        gu = torch.randn(M, 2 * inter, device=dev).to(torch.bfloat16)
        report(f"swiglu_quant 4096 x {inter}",
               _time_us(lambda: ops.swiglu_quant(gu, want_m=False), 9, flush),
               M * inter * 5 + M * 4)
        del gu


def misc(once: bool) -> None:
    dev = torch.device("cuda:0")
    flush = None if once else torch.empty(512 << 20, dtype=torch.uint8, device=dev)

    def run(fn) -> float:
        if once:
            fn()
            torch.cuda.synchronize()
            return float("nan")
        return _time_us(fn, 9, flush)

    def report(case: str, us: float, nbytes: int, copy: bool = True) -> None:
        if once:
            return
        line = {"case": case, "us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
                "bytes": nbytes}
        if copy:
            src = torch.empty(nbytes // 2, dtype=torch.uint8, device=dev)
            dst = torch.empty_like(src)
            line["copy_same_bytes_GBps"] = round(nbytes / _time_us(lambda: dst.copy_(src), 9,
                                                                   flush) / 1e3, 1)
        print(json.dumps(line), flush=True)

    # fused AdamW + per-channel re-quantisation of a 4096 x 4096 projection
    # (29 bytes per element: w, g, m, v in; w, m, v, the zeroed g and int8 out)
    n = k = 4096
    w = (0.02 * torch.randn(n, k, device=dev)).to(torch.bfloat16)
    g = 1e-3 * torch.randn(n, k, device=dev)
    m = torch.zeros_like(g)
    v = torch.zeros_like(g)
    report("adamw_requant_rows 4096 x 4096",
           run(lambda: ops.adamw_requant_rows(w, g, m, v, 1, 1e-5, 0.01)), n * k * 29 + n * 4)
    del w, g, m, v
    # boundary-activation checkpoint (bf16 [4096, 4096]) into pinned host memory:
    # mode 1 is the SM store kernel, mode 0 the copy engine
    x = torch.randn(4096, 4096, device=dev).to(torch.bfloat16)
    host = torch.empty(x.numel() * 2, dtype=torch.uint8, pin_memory=True)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for mode, name in ((1, "ckpt_store_kernel (SM stores)"), (0, "copy engine")):
        report(f"ckpt_save 32 MB, {name}",
               run(lambda: _native.call("lema_ckpt_save", x.data_ptr(), host.data_ptr(),
                                        x.numel() * 2, mode, stream, None, None)),
               x.numel() * 2, copy=False)
    # generic quantisers: rows that are not a whole number of 16-byte vectors
    xo = torch.randn(4096, 4100, device=dev).to(torch.bfloat16)
    report("quantize_rows (generic) 4096 x 4100", run(lambda: ops.quantize_rows(xo)),
           4096 * 4100 * 3 + 4096 * 4)
    cs = 1 + 0.1 * torch.rand(4100, device=dev)
    report("quantize_rows_colscaled (generic) 4096 x 4100",
           run(lambda: ops.quantize_rows_colscaled(xo, cs)), 4096 * 4100 * 3 + 4096 * 4)
    # the per-step device-error snapshot (one thread; latency only)
    word = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    report("error_snapshot_kernel", run(lambda: _native.call(
        "lema_device_error_async", word.data_ptr(), stream)), 4, copy=False)
    if once:  # GQA backward whose dK/dV CTAs split per query head: delta + reduce kernels
        B, S, H, Hkv = 1, 1024, 16, 4
        q = torch.randn(B * S, H * D, device=dev).to(torch.bfloat16)
        kk = torch.randn(B * S, Hkv * D, device=dev).to(torch.bfloat16)
        vv = torch.randn(B * S, Hkv * D, device=dev).to(torch.bfloat16)
        o, lse = ops.attention_fwd(q, kk, vv, B, S, H, Hkv, D ** -0.5)
        ops.attention_bwd(q, kk, vv, o, lse, torch.randn_like(q), B, S, H, Hkv, D ** -0.5)
        torch.cuda.synchronize()


def main(argv: list[str]) -> None:
    if not argv or argv[0] not in ("attention", "producers", "misc"):
        raise SystemExit("usage: python -m lema_b200.kernel_bench "
                         "{attention [small | long] | producers | misc [once]}")
    if argv[0] == "attention":
        attention(argv[1] if len(argv) > 1 else "")
    elif argv[0] == "producers":
        producers()
    else:
        misc(len(argv) > 1 and argv[1] == "once")
    if _native.device_error() != 0:
        raise SystemExit("a kernel recorded a device error")


if __name__ == "__main__":
    main(sys.argv[1:])
