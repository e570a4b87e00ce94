"""Benchmark of the W8A8 hot path on B200 (one JSON line on stdout).

Workloads (``--workload``):
  llama7b_streamed_lora (default)
                    one LoRA training step of the 32-layer Llama-2-7B-shaped
                    model (random init, vocab 32000, all seven projections
                    W8A8, LoRA r16 alpha 32 on q/v) on bs=8 x seq=512 tokens
                    per GPU: int8 weight segments streamed from pinned host
                    RAM per layer, boundary activations offloaded to pinned
                    host and restored for the recompute, data-parallel LoRA
                    gradient all-reduce (NCCL) for N > 1. Metric: tokens/s.
  llama7b_selective_ft_2048
                    the long-sequence case: bs 1 x seq 2048, 512-token chunked
                    attention, activations offloaded, selective full
                    fine-tuning of q/k/v/o in the last 4 layers (fp32 AdamW
                    states in pinned host RAM). Metric: tokens/s.
  mixtral_streamed_lora
                    one LoRA training step of a 32-layer Mixtral-8x7B-shaped
                    MoE model (GQA 32 q / 8 kv heads, 8 experts x SwiGLU
                    14336, top-2 softmax routing; W8A8 attention projections
                    and grouped W8A8 experts, 1.45 GB per layer) on bs=8 x
                    seq=512 per GPU, streamed from pinned host RAM as above.
                    Metric: tokens/s. Needs ~47 GB of pinned host RAM per rank.
  w8a8_linear_4096  one W8A8 linear forward step (K1 quantise + K2/K3 GEMM with
                    fused epilogue) at M=N=K=4096, the per-layer shape of the
                    7B streamed model at bs=8 x seq=512. Metric: int8 TOPS.

Contract: ``python bench.py --gpus N --steps K --warmup W`` (N>1 under torchrun,
one rank per GPU, replicas: each rank runs the same step on its own data, no
collective on the data path). W warm-up steps, then K timed steps bracketed by
barrier + synchronize; the device time is the max over ranks. ``--impl
reference`` times the CPU restatement of the path (the reference has no W8A8
implementation to run, and its Python package is not installed on the GPU
host) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "W8A8 GEMM TOPS (% INT8 peak); 7B streamed LoRA tokens/s at 1/2/4/8 B200"
INT8_SPEC_TOPS = 4500.0
# DRAM bytes per GEMM launch measured with ncu (dram__bytes_read.sum + dram__bytes_write.sum)
LINEAR_GEMM_TRAFFIC_BYTES = 33_630_464 + 668_672      # M=N=K=4096, CTA-pair kernel
TRAIN_GEMM_TRAFFIC_BYTES = 136_200_000                # mean of qkv / o / gate_up / down
L2_BYTES = 126 * 2**20


def read_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {}


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        def pump():
            for line in self.proc.stdout:
                self.rows.append([c.strip() for c in line.split(",")])
        self.thread = threading.Thread(target=pump, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_over_ranks(x: float, world: int) -> list[float]:
    """Every rank's value of x, in rank order (all ranks take part)."""
    if world == 1:
        return [x]
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


# ---------------------------------------------------------------------------
# CPU legs (oracle restatement on the host cores)
# ---------------------------------------------------------------------------

def cpu_linear_sample(M: int, N: int, K: int, rows: int, reps: int, threads: int) -> dict:
    """Times the oracle's W8A8 forward (quantise + int8 GEMM + epilogue) on a
    `rows`-row slice of the M x N x K workload; returns TOPS over the slice."""
    import numpy as np
    from oracle import oracle as O
    O.set_threads(threads)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(rows, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    xb, wb = O.torch_bf16_to_bits(x), O.torch_bf16_to_bits(w)
    wq, sw = O.c_quantize_rows(wb)
    times = []
    for _ in range(reps + 1):
        t0 = time.perf_counter()
        xq, sx = O.c_quantize_rows(xb)
        acc = O.c_int8_gemm(xq, wq)
        O.c_epilogue(acc, sx, sw, None)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times[1:])
    ops_ = 2.0 * rows * N * K
    return {"tops": ops_ / t / 1e12, "seconds": t, "rows": rows,
            "sample": f"{rows} of {M} rows x N={N} x K={K}, median of {reps} after 1 warm-up"}


# ---------------------------------------------------------------------------
# GPU workload: one W8A8 linear forward at 4096^3
# ---------------------------------------------------------------------------

def run_linear(args, world, rank, local) -> dict | None:
    from lema_b200 import _native, ops

    dev = torch.device("cuda", local)
    M = N = K = 4096
    ops_per_step = 2.0 * M * N * K
    # Rotate through enough distinct input/weight sets that every step reads
    # operands that are not L2-resident (footprint > 2 x L2).
    set_bytes = M * K * 2 + N * K + M * N * 2 + M * K
    n_sets = max(2, int(2 * L2_BYTES // set_bytes) + 1)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    xs, wqs, sws = [], [], []
    for i in range(n_sets):
        x = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
        x[:, :41] *= 20.0
        w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        wq, sw = ops.quantize_weight(w)
        xs.append(x)
        wqs.append(wq)
        sws.append(sw)
    xq = torch.empty(M, K, dtype=torch.int8, device=dev)
    sx = torch.empty(M, dtype=torch.float32, device=dev)
    ys = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(n_sets)]
    stream = torch.cuda.current_stream(dev)

    gemm_events = []

    def step(i, record=False):
        j = i % n_sets
        ops.quantize_rows(xs[j], out=xq, scale=sx)
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ops.w8a8_gemm(xq, sx, wqs[j], sws[j], out=ys[j])
        if record:
            e1.record(stream)
            gemm_events.append((e0, e1))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i, record=True)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    ms_max = max_over_ranks(ms, world)
    gemm_ms = statistics.mean(a.elapsed_time(b) for a, b in gemm_events)
    dev_err = _native.device_error()
    if dev_err:
        raise RuntimeError(f"kernel device error word {dev_err:#x}")

    # End to end through the public op with host buffers: pinned x -> H2D ->
    # w8a8_linear -> D2H of y, every step.
    x_host = [xs[j % n_sets].cpu().pin_memory() for j in range(2)]
    y_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    for i in range(args.warmup):
        xd = x_host[i % 2].to(dev, non_blocking=True)
        y = ops.w8a8_linear(xd, wqs[i % n_sets], sws[i % n_sets])
        y_host.copy_(y, non_blocking=True)
    torch.cuda.synchronize(dev)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        xd = x_host[i % 2].to(dev, non_blocking=True)
        y = ops.w8a8_linear(xd, wqs[i % n_sets], sws[i % n_sets])
        y_host.copy_(y, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)

    if rank != 0:
        return None
    peaks = read_peaks()
    lt_peak = args.int8_peak_tops or measure_int8_peak(dev)
    pk = int8_peaks(peaks)
    # the GEMM is timed alone here: the burst figure applies
    int8_peak = pk.get("burst", lt_peak)
    peak_source = ("2 x bf16_tflops of MEASURED_PEAKS.json (dense int8 = 2 x dense bf16 on "
                   "B200), of measured" if "burst" in pk else
                   "measured cuBLASLt int8 GEMM (torch._int_mm 8192^3, burst)")
    value = ops_per_step * args.steps * world / (ms_max / 1e3) / 1e12
    achieved = ops_per_step / (gemm_ms / 1e3) / 1e12
    e2e_value = ops_per_step * args.steps * world / (e2e_ms / 1e3) / 1e12
    res = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TOPS (int8, whole job)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 x int8 -> s32 -> bf16",
        "data": "synthetic (seeded randn activations with 1% outlier channels x20, W ~ N(0,0.02))",
        "config": {"workload": "w8a8_linear_4096: x[4096,4096] bf16 -> quantise -> int8 GEMM "
                               "with W[4096,4096] int8 -> bf16 y",
                   "M": M, "N": N, "K": K, "parallelism": f"replicas x{world}",
                   "l2": f"rotating {n_sets} operand sets ({n_sets * set_bytes / 2**20:.0f} MiB) "
                         "> L2, no flush"},
        "gpu_launches": 2 * args.steps,
        "roofline": {"bound": "tensor", "kernel": "gemm_sm100_pair_kernel<i8>",
                     "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
                     "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
                     "peak_source": peak_source,
                     "frac_of_spec_4500": round(achieved / INT8_SPEC_TOPS, 4),
                     "cublaslt_int8_8192_tops": round(lt_peak, 1),
                     # DRAM bytes (read + write) per launch of the CTA-pair kernel at
                     # 4096^3 from an ncu capture (--set full, one launch)
                     "traffic": LINEAR_GEMM_TRAFFIC_BYTES,
                     "algorithmic_ops_per_launch": ops_per_step,
                     "avg_launch_ms": round(gemm_ms, 5)},
        "clocks": clk,
        "e2e": {"value": round(e2e_value, 2), "unit": "TOPS (int8, whole job)",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                "path": "lema_b200.ops.w8a8_linear with pinned host x / y"},
    }
    if not args.skip_cpu:
        threads = len(os.sched_getaffinity(0))
        c = cpu_linear_sample(M, N, K, rows=args.cpu_rows, reps=3, threads=threads)
        res["cpu_baseline"] = {"value": round(c["tops"], 4), "unit": "TOPS", "cores": threads,
                               "kind": "port", "sample": c["sample"]}
    res["peaks_file"] = {k: peaks.get(k) for k in ("hbm_gbs", "bf16_tflops")}
    return res


# ---------------------------------------------------------------------------
# GPU workload: one streamed LoRA training step of the 7B-shaped model
# ---------------------------------------------------------------------------

def check_host_ram(shape, ranks_on_host: int) -> None:
    """Refuses (before pinning anything) a streamed workload whose pinned weight
    segments, for every rank on this host, would not fit in 80 % of the host's
    available memory."""
    import psutil
    per_layer = 0
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        o, i = shape.proj_shapes()[n]
        per_layer += o * i
    per_layer += 3 * shape.experts * shape.intermediate * shape.hidden
    need = per_layer * shape.layers * ranks_on_host
    avail = psutil.virtual_memory().available
    if need > 0.8 * avail:
        raise RuntimeError(f"{need / 1e9:.0f} GB of pinned weight segments needed for "
                           f"{ranks_on_host} rank(s) on this host, {avail / 1e9:.0f} GB "
                           "available: refusing")


def measure_h2d_gbs(dev, nbytes=1 << 30) -> float:
    """Pinned host -> device copy bandwidth of this GPU (one 1 GiB copy, best of 3)."""
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = float("inf")
    for _ in range(3):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return nbytes / (best / 1e3) / 1e9


def cpu_train_sample(seq: int, threads: int, moe: bool = False, reps: int = 1) -> dict:
    """CPU restatement of one streamed layer's work (no-grad forward, recompute
    with grad, backward) on one Llama-2-7B-shaped block (or, with ``moe``, one
    Mixtral-8x7B-shaped block: GQA attention + 8 experts, top-2) with the
    oracle's W8A8 linears (and W8A8 experts), LoRA r16 on q/v, for `seq` tokens;
    scaled to the 32-layer model (the embedding/head are not included)."""
    from lema_b200.llama import LlamaBlock, LlamaShape, apply_lora, rope_cos_sin
    from oracle import oracle as O
    from oracle.torch_ref import OracleExperts, swap_linears
    torch.set_num_threads(threads)
    O.set_threads(threads)
    g = torch.Generator().manual_seed(0)
    if moe:
        from lema_b200.moe import MixtralBlock, MixtralShape
        shape = MixtralShape()
        blk = MixtralBlock(shape, quantized=False, device="cpu")
        names = ("q_proj", "k_proj", "v_proj", "o_proj")
        label = "Mixtral-8x7B-shaped"
    else:
        shape = LlamaShape()
        blk = LlamaBlock(shape, quantized=False, device="cpu")
        names = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
        label = "Llama-2-7B-shaped"
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if "layernorm" in name:
                continue
            std = shape.hidden ** -0.5 if name.endswith("gate.weight") else 0.02
            p.copy_(std * torch.randn(p.shape, generator=g))
    apply_lora(blk, 16, 32.0)
    swap_linears(blk, names)
    if moe:
        ex = blk.mlp.experts
        blk.mlp.experts = OracleExperts(ex.gate_up_proj.data, ex.down_proj.data)
        for m in list(blk.mlp.experts.gu) + list(blk.mlp.experts.dn):
            m.wdeq_f32()
    blk.self_attn.attn_impl = "eager"
    for name in names:
        blk.base_projection(name).wdeq_f32()  # frozen weights: dequantised once, outside timing
    x = torch.randn(1, seq, shape.hidden, generator=g).to(torch.bfloat16)
    dy = torch.randn(1, seq, shape.hidden, generator=g).to(torch.bfloat16)
    cos, sin = rope_cos_sin(shape, seq, "cpu", torch.bfloat16)
    times = []
    for _ in range(max(1, reps)):  # the layer is built once; each repeat is timed alone
        t0 = time.perf_counter()
        with torch.no_grad():
            blk(x, cos, sin)
        xr = x.clone().requires_grad_(True)
        blk(xr, cos, sin).backward(dy)
        times.append(time.perf_counter() - t0)
    t_layer = statistics.median(times)
    return {"tokens_per_s": seq / (shape.layers * t_layer), "seconds_per_layer": t_layer,
            "reps": times,
            "sample": f"1 {label} layer, {seq} tokens, no-grad forward + recompute + "
                      f"backward through the oracle W8A8 linears ({t_layer:.2f} s), scaled x32 "
                      "layers (embedding / lm_head excluded)"}


REF_PKG = os.path.join(ROOT, "baseline", "_ref")


def reference_train_sample(threads: int, budget_s: float = 30.0, batch: int = 8,
                           seq: int = 512, hidden: int = 4096, inter: int = 11008,
                           vocab: int = 32000, heads: int = 32) -> dict | None:
    """The reference's own training step on the host cores, from the reference
    package installed in baseline/_ref: ``backend="python"``, ``device="cpu"``,
    bf16, LoRA r16 alpha 32 on q/v, AdamW, Llama-2-7B shapes (vocab 32000,
    random weights) at the full bs x seq. Two timings, each after one warm-up:
    ``LemaTrainer.train_step`` (src/lema/_trainer.py:75-194) of a one-layer
    truncation (embedding, one streamed decoder layer, head, loss, optimizer),
    and one decoder layer's share of a step through the reference adapter's own
    calls (``construct_layer_module``, the no-grad ``forward_layer``, the
    ``forward_layer`` with grad and its backward; src/lema/_trainer.py:101-112,
    140-167). Repeated until ``budget_s`` of timed work (at least once each).
    The 32-layer step is extrapolated as the one-layer step plus 31 layers.
    Returns None when the reference package is not installed."""
    if not os.path.exists(os.path.join(REF_PKG, "lema", "__init__.py")):
        return None
    import json as _json
    import tempfile

    from safetensors.torch import save_file
    if REF_PKG not in sys.path:
        sys.path.insert(0, REF_PKG)
    from lema import LemaConfig, LemaModel
    torch.set_num_threads(threads)
    H, I, V = hidden, inter, vocab
    g = torch.Generator().manual_seed(0)

    def w(*shape):
        return (0.02 * torch.randn(*shape, generator=g)).to(torch.bfloat16)
    p = "model.layers.0"
    sd = {"model.embed_tokens.weight": w(V, H), "model.norm.weight": torch.ones(H).bfloat16(),
          "lm_head.weight": w(V, H), f"{p}.input_layernorm.weight": torch.ones(H).bfloat16(),
          f"{p}.post_attention_layernorm.weight": torch.ones(H).bfloat16()}
    for n, shape in {"self_attn.q_proj": (H, H), "self_attn.k_proj": (H, H),
                     "self_attn.v_proj": (H, H), "self_attn.o_proj": (H, H),
                     "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H),
                     "mlp.down_proj": (H, I)}.items():
        sd[f"{p}.{n}.weight"] = w(*shape)
    step_t, layer_t = [], []
    with tempfile.TemporaryDirectory() as d:
        save_file(sd, os.path.join(d, "model.safetensors"))
        del sd
        _json.dump({"model_type": "llama", "architectures": ["LlamaForCausalLM"],
                    "hidden_size": H, "num_attention_heads": heads,
                    "num_key_value_heads": heads, "intermediate_size": I,
                    "num_hidden_layers": 1, "vocab_size": V, "rms_norm_eps": 1e-5,
                    "rope_theta": 10000.0, "max_position_embeddings": 4096,
                    "tie_word_embeddings": False, "hidden_act": "silu",
                    "torch_dtype": "bfloat16", "dtype": "bfloat16"},
                   open(os.path.join(d, "config.json"), "w"))
        cfg = LemaConfig(model_name_or_path=d, model_type="llama",
                         gbi_path=os.path.join(d, "model.safetensors"), device="cpu",
                         dtype="bfloat16", lora_rank=16, lora_alpha=32,
                         lora_target_modules=["q_proj", "v_proj"], save_steps=0,
                         backend="python", attn_implementation="eager", max_ram_gb=16.0,
                         max_vram_gb=1.0, vram_fraction=1.0)
        model = LemaModel(cfg)
        model.initialize_lora()
        opt = torch.optim.AdamW(model.lora_manager.get_trainable_parameters(), lr=1e-4)
        trainer = model.get_trainer(opt)
        adapter, lm = model.adapter, model.lora_manager
        ids = torch.randint(0, V, (batch, seq), generator=g)
        x = torch.randn(batch, seq, H, generator=g).to(torch.bfloat16)
        dy = torch.randn(batch, seq, H, generator=g).to(torch.bfloat16)

        def one_layer():
            module = adapter.construct_layer_module(1, None, lm)
            with torch.no_grad():
                adapter.forward_layer(module, x, gradient_checkpointing=False)
            xr = x.detach().requires_grad_(True)
            out = adapter.forward_layer(module, xr, gradient_checkpointing=False)
            (out[0] if isinstance(out, tuple) else out).backward(dy)
            adapter.release_layer_module(module)

        trainer.train_step(ids, labels=ids)  # warm-up
        one_layer()
        t_start = time.perf_counter()
        while not step_t or time.perf_counter() - t_start < budget_s:
            t0 = time.perf_counter()
            trainer.train_step(ids, labels=ids)
            step_t.append(time.perf_counter() - t0)
            t0 = time.perf_counter()
            one_layer()
            layer_t.append(time.perf_counter() - t0)
        trainer.close()
    t1, tl = statistics.median(step_t), statistics.median(layer_t)
    t32 = t1 + 31 * tl
    return {"tokens_per_s_32": batch * seq / t32, "step_s_32": t32, "step_s_1": t1,
            "layer_s": tl, "samples": len(step_t), "timed_s": sum(step_t) + sum(layer_t),
            "sample": (f"the reference's own LemaTrainer.train_step (backend=python, cpu, bf16, "
                       f"LoRA r16 q/v, AdamW), hidden {H} / MLP {I} / {heads} heads at bs "
                       f"{batch} x seq {seq}, vocab {V}: a one-layer truncation {t1:.2f} s per "
                       f"step, one decoder layer's share through the reference adapter "
                       f"{tl:.2f} s (median of {len(step_t)}); 32 layers extrapolated as the "
                       f"one-layer step + 31 layers = {t32:.1f} s")}


def run_train(args, world, rank, local) -> dict | None:
    from lema_b200 import _native, ops
    from lema_b200.llama import LlamaShape
    from lema_b200.tensorstore import ActivationCheckpointStore
    from lema_b200.trainer import StreamedLoraTrainer

    dev = torch.device("cuda", local)
    # run next to the GPU before pinning gigabytes of host memory (restored for the
    # CPU baseline, which uses every host thread)
    from lema_b200.topology import bind_to_gpu_cpus
    all_cpus = os.sched_getaffinity(0)
    local_cpus = bind_to_gpu_cpus(dev)
    shape = LlamaShape(layers=args.layers)
    long_ft = args.workload == "llama7b_selective_ft_2048"
    moe = args.workload == "mixtral_streamed_lora"
    model = "Llama-2-7B"
    shard = args.weight_stream == "sharded"
    if shard and world < 2:
        raise SystemExit("--weight-stream sharded needs --gpus >= 2")
    if args.vram_slots is None:
        args.vram_slots = 3 if shard else 2
    from lema_b200 import ops
    ops.set_dgrad_mode(args.dgrad)
    if moe:
        from lema_b200.moe import MixtralShape
        shape = MixtralShape(layers=args.layers)
        model = "Mixtral-8x7B"
        check_host_ram(shape, 1 if shard else int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
        batch, seq = 8, 512
        tr = StreamedLoraTrainer(shape, dev, batch=batch, seq=seq, lora_rank=16,
                                 lora_alpha=32.0, seed=0, resident_layers=args.resident_layers,
                                 weight_shard=shard, vram_slots=args.vram_slots,
                                 ckpt_mode=CKPT_MODES[args.ckpt],
                                 ckpt_hbm_budget=ckpt_budget_bytes(args), attn_impl=args.attn)
        workload = (f"mixtral_streamed_lora: {shape.layers} x [hidden 4096, 32 q / 8 kv heads "
                    "x 128, 8 experts x SwiGLU 14336, top-2 softmax routing], vocab 32000, LoRA "
                    "r16 a32 on q/v, W8A8 attention projections and grouped W8A8 experts "
                    f"streamed from pinned RAM ({tr.ws.seg_bytes / 1e9:.2f} GB per layer), "
                    "activation checkpoints offloaded to pinned host")
    elif long_ft:
        # bs 1 x seq 2048, 512-token chunked attention, activations offloaded, selective
        # full fine-tuning of q/k/v/o in the last 4 layers (fp32 AdamW states in host RAM)
        batch, seq = 1, 2048
        last4 = tuple(range(max(0, shape.layers - 4), shape.layers))
        tr = StreamedLoraTrainer(shape, dev, batch=batch, seq=seq, targets=(), seed=0,
                                 resident_layers=args.resident_layers, attn_chunk=512,
                                 full_ft_layers=last4, ckpt_mode=CKPT_MODES[args.ckpt],
                                 ckpt_hbm_budget=ckpt_budget_bytes(args),
                                 attn_impl=args.attn)
        workload = (f"llama7b_selective_ft_2048: {shape.layers} x [hidden 4096, 32x128 heads, "
                    "MLP 11008], vocab 32000, bs 1 x seq 2048, 512-token chunked causal "
                    "attention, W8A8 projections streamed from pinned RAM, activation "
                    f"checkpoints offloaded to pinned host, full fine-tuning of q/k/v/o in layers {list(last4)} "
                    "(fp32 AdamW states in pinned host RAM, re-quantised each step)")
    else:
        batch, seq = 8, 512
        tr = StreamedLoraTrainer(shape, dev, batch=batch, seq=seq, lora_rank=16,
                                 lora_alpha=32.0, seed=0, resident_layers=args.resident_layers,
                                 weight_shard=shard, vram_slots=args.vram_slots,
                                 ckpt_mode=CKPT_MODES[args.ckpt],
                                 ckpt_hbm_budget=ckpt_budget_bytes(args), attn_impl=args.attn)
        workload = (f"llama7b_streamed_lora: {shape.layers} x [hidden 4096, 32x128 heads, MLP "
                    "11008], vocab 32000, LoRA r16 a32 on q/v, W8A8 projections streamed "
                    "from pinned RAM, activation checkpoints offloaded to pinned host")
    tokens_per_step = batch * seq
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    n_batches = 4
    ids_dev = [torch.randint(0, shape.vocab, (batch, seq), device=dev, generator=gen)
               for _ in range(n_batches)]
    for i in range(args.warmup):
        tr.train_step(ids_dev[i % n_batches])
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    launches0 = _native.kernel_launches
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    losses = []
    for i in range(args.steps):
        losses.append(tr.train_step(ids_dev[i % n_batches]))
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop()
    launches = _native.kernel_launches - launches0
    ms = t0.elapsed_time(t1)
    ms_max = max_over_ranks(ms, world)
    # What the boundary-activation placement costs: the same K steps with the
    # other placement — every checkpoint in HBM (the reference's own,
    # src/lema/_trainer.py:109-111) when some were offloaded, else every one
    # offloaded to pinned host memory.
    ckpt_policy = {"device_slots": tr.ckpt.device_slots, "host_slots": tr.ckpt.host_slots,
                   "slot_bytes": math.prod(tr.ckpt.shape) * 2}
    ckpt_alt_ms = None
    if tr.L > 0:
        kept = tr.ckpt
        alt_mode = (ActivationCheckpointStore.DEVICE if kept.host_slots > 0 else 0)
        tr.ckpt = ActivationCheckpointStore(tr.L, kept.shape, dev, mode=alt_mode,
                                            h2d_stream=tr.ws.h2d_stream)
        for i in range(2):  # the new store's pinned slots and events warm up
            tr.train_step(ids_dev[i % n_batches])
        barrier(world)
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for i in range(args.steps):
            tr.train_step(ids_dev[i % n_batches])
        c1.record(stream)
        torch.cuda.synchronize(dev)
        ckpt_alt_ms = max_over_ranks(c0.elapsed_time(c1), world) / args.steps
        ckpt_policy["alternative"] = "all in HBM" if alt_mode == 2 else "all offloaded"
        tr.ckpt = kept
    # The same K steps again with an event pair around every int8 GEMM launch
    # (the tensor roofline). Kept out of the region above: an event record
    # between two kernels ends the programmatic overlap of the GEMM's set-up
    # with its producer, which costs a compute-bound step a few percent.
    barrier(world)
    ops.GemmTimer.enable(True)
    r0 = torch.cuda.Event(enable_timing=True)
    r1 = torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    for i in range(args.steps):
        tr.train_step(ids_dev[i % n_batches])
    r1.record(stream)
    torch.cuda.synchronize(dev)
    gemm_ops, gemm_ms, gemm_launches = ops.GemmTimer.summary()
    timed_step_ms = max_over_ranks(r0.elapsed_time(r1), world) / args.steps
    barrier(world)
    dev_err = _native.device_error()
    if dev_err:
        raise RuntimeError(f"kernel device error word {dev_err:#x}")
    # end to end: token ids from pinned host memory every step, loss read back
    ids_host = [t.cpu().pin_memory() for t in ids_dev]
    torch.cuda.synchronize(dev)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        loss = tr.train_step(ids_host[i % n_batches])
        loss_val = float(loss.item())
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    h2d_gbs = measure_h2d_gbs(dev)  # every rank at once: the rate each gets beside the others
    h2d_gbs_ranks = gather_over_ranks(h2d_gbs, world)
    step_ms_ranks = gather_over_ranks(ms / args.steps, world)
    seg_bytes = tr.ws.chunk  # per rank: the whole segment, or (sharded) its chunk
    streamed = shape.layers - args.resident_layers
    h2d_per_step = (2 * streamed - min(tr.nslots, streamed)) * seg_bytes + tr.ckpt.moved_bytes
    d2h_per_step = tr.ckpt.moved_bytes
    if tr.full_ft is not None:  # bf16 weight + fp32 m, v in; the same + int8 rows out
        n_ft = sum(w.numel() for w in tr.full_ft.true.values())
        h2d_per_step += n_ft * 10
        d2h_per_step += n_ft * 11
    tr.close()
    if rank != 0:
        return None
    value = tokens_per_step * world * args.steps / (ms_max / 1e3)
    e2e_value = tokens_per_step * world * args.steps / (e2e_ms / 1e3)
    lt_peak = args.int8_peak_tops or measure_int8_peak(dev)
    achieved = gemm_ops / (gemm_ms / 1e3) / 1e12
    step_s = ms_max / 1e3 / args.steps
    peaks = read_peaks()
    pk = int8_peaks(peaks)
    # the in-step GEMMs run inside a long step: the sustained figure applies
    int8_peak = pk.get("sustained", pk.get("burst", lt_peak))
    peak_source = ("2 x bf16_tflops_sustained of MEASURED_PEAKS.json (dense int8 = 2 x dense "
                   "bf16 on B200)" if "sustained" in pk else
                   "2 x bf16_tflops of MEASURED_PEAKS.json" if "burst" in pk else
                   "measured cuBLASLt int8 GEMM (torch._int_mm 8192^3, burst)")
    h2d_frac = h2d_per_step / (h2d_gbs * 1e9) / step_s
    gemm_rec = gemm_4096_record(dev, peaks, local) if args.workload == "llama7b_streamed_lora" \
        else None
    res = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s (whole job)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 W8A8 projections (bf16 activations; bf16 attention, LoRA, lm_head)",
        "data": f"synthetic (random-init {model}-shaped weights, token ids uniform in "
                "[0, 32000), labels = inputs)",
        "config": {"workload": workload,
                   "global_batch": batch * world, "seq_len": seq,
                   "parallelism": f"dp{world}",
                   "resident_layers": args.resident_layers,
                   "vram_slots": args.vram_slots,
                   "dgrad": args.dgrad,
                   "attention": args.attn,
                   "checkpoints": args.ckpt + ("" if args.ckpt_budget_gb is None
                                               else f" {args.ckpt_budget_gb} GB"),
                   "weight_stream": ("sharded: 1/N of each segment per rank over PCIe, NCCL "
                                     "all-gather over NVLink" if shard else
                                     "own: every rank streams its own full segments"),
                   "l2": f"per-step weight stream {h2d_per_step / 1e9:.1f} GB and "
                         "activations >> L2"},
        "gpu_launches": launches,
        "loss_last": round(float(losses[-1]), 4),
        "roofline": {"bound": "tensor", "kernel": "gemm_sm100 int8 (every int8 GEMM launch of "
                                                  "the timed steps: W8A8 projections, grouped "
                                                  "experts, int8-dy dgrads when selected)",
                     "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOPS",
                     "frac": round(achieved / int8_peak, 4),
                     "peak_source": peak_source + " (of measured)",
                     "frac_of_spec_4500": round(achieved / INT8_SPEC_TOPS, 4),
                     "cublaslt_int8_8192_tops": round(lt_peak, 1),
                     "frac_of_cublaslt": round(achieved / lt_peak, 4),
                     # DRAM bytes (read + write) per launch, averaged over a layer's four
                     # int8 GEMMs, from an ncu capture of this workload (4 metrics, 8 launches)
                     "traffic": TRAIN_GEMM_TRAFFIC_BYTES if not (long_ft or moe) else None,
                     "measured_over": f"a second run of the {args.steps} timed steps with "
                                      "an event pair around each int8 GEMM launch",
                     "instrumented_ms_per_step": round(timed_step_ms, 3),
                     "gemm_launches": gemm_launches,
                     "gemm_launches_untimed": ops.GemmTimer.dropped,
                     "gemm_ms_per_step": round(gemm_ms / args.steps, 3),
                     "algorithmic_ops_per_step": gemm_ops / args.steps},
        # the H2D rate is measured with every rank copying at once, which a step's
        # stream (it pauses between layers) never quite reaches
        "step_bound": "pcie (host -> device weight stream)" if h2d_frac > 0.75 else
                      "compute",
        "pcie": {"h2d_gbs_measured": round(h2d_gbs, 1),
                 "h2d_bytes_per_step": h2d_per_step, "d2h_bytes_per_step": d2h_per_step,
                 "h2d_bound_ms": round(h2d_per_step / (h2d_gbs * 1e9) * 1e3, 2),
                 "h2d_frac_of_step": round(h2d_frac, 3),
                 "per_rank": {"h2d_gbs_measured": [round(v, 1) for v in h2d_gbs_ranks],
                              "ms_per_step": [round(v, 2) for v in step_ms_ranks],
                              "stream_gbs": [round(h2d_per_step / v / 1e6, 1)
                                             for v in step_ms_ranks]}},
        "clocks": clk,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s (whole job)",
                "h2d_bytes_per_step": batch * seq * 8, "d2h_bytes_per_step": 4,
                "path": "StreamedLoraTrainer.train_step(ids in pinned host memory) + loss.item()"},
    }
    res["config"]["host_cpus"] = (f"{len(local_cpus)} GPU-local CPUs" if local_cpus
                                  else "unbound")
    if ckpt_alt_ms is not None:
        step_ms = ms_max / args.steps
        off_ms, dev_ms = ((step_ms, ckpt_alt_ms) if ckpt_policy["host_slots"] > 0
                          else (ckpt_alt_ms, step_ms))
        res["ckpt_offload"] = {
            **ckpt_policy,
            "policy": args.ckpt,
            "offload_all_overhead_ms": round(off_ms - dev_ms, 3),
            "timed_overhead_ms": round(step_ms - dev_ms, 3) if ckpt_policy["host_slots"] else 0.0,
            "timed_overhead_frac_of_step": round((step_ms - dev_ms) / step_ms, 4)
            if ckpt_policy["host_slots"] else 0.0,
            "alternative_ms_per_step": round(ckpt_alt_ms, 3),
            "what": "device_slots layers' boundary activations kept in HBM, host_slots "
                    "offloaded; the same steps were re-timed with the other placement "
                    "(alternative) to price the offload"}
    if gemm_rec is not None:
        res["gemm_4096"] = gemm_rec
    if not args.skip_cpu:
        os.sched_setaffinity(0, all_cpus)
        threads = len(all_cpus)
        c = cpu_train_sample(args.cpu_seq, threads, moe=moe)
        port = {"value": round(c["tokens_per_s"], 3), "unit": "tokens/s", "cores": threads,
                "kind": "port", "sample": c["sample"]}
        r = None if (moe or long_ft) else reference_train_sample(threads, budget_s=0.0)
        if r is not None:
            res["cpu_baseline"] = {"value": round(r["tokens_per_s_32"], 3), "unit": "tokens/s",
                                   "cores": threads, "kind": "reference",
                                   "sample": r["sample"]}
            res["cpu_baseline_port"] = port
        else:
            res["cpu_baseline"] = port
    return res


def int8_peaks(peaks: dict) -> dict:
    """Dense int8 peaks derived from MEASURED_PEAKS.json: B200's dense int8
    tensor rate is twice its dense bf16 rate, and the file holds the measured
    bf16 GEMM rate as a burst and sustained under the power cap."""
    out = {}
    if peaks.get("bf16_tflops"):
        out["burst"] = 2.0 * float(peaks["bf16_tflops"])
    if peaks.get("bf16_tflops_sustained"):
        out["sustained"] = 2.0 * float(peaks["bf16_tflops_sustained"])
    return out


def gemm_4096_record(dev, peaks: dict, local: int) -> dict:
    """The W8A8 GEMM alone at M = N = K = 4096 (int8 operands, fp32 scales,
    bf16 output through the fused epilogue): 20 back-to-back launches between
    two CUDA events, operands rotated over sets larger than 2 x L2, median of 7
    repeats; cuBLASLt's int8 GEMM (torch._int_mm) on the same operands beside
    it, and the SM clock sampled meanwhile."""
    from lema_b200 import ops
    M = N = K = 4096
    nsets = int(2 * L2_BYTES // (M * K + N * K + M * N * 2)) + 2
    g = torch.Generator(device=dev).manual_seed(7)
    A = [torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
         for _ in range(nsets)]
    B = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
         for _ in range(nsets)]
    sx = torch.rand(M, device=dev, generator=g) * 1e-3
    sw = torch.rand(N, device=dev, generator=g) * 1e-3
    Y = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(nsets)]

    def ours(n):
        for i in range(n):
            ops.w8a8_gemm(A[i % nsets], sx, B[i % nsets], sw, out=Y[i % nsets])

    def lt(n):
        for i in range(n):
            torch._int_mm(A[i % nsets], B[i % nsets].t())

    ours(5)
    lt(5)
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    t_ours, t_lt = [], []
    for _ in range(7):
        for fn, acc in ((ours, t_ours), (lt, t_lt)):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn(20)
            e1.record()
            torch.cuda.synchronize(dev)
            acc.append(e0.elapsed_time(e1) / 20 * 1e3)
    clk = clocks.stop()
    us, us_lt = statistics.median(t_ours), statistics.median(t_lt)
    ops_ = 2.0 * M * N * K
    tops = ops_ / (us * 1e-6) / 1e12
    rec = {"us": round(us, 2), "tops": round(tops, 1),
           "frac_of_spec_4500": round(tops / INT8_SPEC_TOPS, 4),
           "cublaslt_us": round(us_lt, 2), "cublaslt_tops": round(ops_ / (us_lt * 1e-6) / 1e12, 1),
           "sm_mhz": clk.get("sm_mhz"), "clock_reasons": clk.get("reasons"),
           "timing": "20 back-to-back launches per event pair, operands rotated over "
                     f"{nsets} sets (> 2 x L2), median of 7, interleaved with cuBLASLt"}
    pk = int8_peaks(peaks)
    if "burst" in pk:
        rec["frac_of_2x_measured_bf16_burst"] = round(tops / pk["burst"], 4)
    del A, B, Y
    torch.cuda.empty_cache()
    return rec


def measure_int8_peak(dev) -> float:
    """Burst throughput of cuBLASLt's int8 GEMM (torch._int_mm) at 8192^3."""
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    bt = b.t()
    for _ in range(3):
        torch._int_mm(a, bt)
    torch.cuda.synchronize(dev)
    best = float("inf")
    for _ in range(10):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, bt)
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1))
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def run_reference(args) -> dict | None:
    """CPU arm: the oracle restatement of the path on all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    threads = len(os.sched_getaffinity(0))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload in ("llama7b_streamed_lora", "llama7b_selective_ft_2048",
                         "mixtral_streamed_lora"):
        moe = args.workload == "mixtral_streamed_lora"
        t_run = time.perf_counter()
        # the oracle's W8A8 restatement of one layer (the port), warm-up repeats dropped
        warm = 1
        c = cpu_train_sample(args.cpu_seq, threads, moe=moe, reps=warm + 2)
        t_layer = statistics.median(c["reps"][warm:])
        port_tps = args.cpu_seq / (32 * t_layer)
        port = {"value": round(port_tps, 3), "unit": "tokens/s", "cores": threads,
                "kind": "port", "sample": c["sample"]}
        r = None if args.workload != "llama7b_streamed_lora" else \
            reference_train_sample(threads, budget_s=30.0)
        if r is not None:
            value, n, per_sample_s = r["tokens_per_s_32"], r["samples"], \
                r["timed_s"] / r["samples"]
            baseline = {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                        "kind": "reference", "sample": r["sample"]}
            timed = {"one_layer_step_s": round(r["step_s_1"], 3),
                     "decoder_layer_s": round(r["layer_s"], 3), "samples": n,
                     "timed_s": round(r["timed_s"], 2)}
            rule = ("tokens/s of the 32-layer model: bs 8 x seq 512 tokens over the one-layer "
                    "step + 31 decoder layers, both timed on the reference's own code")
            note = ("the reference's own Python training step (bf16; it has no W8A8 path) on "
                    "the host cores; cpu_baseline_port times the oracle's W8A8 restatement")
        else:
            value, n, per_sample_s = port_tps, len(c["reps"]) - warm, t_layer
            baseline = port
            timed = {"layer_s": round(t_layer, 3), "samples": n, "tokens": args.cpu_seq}
            rule = (f"one layer at {args.cpu_seq} tokens scaled x32 layers; embedding / "
                    "lm_head excluded")
            note = ("the reference package is not installed in baseline/_ref: the oracle's "
                    "W8A8 restatement is timed")
        out = {
            "metric": METRIC, "impl": "reference", "value": round(value, 3),
            "unit": "tokens/s (whole job)", "n_gpus": world, "steps": n, "warmup": 1,
            "ms_per_step": round(per_sample_s * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 (the reference's own path)" if r is not None else
                     "int8 W8A8 projections (bf16 activations)",
            "data": "synthetic",
            "config": {"workload": f"{args.workload} (CPU samples, extrapolated to 32 layers)",
                       "global_batch": 8, "seq_len": 512, "parallelism": "cpu"},
            "scaled_from": {"timed": timed, "rule": rule,
                            "steps_requested": args.steps, "warmup_requested": args.warmup},
            "cpu_baseline": baseline,
            "e2e": {"value": round(value, 3), "unit": "tokens/s (whole job)",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(time.perf_counter() - t_run, 1),
            "note": note,
        }
        if r is not None:
            out["cpu_baseline_port"] = port
        return out
    M = N = K = 4096
    for _ in range(max(1, args.warmup)):
        cpu_linear_sample(M, N, K, rows=args.cpu_rows, reps=1, threads=threads)
    vals = [cpu_linear_sample(M, N, K, rows=args.cpu_rows, reps=1, threads=threads)
            for _ in range(args.steps)]
    tops = statistics.median(v["tops"] for v in vals)
    return {
        "metric": METRIC, "impl": "reference", "value": round(tops, 4),
        "unit": "TOPS (int8, whole job)", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(statistics.median(v["seconds"] for v in vals) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> s32 -> bf16", "data": "synthetic",
        "config": {"workload": "w8a8_linear_4096 (row sample on CPU)", "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": round(tops, 4), "unit": "TOPS", "cores": threads,
                         "kind": "port", "sample": vals[0]["sample"]},
        "e2e": {"value": round(tops, 4), "unit": "TOPS (int8, whole job)",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no W8A8 linear; the CPU restatement in oracle/ is timed",
    }


CKPT_MODES = {"budget": None, "host": 0, "host-kernel": 1, "device": 2}


def ckpt_budget_bytes(args) -> int | None:
    """HBM bytes for boundary activations under --ckpt budget (None: the trainer's default)."""
    return None if args.ckpt_budget_gb is None else int(args.ckpt_budget_gb * 1e9)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="llama7b_streamed_lora",
                    choices=["llama7b_streamed_lora", "llama7b_selective_ft_2048",
                             "mixtral_streamed_lora",
                             "w8a8_linear_4096"])
    ap.add_argument("--weight-stream", choices=["own", "sharded"], default="own",
                    help="own (default): every rank streams its own segments; sharded: each "
                         "rank uploads 1/N of every segment and the rest is all-gathered over "
                         "NVLink (opt-in; adds a weight collective)")
    ap.add_argument("--vram-slots", type=int, default=None,
                    help="VRAM slots of the weight stream (uploads run slots-1 layers ahead); "
                         "default 2 (the reference's double buffering), 3 when sharded")
    ap.add_argument("--dgrad", choices=["bf16", "int8"], default="bf16",
                    help="straight-through dgrad of the frozen projections: bf16 (the "
                         "operator contract, default) or the opt-in int8-dy variant")
    ap.add_argument("--attn", choices=["sdpa", "tcgen05"], default="sdpa",
                    help="block attention: torch SDPA (default) or this library's tcgen05 "
                         "kernels (opt-in, head_dim 128)")
    ap.add_argument("--ckpt", choices=list(CKPT_MODES), default="host",
                    help="boundary activations: host (default: all offloaded to pinned host "
                         "by the copy engine), host-kernel (all offloaded by the SM store "
                         "kernel), budget (kept in HBM while they fit a quarter of the free "
                         "memory, the rest offloaded) or device (all kept in HBM)")
    ap.add_argument("--ckpt-budget-gb", type=float, default=None,
                    help="with --ckpt budget: HBM bytes (GB) for boundary activations "
                         "(default a quarter of the free memory); layers past it are offloaded")
    ap.add_argument("--resident-layers", type=int, default=0,
                    help="keep this many blocks' int8 segments resident in HBM")
    ap.add_argument("--cpu-seq", type=int, default=128)
    ap.add_argument("--layers", type=int, default=32,
                    help="decoder layers of the streamed model (32 = Llama-2-7B; fewer only "
                         "for short profiling runs, never for a reported number)")
    ap.add_argument("--cpu-rows", type=int, default=256)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--int8-peak-tops", type=float, default=0.0)
    args = ap.parse_args()
    train = args.workload in ("llama7b_streamed_lora", "llama7b_selective_ft_2048",
                              "mixtral_streamed_lora")
    if args.steps is None:
        args.steps = (3 if args.impl == "reference" else 10) if train else 50
    if args.warmup is None:
        args.warmup = 3 if train else 5
    if args.warmup < 3 and args.impl != "reference":
        args.warmup = 3
    if args.impl == "reference":
        res = run_reference(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.workload == "w8a8_linear_4096":
            res = run_linear(args, world, rank, local)
        else:
            res = run_train(args, world, rank, local)
        if res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
