"""GPU parity tests of the sm_100a kernels against the CPU oracle, called
through the C ABI (lema_b200.ops wraps it with torch tensors).

Bars: int8 quantised values, scales and s32 accumulators bit-exact; the
dequant epilogue bit-exact too (same fp32 operation order, no FMA); the bf16
dgrad GEMM within |dev - ref| <= 2^-7 * |ref| + 2^-9 * rms(ref) of the
double-accumulated reference (fp32 summation order + one bf16 rounding).
"""
import numpy as np
import pytest
import torch

from lema_b200 import _native
from lema_b200 import ops

pytestmark = pytest.mark.gpu


def bits(t):
    from oracle.oracle import torch_bf16_to_bits
    return torch_bf16_to_bits(t)


def rand_bf16(shape, seed, scale=1.0, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    if outliers and shape[-1] >= 10:
        idx = torch.randperm(shape[-1], generator=g)[: max(1, shape[-1] // 100)]
        x[..., idx] *= 20.0
    return x.to(torch.bfloat16)


# --------------------------------------------------------------------------- K2 first:
# the smallest tcgen05 case runs before anything else.

def test_gemm_tiny_s32_exact(cuda_device, oracle):
    rng = np.random.default_rng(0)
    a = rng.integers(-127, 128, size=(128, 128), dtype=np.int8)
    b = rng.integers(-127, 128, size=(128, 128), dtype=np.int8)
    sx = np.ones(128, np.float32)
    sw = np.ones(128, np.float32)
    dev = cuda_device
    y, acc = ops.w8a8_gemm(torch.from_numpy(a).to(dev), torch.from_numpy(sx).to(dev),
                           torch.from_numpy(b).to(dev), torch.from_numpy(sw).to(dev),
                           want_acc=True)
    ref = oracle.c_int8_gemm(a, b)
    np.testing.assert_array_equal(acc.cpu().numpy(), ref)


# --------------------------------------------------------------------------- K1

@pytest.mark.parametrize("shape", [(512, 4096), (3, 11008), (17, 14336), (5, 20000),
                                   (64, 4104), (9, 33), (1, 8), (300, 1),
                                   # many rows (several CTA waves), long rows
                                   (2000, 4096), (700, 11008), (301, 24576), (1000, 1032)])
def test_quantize_rows_bitexact(cuda_device, oracle, shape):
    x = rand_bf16(shape, seed=shape[0] + shape[1])
    if shape[0] > 2:
        x[1] = 0.0
    q, s = ops.quantize_rows(x.to(cuda_device))
    qr, sr = oracle.c_quantize_rows(bits(x))
    np.testing.assert_array_equal(s.cpu().numpy(), sr)
    np.testing.assert_array_equal(q.cpu().numpy(), qr)


def test_quantize_rows_strided_and_f32(cuda_device, oracle):
    base = rand_bf16((40, 1000), seed=5).to(cuda_device)
    view = base[:, 3:903]  # unaligned start, row pitch 1000
    q, s = ops.quantize_rows(view)
    qr, sr = oracle.c_quantize_rows(bits(view.cpu()))
    np.testing.assert_array_equal(q.cpu().numpy(), qr)
    np.testing.assert_array_equal(s.cpu().numpy(), sr)
    for shape in ((33, 4096), (1000, 3000)):
        xf = torch.randn(*shape, generator=torch.Generator().manual_seed(9)) * 0.02
        q, s = ops.quantize_rows(xf.to(cuda_device))
        qr, sr = oracle.c_quantize_rows_f32(xf.numpy())
        np.testing.assert_array_equal(q.cpu().numpy(), qr)
        np.testing.assert_array_equal(s.cpu().numpy(), sr)


def test_quantize_adversarial_rows(cuda_device, oracle):
    """Rows whose quotients x / s sit on or near half-integers, and rows with
    subnormal scales: the device quotient must round exactly like the oracle's
    IEEE division."""
    allbits = np.arange(65536, dtype=np.uint32)
    f = (allbits << 16).view(np.float32)
    f = f[np.isfinite(f)]
    rng = np.random.default_rng(7)
    pos = np.unique(np.abs(f[f != 0]))
    amaxes = np.concatenate([pos[:24], pos[-8:], rng.choice(pos, 80, replace=False),
                             np.float32([1.0, 127.0, 254.0, 2.0, 0.5, 63.5])])
    rows = []
    for amax in amaxes.astype(np.float32):
        cand = f[np.abs(f) <= amax]
        row = rng.choice(cand, 4095, replace=True).astype(np.float32)
        rows.append(np.concatenate([[amax], row]))
    # exact ties: s = 1 (amax 127) and s = 2 (amax 254) with k + 0.5 values
    ties = np.float32([127.0] + [k + 0.5 for k in range(-127, 127)] + [0.0] * 3841)
    rows.append(ties)
    rows.append(ties * 2)
    x = torch.from_numpy(np.stack(rows)).to(torch.bfloat16)
    q, s = ops.quantize_rows(x.to(cuda_device))
    qr, sr = oracle.c_quantize_rows(bits(x))
    np.testing.assert_array_equal(s.cpu().numpy(), sr)
    np.testing.assert_array_equal(q.cpu().numpy(), qr)


def test_quantize_empty(cuda_device):
    x = torch.empty(0, 64, dtype=torch.bfloat16, device=cuda_device)
    q, s = ops.quantize_rows(x)
    assert q.shape == (0, 64) and s.shape == (0,)


# --------------------------------------------------------------------------- K2/K3

GEMM_SHAPES = [
    (512, 4096, 4096),   # the single-linear workload
    (128, 256, 128),
    (200, 300, 208),     # ragged M and N, K tail inside a 128-byte slice
    (1, 64, 32),
    (257, 520, 4112),
    (1024, 11008, 4096),  # gate/up shape, 128x256 tiles
    (333, 4096, 11008),   # down shape, K = 11008
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_w8a8_gemm_bitexact(cuda_device, oracle, M, N, K):
    x = rand_bf16((M, K), seed=M * 7 + K)
    w = rand_bf16((N, K), seed=N * 13 + K, scale=0.02, outliers=False)
    g = torch.Generator().manual_seed(M + N)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    ref = oracle.w8a8_linear_ref(bits(x), bits(w), bits(bias))
    dev = cuda_device
    xq, sx = ops.quantize_rows(x.to(dev))
    wq, sw = ops.quantize_weight(w.to(dev))
    np.testing.assert_array_equal(wq.cpu().numpy(), ref["wq"])
    np.testing.assert_array_equal(sw.cpu().numpy(), ref["sw"])
    y, acc = ops.w8a8_gemm(xq, sx, wq, sw, bias=bias.to(dev), want_acc=True)
    np.testing.assert_array_equal(acc.cpu().numpy(), ref["acc"])
    np.testing.assert_array_equal(bits(y), ref["y"])
    # no-bias epilogue skips the add entirely
    y0 = ops.w8a8_gemm(xq, sx, wq, sw)
    np.testing.assert_array_equal(bits(y0), oracle.c_epilogue(ref["acc"], ref["sx"], ref["sw"], None))


def test_w8a8_linear_fwd_fused_entry(cuda_device, oracle):
    x, w, bias = oracle.cfg1_inputs(seed=0)
    ref = oracle.w8a8_linear_ref(bits(x), bits(w), bits(bias))
    dev = cuda_device
    wq, sw = ops.quantize_weight(w.to(dev))
    y = ops.w8a8_linear_forward(x.to(dev), wq, sw, bias.to(dev))
    np.testing.assert_array_equal(bits(y), ref["y"])


def test_gemm_full_size_checksums(cuda_device, oracle):
    """M=N=K=4096: exact int64 row and column sums of the s32 accumulator."""
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(11)
    a = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8, device=dev, generator=g)
    ones = torch.ones(4096, dtype=torch.float32, device=dev)
    _, acc = ops.w8a8_gemm(a, ones, b, ones, want_y=False, want_acc=True)
    rs, cs = oracle.c_int8_gemm_checksums(a.cpu().numpy(), b.cpu().numpy())
    np.testing.assert_array_equal(acc.long().sum(1).cpu().numpy(), rs)
    np.testing.assert_array_equal(acc.long().sum(0).cpu().numpy(), cs)
    # and a sampled block exactly
    blk = oracle.c_int8_gemm(a[1000:1130].cpu().numpy(), b[2000:2300].cpu().numpy())
    np.testing.assert_array_equal(acc[1000:1130, 2000:2300].cpu().numpy(), blk)


def test_gemm_k_zero_gives_bias(cuda_device):
    dev = cuda_device
    xq = torch.empty(5, 0, dtype=torch.int8, device=dev)
    wq = torch.empty(7, 0, dtype=torch.int8, device=dev)
    bias = torch.arange(7, dtype=torch.float32, device=dev).to(torch.bfloat16)
    y = ops.w8a8_gemm(xq, torch.ones(5, device=dev), wq, torch.ones(7, device=dev), bias=bias)
    assert torch.equal(y, bias.expand(5, 7))


# --------------------------------------------------------------------------- K4

def _dgrad_tol_check(dev_bits, ref_f32):
    dv = torch.from_numpy(dev_bits.view(np.int16)).view(torch.bfloat16).float().numpy()
    rms = float(np.sqrt(np.mean(ref_f32.astype(np.float64) ** 2))) + 1e-30
    err = np.abs(dv - ref_f32)
    bound = 2.0 ** -7 * np.abs(ref_f32) + 2.0 ** -9 * rms
    assert np.all(err <= bound), f"max err {err.max()} (rms {rms})"


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (100, 300, 200), (64, 11008, 4096)])
def test_dequant_transpose_and_dgrad(cuda_device, oracle, M, N, K):
    dev = cuda_device
    w = rand_bf16((N, K), seed=N + K, scale=0.02, outliers=False)
    wq, sw = ops.quantize_weight(w.to(dev))
    wdT = ops.dequant_transpose(wq, sw)
    ref_wdT = oracle.c_dequant_transpose(wq.cpu().numpy(), sw.cpu().numpy())
    np.testing.assert_array_equal(bits(wdT.contiguous()), ref_wdT)
    dy = rand_bf16((M, N), seed=M + 3, outliers=False)
    dx = ops.w8a8_dgrad(dy.to(dev), wq, sw)
    # dx[m, k] = sum_n dy[m, n] * wdT[k, n]: wdT is the [K, N] right operand
    _, ref = oracle.c_bf16_gemm_tn(bits(dy), ref_wdT)
    _dgrad_tol_check(bits(dx), ref)


@pytest.mark.parametrize("shape", [(64, 4096), (7, 4100), (3, 11008), (5, 24576), (1, 8),
                                   (300, 16), (0, 64), (9, 8192), (40, 22016), (2, 24584),
                                   (600, 2048)])
def test_quantize_rows_colscaled_bitexact(cuda_device, oracle, shape):
    """Rows of fp32(x) * cs quantised: the vector paths (cols % 8 == 0, 128 to
    512 threads per row up to 24576 columns), the generic path (ragged or longer
    rows) and the empty case, all bit-exact."""
    x = rand_bf16(shape, seed=shape[0] * 3 + shape[1], outliers=False)
    g = torch.Generator().manual_seed(shape[1])
    cs = torch.rand(shape[1], generator=g) * 0.01 + 1e-4
    if shape[0] > 2:
        x[1] = 0.0
    q, s = ops.quantize_rows_colscaled(x.to(cuda_device), cs.to(cuda_device))
    f = (x.float().numpy() * cs.numpy()[None, :]).astype(np.float32)
    qr, sr = oracle.c_quantize_rows_f32(f)
    np.testing.assert_array_equal(q.cpu().numpy(), qr)
    np.testing.assert_array_equal(s.cpu().numpy(), sr)


@pytest.mark.parametrize("N,K", [(4096, 4096), (11008, 4096), (4096, 11008), (37, 129),
                                 (64, 128), (1, 5), (22016, 4096), (130, 260), (200, 33)])
def test_transpose_i8_exact(cuda_device, N, K):
    g = torch.Generator(device=cuda_device).manual_seed(N + K)
    wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=cuda_device, generator=g)
    t = ops.transpose_i8(wq)
    assert torch.equal(t, wq.t())
    # strided source (a column window of a wider matrix) takes the scalar loads
    if K > 3:
        t2 = ops.transpose_i8(wq[:, 1:K - 1])
        assert torch.equal(t2, wq[:, 1:K - 1].t())


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (100, 300, 200), (64, 11008, 4096),
                                   (1024, 4096, 11008)])
def test_w8a8_dgrad_int8(cuda_device, oracle, M, N, K):
    """The optional int8-dy dgrad: bit-exact against its own restatement (scaled
    quantiser, s32 GEMM, epilogue with unit column scales), and within a 2e-2
    relative RMS of the bf16 straight-through dgrad it approximates."""
    dev = cuda_device
    w = rand_bf16((N, K), seed=N * 3 + K, scale=0.02, outliers=False)
    wq, sw = ops.quantize_weight(w.to(dev))
    dy = rand_bf16((M, N), seed=M + 5, outliers=False)
    dx = ops.w8a8_dgrad_int8(dy.to(dev), wq, sw)
    ref = oracle.dgrad_int8_ref(bits(dy), wq.cpu().numpy(), sw.cpu().numpy())
    np.testing.assert_array_equal(bits(dx), ref["dx"])
    # against the contract's bf16 dgrad (double-accumulated)
    ref_wdT = oracle.c_dequant_transpose(wq.cpu().numpy(), sw.cpu().numpy())
    _, exact = oracle.c_bf16_gemm_tn(bits(dy), ref_wdT)
    got = torch.from_numpy(bits(dx).view(np.int16)).view(torch.bfloat16).float().numpy()
    rms = float(np.sqrt(np.mean(exact.astype(np.float64) ** 2)))
    rel = float(np.sqrt(np.mean((got.astype(np.float64) - exact) ** 2))) / rms
    assert rel <= 2e-2, rel
    # the mode switch routes the straight-through dgrad through the same entry point
    prev = ops.dgrad_mode()
    ops.set_dgrad_mode("int8")
    try:
        assert torch.equal(ops.w8a8_dgrad(dy.to(dev), wq, sw), dx)
    finally:
        ops.set_dgrad_mode(prev)


def test_bf16_gemm_tn(cuda_device, oracle):
    dev = cuda_device
    a = rand_bf16((300, 520), seed=1, outliers=False)
    b = rand_bf16((260, 520), seed=2, outliers=False)
    y = ops.bf16_gemm_tn(a.to(dev), b.to(dev))
    _, ref = oracle.c_bf16_gemm_tn(bits(a), bits(b))
    _dgrad_tol_check(bits(y), ref)


# --------------------------------------------------------------------------- K6

def test_grouped_gemm_matches_per_expert(cuda_device, oracle):
    dev = cuda_device
    E, N, K = 8, 384, 512
    counts = [130, 0, 7, 256, 1, 300, 64, 129]
    offsets = np.concatenate([[0], np.cumsum(counts)]).tolist()
    T = offsets[-1]
    x = rand_bf16((T, K), seed=21)
    w = rand_bf16((E, N, K), seed=22, scale=0.02, outliers=False)
    xq, sx = ops.quantize_rows(x.to(dev))
    wq, sw = ops.quantize_rows(w.reshape(E * N, K).to(dev))
    wq3 = wq.reshape(E, N, K) if wq.is_contiguous() else wq.contiguous().reshape(E, N, K)
    y = ops.grouped_w8a8_gemm(xq, sx, wq3, sw.reshape(E, N), offsets)
    xb = bits(x)
    wqn = wq.cpu().numpy().reshape(E, N, K)
    swn = sw.cpu().numpy().reshape(E, N)
    xqn, sxn = oracle.c_quantize_rows(xb)
    for e in range(E):
        r0, r1 = offsets[e], offsets[e + 1]
        if r1 == r0:
            continue
        acc = oracle.c_int8_gemm(xqn[r0:r1], wqn[e])
        ref = oracle.c_epilogue(acc, sxn[r0:r1], swn[e], None)
        np.testing.assert_array_equal(bits(y[r0:r1].contiguous()), ref, err_msg=f"expert {e}")


# --------------------------------------------------------------------------- K5

@pytest.mark.parametrize("mode", [0, 1])
def test_ckpt_save_restore_roundtrip(cuda_device, mode):
    import ctypes as C
    from lema_b200 import _native as N
    dev = cuda_device
    src = torch.randn(4096 * 8 + 3, device=dev).to(torch.bfloat16)
    nbytes = src.numel() * 2
    host = torch.empty(src.numel(), dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.Stream(device=dev)
    ready = torch.cuda.Event()
    ready.record(torch.cuda.current_stream(dev))
    done = torch.cuda.Event()
    N.call("lema_ckpt_save", src.data_ptr(), host.data_ptr(), nbytes, mode, stream.cuda_stream,
           C.c_void_p(ready.cuda_event), C.c_void_p(done.cuda_event))
    done.synchronize()
    assert torch.equal(host.view(torch.int16), src.cpu().view(torch.int16))
    back = torch.empty_like(src)
    N.call("lema_ckpt_restore", host.data_ptr(), back.data_ptr(), nbytes, stream.cuda_stream,
           None, C.c_void_p(done.cuda_event))
    done.synchronize()
    assert torch.equal(back.view(torch.int16), src.view(torch.int16))


def test_ckpt_kernel_mode_rejects_pageable_memory(cuda_device):
    from lema_b200 import _native as N
    src = torch.zeros(64, device=cuda_device)
    host = torch.zeros(64)  # pageable
    with pytest.raises(N.LemaError):
        N.call("lema_ckpt_save", src.data_ptr(), host.data_ptr(), 256, 1, None, None, None)


# --------------------------------------------------------------------------- tile paths
# Every GEMM tile path (1-SM 128x128, 1-SM 128x256, CTA-pair 256x256) against
# the oracle, forced with LEMA_GEMM_TILE.

PATH_SHAPES = [(300, 520, 4112), (1000, 768, 640), (4096, 4096, 4096), (64, 256, 128)]


@pytest.mark.parametrize("path", ["1sm128", "1sm256", "pair"])
@pytest.mark.parametrize("M,N,K", PATH_SHAPES)
def test_gemm_tile_paths_bitexact(cuda_device, oracle, monkeypatch, path, M, N, K):
    monkeypatch.setenv("LEMA_GEMM_TILE", path)
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    sx = torch.rand(M, device=dev, generator=g) * 0.01 + 1e-4
    sw = torch.rand(N, device=dev, generator=g) * 1e-3 + 1e-5
    bias = (torch.randn(N, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    y, acc = ops.w8a8_gemm(a, sx, b, sw, bias=bias, want_acc=True)
    an, bn = a.cpu().numpy(), b.cpu().numpy()
    if M * N * K <= 2 ** 31:
        ref = oracle.c_int8_gemm(an, bn)
        np.testing.assert_array_equal(acc.cpu().numpy(), ref)
    else:
        rs, cs = oracle.c_int8_gemm_checksums(an, bn)
        np.testing.assert_array_equal(acc.long().sum(1).cpu().numpy(), rs)
        np.testing.assert_array_equal(acc.long().sum(0).cpu().numpy(), cs)
        ref = acc.cpu().numpy()
        blk = oracle.c_int8_gemm(an[3900:4096], bn[3800:4096])
        np.testing.assert_array_equal(ref[3900:4096, 3800:4096], blk)
    yref = oracle.c_epilogue(acc.cpu().numpy(), sx.cpu().numpy(), sw.cpu().numpy(), bits(bias))
    np.testing.assert_array_equal(bits(y), yref)


@pytest.mark.parametrize("path", ["1sm128", "1sm256", "pair"])
def test_bf16_gemm_tile_paths(cuda_device, oracle, monkeypatch, path):
    monkeypatch.setenv("LEMA_GEMM_TILE", path)
    dev = cuda_device
    a = rand_bf16((600, 1040), seed=31, outliers=False)
    b = rand_bf16((520, 1040), seed=32, outliers=False)
    y = ops.bf16_gemm_tn(a.to(dev), b.to(dev))
    _, ref = oracle.c_bf16_gemm_tn(bits(a), bits(b))
    _dgrad_tol_check(bits(y), ref)


# Stream-K: when the tile count leaves the last wave part-empty, every worker
# gets an equal range of K-slices; a tile cut across workers is finished by its
# owner (the worker holding its first slices), which adds the other workers'
# s32 partials published through a per-stream workspace. LEMA_GEMM_SPLIT=1
# forces the plan down to one K-slice per worker, so a tile can have many
# contributors.
SPLIT_CASES = [("pair", 768, 1024, 4096),     # 12 tiles over 74 pairs: 6-7 workers a tile
               ("pair", 300, 520, 8208),      # ragged M, N; 65 K-slices per tile
               ("pair", 512, 1024, 4096),     # 8 tiles, ~9 workers each
               ("1sm256", 384, 1024, 16384),  # 12 tiles over 148 CTAs
               ("1sm128", 333, 600, 11008),
               ("1sm128", 128, 256, 2048),    # 2 tiles of 16 slices: 16 one-slice workers each
               ("pair", 4096, 4096, 4096)]    # 2 whole waves, then 108 tiles over 74 ranges


@pytest.mark.parametrize("raster", ["1", "8"])
@pytest.mark.parametrize("path,M,N,K", SPLIT_CASES)
def test_gemm_stream_k_bitexact(cuda_device, oracle, monkeypatch, path, M, N, K, raster):
    monkeypatch.setenv("LEMA_GEMM_TILE", path)
    monkeypatch.setenv("LEMA_GEMM_RASTER", raster)
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(M * 7 + K)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    sx = torch.rand(M, device=dev, generator=g) * 0.01 + 1e-4
    sw = torch.rand(N, device=dev, generator=g) * 1e-3 + 1e-5
    monkeypatch.setenv("LEMA_GEMM_SPLIT", "0")
    y_whole = ops.w8a8_gemm(a, sx, b, sw)
    monkeypatch.setenv("LEMA_GEMM_SPLIT", "1")
    for _ in range(2):  # the second launch reuses the workspace under a new epoch
        y, acc = ops.w8a8_gemm(a, sx, b, sw, want_acc=True)
        y2 = ops.w8a8_gemm(a, sx, b, sw)  # TMA-store epilogue (no raw accumulator output)
        assert torch.equal(y2.view(torch.int16), y_whole.view(torch.int16))
        if M * N * K <= 2 ** 31:
            ref = oracle.c_int8_gemm(a.cpu().numpy(), b.cpu().numpy())
        else:  # exact row / column sums and a corner block
            rs, cs = oracle.c_int8_gemm_checksums(a.cpu().numpy(), b.cpu().numpy())
            np.testing.assert_array_equal(acc.long().sum(1).cpu().numpy(), rs)
            np.testing.assert_array_equal(acc.long().sum(0).cpu().numpy(), cs)
            ref = acc.cpu().numpy().copy()
            ref[-200:, -300:] = oracle.c_int8_gemm(a[-200:].cpu().numpy(), b[-300:].cpu().numpy())
        np.testing.assert_array_equal(acc.cpu().numpy(), ref)
        yref = oracle.c_epilogue(acc.cpu().numpy(), sx.cpu().numpy(), sw.cpu().numpy(), None)
        np.testing.assert_array_equal(bits(y), yref)
        np.testing.assert_array_equal(bits(y2), yref)


def test_gemm_stream_k_default_plan_bitexact(cuda_device, oracle, monkeypatch):
    """The default plan (no forcing) at the training shapes: q/k/v stacked
    (12288 columns), o (4096) and down (K = 11008), against the whole-tile
    schedule, bit for bit."""
    monkeypatch.delenv("LEMA_GEMM_SPLIT", raising=False)
    monkeypatch.delenv("LEMA_GEMM_TILE", raising=False)
    dev = cuda_device
    for M, N, K in ((4096, 12288, 4096), (4096, 4096, 4096), (4096, 4096, 11008)):
        g = torch.Generator(device=dev).manual_seed(N + K)
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        sx = torch.rand(M, device=dev, generator=g) * 0.01 + 1e-4
        sw = torch.rand(N, device=dev, generator=g) * 1e-3 + 1e-5
        y = ops.w8a8_gemm(a, sx, b, sw)
        monkeypatch.setenv("LEMA_GEMM_SPLIT", "0")
        y_whole = ops.w8a8_gemm(a, sx, b, sw)
        monkeypatch.delenv("LEMA_GEMM_SPLIT")
        assert torch.equal(y.view(torch.int16), y_whole.view(torch.int16)), (M, N, K)


def test_gemm_stream_k_wait_timeout_records_error_and_recovers(cuda_device, oracle,
                                                               monkeypatch):
    """The abort path of the bounded waits: with the test hook that withholds
    every partial's publish and a wait budget of about 1 ms, each owner's wait
    for its contributors runs out; the kernel records 0x104 in the error word,
    drains, frees its TMEM and returns, and the next GEMM on the same stream
    and workspace is bit-exact."""
    monkeypatch.setenv("LEMA_GEMM_TILE", "pair")
    monkeypatch.setenv("LEMA_GEMM_SPLIT", "1")
    dev = cuda_device
    M, N_, K = 768, 1024, 4096  # 12 tiles cut over 74 pairs: every tile has contributors
    g = torch.Generator(device=dev).manual_seed(77)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (N_, K), dtype=torch.int8, device=dev, generator=g)
    sx = torch.rand(M, device=dev, generator=g) * 0.01 + 1e-4
    sw = torch.rand(N_, device=dev, generator=g) * 1e-3 + 1e-5
    assert _native.device_error() == 0
    _native.gemm_set_test_hooks(skip_publish=True, wait_budget_cycles=2_000_000)
    try:
        ops.w8a8_gemm(a, sx, b, sw)
        torch.cuda.synchronize()
    finally:
        _native.gemm_set_test_hooks(False, 0)
    assert _native.device_error() == 0x104
    y, acc = ops.w8a8_gemm(a, sx, b, sw, want_acc=True)
    np.testing.assert_array_equal(acc.cpu().numpy(),
                                  oracle.c_int8_gemm(a.cpu().numpy(), b.cpu().numpy()))
    assert _native.device_error() == 0


def test_bf16_gemm_split_tail_deterministic(cuda_device, oracle, monkeypatch):
    """bf16 kind: the owner adds fp32 partials in a fixed order, so a split GEMM
    is within the bf16 bar and identical from run to run."""
    monkeypatch.setenv("LEMA_GEMM_TILE", "pair")
    monkeypatch.setenv("LEMA_GEMM_SPLIT", "1")
    dev = cuda_device
    a = rand_bf16((512, 8192), seed=51, outliers=False).to(dev)
    b = rand_bf16((512, 8192), seed=52, outliers=False).to(dev)
    y1 = ops.bf16_gemm_tn(a, b)
    y2 = ops.bf16_gemm_tn(a, b)
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    _, ref = oracle.c_bf16_gemm_tn(bits(a.cpu()), bits(b.cpu()))
    _dgrad_tol_check(bits(y1), ref)


@pytest.mark.parametrize("path", ["1sm128", "pair"])
def test_grouped_gemm_tile_paths(cuda_device, oracle, monkeypatch, path):
    monkeypatch.setenv("LEMA_GEMM_TILE", path)
    dev = cuda_device
    E, N, K = 4, 512, 384
    counts = [300, 0, 513, 77]
    offsets = np.concatenate([[0], np.cumsum(counts)]).tolist()
    T = offsets[-1]
    g = torch.Generator(device=dev).manual_seed(41)
    xq = torch.randint(-127, 128, (T, K), dtype=torch.int8, device=dev, generator=g)
    sx = torch.rand(T, device=dev, generator=g) * 0.01 + 1e-4
    wq = torch.randint(-127, 128, (E, N, K), dtype=torch.int8, device=dev, generator=g)
    sw = torch.rand(E, N, device=dev, generator=g) * 1e-3 + 1e-5
    y = ops.grouped_w8a8_gemm(xq, sx, wq, sw, offsets)
    xqn, sxn, wqn, swn = (t.cpu().numpy() for t in (xq, sx, wq, sw))
    for e in range(E):
        r0, r1 = offsets[e], offsets[e + 1]
        if r1 == r0:
            continue
        acc = oracle.c_int8_gemm(xqn[r0:r1], wqn[e])
        ref = oracle.c_epilogue(acc, sxn[r0:r1], swn[e], None)
        np.testing.assert_array_equal(bits(y[r0:r1].contiguous()), ref, err_msg=f"expert {e}")


@pytest.mark.parametrize("path", ["1sm128", "pair"])
def test_grouped_dgrad_matches_oracle(cuda_device, oracle, monkeypatch, path):
    """Per-expert straight-through dgrad over rows sorted by expert (empty and
    ragged experts included) against the oracle's dequant + double GEMM."""
    monkeypatch.setenv("LEMA_GEMM_TILE", path)
    dev = cuda_device
    E, N, K = 5, 640, 384
    counts = [300, 0, 129, 1, 200]
    offsets = np.concatenate([[0], np.cumsum(counts)]).tolist()
    T = offsets[-1]
    w = rand_bf16((E * N, K), seed=51, scale=0.02, outliers=False)
    wq, sw = ops.quantize_rows(w.to(dev))
    dy = rand_bf16((T, N), seed=52, outliers=False)
    dx = ops.grouped_w8a8_dgrad(dy.to(dev), wq.reshape(E, N, K), sw.reshape(E, N), offsets)
    wqn, swn = wq.cpu().numpy().reshape(E, N, K), sw.cpu().numpy().reshape(E, N)
    for e in range(E):
        r0, r1 = offsets[e], offsets[e + 1]
        if r1 == r0:
            continue
        wdT = oracle.c_dequant_transpose(wqn[e], swn[e])
        _, ref = oracle.c_bf16_gemm_tn(bits(dy[r0:r1].contiguous()), wdT)
        _dgrad_tol_check(bits(dx[r0:r1].contiguous()), ref)


@pytest.mark.parametrize("E,N,K,counts", [(5, 640, 384, [300, 0, 129, 1, 200]),
                                          (8, 4096, 1024, [512, 384, 0, 640, 128, 256, 64, 33])])
def test_grouped_dgrad_int8_bitexact(cuda_device, oracle, E, N, K, counts):
    """The int8-dy grouped dgrad: each expert's rows bit-exact against the oracle's
    int8-dy chain with that expert's weight (empty and ragged experts included),
    and through the mode switch of ``grouped_w8a8_dgrad``."""
    dev = cuda_device
    offsets = np.concatenate([[0], np.cumsum(counts)]).tolist()
    T = offsets[-1]
    w = rand_bf16((E * N, K), seed=61 + N, scale=0.02, outliers=False)
    wq, sw = ops.quantize_rows(w.to(dev))
    dy = rand_bf16((T, N), seed=62 + N, outliers=False)
    wq3, sw2 = wq.reshape(E, N, K), sw.reshape(E, N)
    dx = ops.grouped_w8a8_dgrad_int8(dy.to(dev), wq3, sw2, offsets)
    wqn, swn = wq.cpu().numpy().reshape(E, N, K), sw.cpu().numpy().reshape(E, N)
    for e in range(E):
        r0, r1 = offsets[e], offsets[e + 1]
        if r1 == r0:
            continue
        ref = oracle.dgrad_int8_ref(bits(dy[r0:r1].contiguous()), wqn[e], swn[e])
        np.testing.assert_array_equal(bits(dx[r0:r1].contiguous()), ref["dx"], err_msg=str(e))
    prev = ops.dgrad_mode()
    ops.set_dgrad_mode("int8")
    try:
        assert torch.equal(ops.grouped_w8a8_dgrad(dy.to(dev), wq3, sw2, offsets), dx)
    finally:
        ops.set_dgrad_mode(prev)


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (77, 300, 200)])
def test_wgrad_fp32_accumulators(cuda_device, oracle, M, N, K):
    """dW = dy^T . x with fp32 output against a double-accumulated reference; the
    bar is fp32 accumulation-order noise: 2e-5 * |ref| + 1e-5 * rms(ref)."""
    dev = cuda_device
    dy = rand_bf16((M, N), seed=61, outliers=False)
    x = rand_bf16((M, K), seed=62, outliers=False)
    dw = ops.w8a8_wgrad(dy.to(dev), x.to(dev)).cpu().numpy()
    _, ref = oracle.c_bf16_gemm_tn(bits(dy.t().contiguous()), bits(x.t().contiguous()))
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    err = np.abs(dw - ref)
    assert np.all(err <= 2e-5 * np.abs(ref) + 1e-5 * rms + 1e-30), err.max()


def test_gemm_timer_records_int8_launches(cuda_device):
    """The library's GEMM timer records one event pair per int8 GEMM launch
    (dense, grouped, inside the fused forward) and none for bf16 GEMMs."""
    dev = cuda_device
    x = rand_bf16((512, 1024), seed=3).to(dev)
    wq, sw = ops.quantize_weight(rand_bf16((768, 1024), seed=4, scale=0.02).to(dev))
    ops.GemmTimer.enable(True)
    ops.w8a8_linear_forward(x, wq, sw)
    xq, sx = ops.quantize_rows(x)
    ops.w8a8_gemm(xq, sx, wq, sw)
    ops.bf16_gemm_tn(x, x[:256])
    wg = wq.view(1, 768, 1024)
    ops.grouped_w8a8_gemm(xq, sx, wg, sw.view(1, 768), [0, 300])
    total_ops, ms, n = ops.GemmTimer.summary()
    assert n == 3 and ops.GemmTimer.dropped == 0
    assert total_ops == 2.0 * 1024 * 768 * (512 + 512 + 300)
    assert 0.0 < ms < 1000.0
    # stopped: nothing more is recorded
    ops.w8a8_gemm(xq, sx, wq, sw)
    ops.GemmTimer.enable(True)
    assert ops.GemmTimer.summary()[2] == 0
