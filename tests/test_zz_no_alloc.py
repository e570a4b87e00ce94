"""GPU test of lema_w8a8_linear_fwd_noalloc, the forward for callers that
cannot allocate device memory (a host binding without a CUDA allocator, or a
process whose device memory belongs to a caching allocator under a fixed
budget). It keeps its quantisation workspace in fixed arrays inside the
library instead of taking one from the caller.

Checked through the C ABI against lema_w8a8_linear_fwd, which takes
caller-allocated workspaces: the two run the same kernels, so outputs must be
bit-identical (the same bar as the other forward tests). Two calls in a row
with different shapes make sure the shared workspace carries nothing from one
call into the next. This file sorts last so a stop-at-first-failure run has
already run every other test; it also passes on its own in a fresh process.
"""
import pytest
import torch

from lema_b200 import _native as N
from lema_b200 import ops

pytestmark = pytest.mark.gpu


def _inputs(M, N_, K, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    x[:, : max(1, K // 100)] *= 20.0
    w = (torch.randn(N_, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    bias = (torch.randn(N_, generator=g) * 0.1).to(torch.bfloat16).to(dev)
    return x.to(torch.bfloat16).to(dev), w, bias


def _allocating(x, wq, sw, bias):
    M, K = x.shape
    N_ = wq.shape[0]
    ldq = (K + 15) // 16 * 16
    xq = torch.empty(M, ldq, dtype=torch.int8, device=x.device)
    sx = torch.empty(M, dtype=torch.float32, device=x.device)
    y = torch.empty(M, N_, dtype=torch.bfloat16, device=x.device)
    N.call("lema_w8a8_linear_fwd", x.data_ptr(), x.stride(0), wq.data_ptr(), wq.stride(0),
           sw.data_ptr(), bias.data_ptr(), y.data_ptr(), N_, xq.data_ptr(), ldq, sx.data_ptr(),
           M, N_, K, torch.cuda.current_stream().cuda_stream)
    return y


def _noalloc(x, wq, sw, bias):
    M, K = x.shape
    N_ = wq.shape[0]
    y = torch.empty(M, N_, dtype=torch.bfloat16, device=x.device)
    N.call("lema_w8a8_linear_fwd_noalloc", x.data_ptr(), x.stride(0), wq.data_ptr(),
           wq.stride(0), sw.data_ptr(), bias.data_ptr(), y.data_ptr(), N_, M, N_, K,
           torch.cuda.current_stream().cuda_stream)
    return y


def test_noalloc_forward_matches_allocating_forward_twice(cuda_device):
    dev = cuda_device
    # 1st call: a large workspace footprint; 2nd: fewer rows and a ragged K, so
    # stale rows / padding from the 1st call would show up if they were read.
    for (M, N_, K, seed) in [(2048, 1024, 4096, 1), (77, 520, 1000, 2)]:
        x, w, bias = _inputs(M, N_, K, seed, dev)
        wq, sw = ops.quantize_weight(w)
        y_ref = _allocating(x, wq, sw, bias)
        y = _noalloc(x, wq, sw, bias)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16)), (M, N_, K)
    assert N.device_error() == 0


def test_noalloc_rejects_oversized_requests(cuda_device):
    dev = cuda_device
    wq = torch.zeros(16, 4096, dtype=torch.int8, device=dev)
    sw = torch.ones(16, dtype=torch.float32, device=dev)
    y = torch.empty(1, 16, dtype=torch.bfloat16, device=dev)
    # 4097 rows x 4096 columns = 16 MiB + 4 KiB of int8 activations: over the limit.
    with pytest.raises(N.LemaError) as e:
        N.call("lema_w8a8_linear_fwd_noalloc", None, 4096, wq.data_ptr(), 4096, sw.data_ptr(),
               None, y.data_ptr(), 16, 4097, 16, 4096, None)
    assert e.value.code == N.LEMA_ERR_UNSUPPORTED and "16 MiB" in str(e.value)
    with pytest.raises(N.LemaError) as e:
        N.call("lema_w8a8_linear_fwd_noalloc", None, 16, wq.data_ptr(), 16, sw.data_ptr(),
               None, y.data_ptr(), 16, 65537, 16, 16, None)
    assert e.value.code == N.LEMA_ERR_UNSUPPORTED and "65536" in str(e.value)


def test_noalloc_never_allocates_a_stream_k_workspace(cuda_device, monkeypatch):
    """With stream-K forced (LEMA_GEMM_SPLIT=1, every shape whose tile count
    leaves a part-empty wave is cut), the allocating forward would create a
    per-stream workspace on its first GEMM on a stream; the allocation-free
    entry point runs every tile whole instead. On a fresh stream, after the
    library's module is loaded (the fixed arrays are part of it), a call leaves
    the workspace count and the device's free memory unchanged, and its output
    is still bit-identical to the allocating forward's."""
    dev = cuda_device
    monkeypatch.setenv("LEMA_GEMM_SPLIT", "1")
    M, N_, K = 768, 1024, 4096  # 12 tiles of 256 x 256: the forced plan would split them
    x, w, bias = _inputs(M, N_, K, 3, dev)
    wq, sw = ops.quantize_weight(w)
    _noalloc(x, wq, sw, bias)  # module load and symbol lookup happen here at the latest
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y = torch.empty(M, N_, dtype=torch.bfloat16, device=dev)
        torch.cuda.synchronize()
        before_ws = N.gemm_workspace_count()
        free_before, _ = torch.cuda.mem_get_info()
        for _ in range(2):
            N.call("lema_w8a8_linear_fwd_noalloc", x.data_ptr(), x.stride(0), wq.data_ptr(),
                   wq.stride(0), sw.data_ptr(), bias.data_ptr(), y.data_ptr(), N_, M, N_, K,
                   s.cuda_stream)
        s.synchronize()
        free_after, _ = torch.cuda.mem_get_info()
        assert N.gemm_workspace_count() == before_ws
        assert free_after == free_before
        y_ref = _allocating(x, wq, sw, bias)  # this one may create the stream's workspace
        s.synchronize()
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    assert N.device_error() == 0
