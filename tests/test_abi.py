"""CPU tests of the C ABI library: it loads, exports every entry point the
header declares, and its host-only logic (argument checks, the memory
manager's packing and prefetch job pool, bounded waits) behaves. No kernel is
launched here."""
import ctypes as C
import re
import threading
import time
from pathlib import Path

import numpy as np
import pytest

from lema_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "lema_b200.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(lema_\w+)\s*\(", text)))


def test_library_loads_and_reports_version():
    assert N.version().startswith("lema_b200")
    assert N.last_error() == ""


def test_every_declared_symbol_is_exported():
    lib = N.lib()
    declared = header_functions()
    assert len(declared) >= 30
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in lema_b200.h but not exported"
    # and the ctypes table covers the header exactly
    assert sorted(N.exported_symbols()) == declared


def test_argument_errors_do_not_touch_the_gpu():
    lib = N.lib()
    rc = lib.lema_quantize_rows(None, 4, 8, 8, None, 16, None, None)
    assert rc == N.LEMA_ERR_INVALID_ARGUMENT and "null" in N.last_error()
    rc = lib.lema_quantize_rows(None, -1, 8, 8, None, 16, None, None)
    assert rc == N.LEMA_ERR_INVALID_ARGUMENT
    # an empty problem is a no-op success
    assert lib.lema_quantize_rows(None, 0, 8, 8, None, 16, None, None) == 0
    rc = lib.lema_w8a8_gemm(None, 16, None, None, 16, None, None, None, 16, None, 16,
                            -1, 4, 4, None)
    assert rc == N.LEMA_ERR_INVALID_ARGUMENT
    offs = (C.c_int64 * 2)(0, 4)
    rc = lib.lema_grouped_w8a8_gemm(None, 16, None, None, 16, None, None, None, 16, offs,
                                    65, 8, 16, None)
    assert rc == N.LEMA_ERR_UNSUPPORTED
    rc = lib.lema_ckpt_save(None, None, 16, 0, None, None, None)
    assert rc == N.LEMA_ERR_INVALID_ARGUMENT
    rc = lib.lema_w8a8_dgrad(None, 8, None, 16, None, None, 16, None, 3, 4, 4, 4, None)
    assert rc == N.LEMA_ERR_MISALIGNED


def test_argument_errors_of_the_dgrad_optimizer_and_timer_entries():
    """The int8-dy dgrad pieces, the fused AdamW step and the GEMM timer reject
    bad arguments (and accept empty problems) before any CUDA call."""
    lib = N.lib()
    fake = 4096  # a non-null address that is never dereferenced
    assert lib.lema_quantize_rows_colscaled(None, None, 4, 8, 8, None, 16, None,
                                            None) == N.LEMA_ERR_INVALID_ARGUMENT
    assert lib.lema_quantize_rows_colscaled(None, None, 0, 8, 8, None, 16, None, None) == 0
    assert lib.lema_quantize_rows_colscaled(fake, fake, 4, 8, 4, fake, 16, fake,
                                            None) == N.LEMA_ERR_INVALID_ARGUMENT  # ldx < cols
    assert lib.lema_transpose_i8(None, 16, 4, 8, None, 16, None) == N.LEMA_ERR_INVALID_ARGUMENT
    assert lib.lema_transpose_i8(None, 16, 0, 8, None, 16, None) == 0
    assert lib.lema_transpose_i8(fake, 16, 40, 8, fake, 16, None) == N.LEMA_ERR_INVALID_ARGUMENT
    rc = lib.lema_w8a8_dgrad_int8(None, 8, None, 16, None, None, 16, None, 8, None, 16, None,
                                  4, 8, 16, None)
    assert rc == N.LEMA_ERR_MISALIGNED  # ldt must be a multiple of 16
    rc = lib.lema_w8a8_dgrad_int8(fake, 8, fake, 16, None, fake, 16, fake, 16, fake, 16, fake,
                                  4, 8, 16, None)
    assert rc == N.LEMA_ERR_INVALID_ARGUMENT and "scales" in N.last_error()
    coef = (1.0, 0.9, 0.1, 0.999, 0.001, 0.03, -0.01, 1e-8)
    assert lib.lema_adamw_requant_rows(None, 8, None, 8, None, None, 8, 0, 8, *coef, 1, None,
                                       16, None, None) == 0
    assert lib.lema_adamw_requant_rows(None, 8, None, 8, None, None, 8, 2, 8, *coef, 1, None,
                                       16, None, None) == N.LEMA_ERR_INVALID_ARGUMENT
    assert lib.lema_adamw_requant_rows(fake, 4, fake, 8, fake, fake, 8, 2, 8, *coef, 1, fake,
                                       16, fake, None) == N.LEMA_ERR_INVALID_ARGUMENT
    assert lib.lema_gemm_timer_start(0) == N.LEMA_ERR_INVALID_ARGUMENT
    ops_, ms = C.c_double(-1.0), C.c_double(-1.0)
    n, dropped = C.c_int64(-1), C.c_int64(-1)
    assert lib.lema_gemm_timer_stop(C.byref(ops_), C.byref(ms), C.byref(n), C.byref(dropped)) == 0
    assert (ops_.value, ms.value, n.value) == (0.0, 0.0, 0)


class HostManager:
    """A host-only (device = -1) native manager: packing and the job pool."""

    def __init__(self, layers=4):
        self.h = C.c_void_p()
        N.call("lema_mm_create", layers, 1 << 20, -1, C.byref(self.h))

    def close(self):
        N.call("lema_mm_destroy", self.h)


def test_manager_pack_and_status_flags():
    mm = HostManager()
    try:
        buf = np.zeros(64, dtype=np.uint8)
        N.call("lema_mm_register_ram_buffer", mm.h, 1000, buf.ctypes.data, buf.nbytes)
        flag = C.c_int32(0)
        N.call("lema_mm_is_layer_in_ram", mm.h, 1000, C.byref(flag))
        assert flag.value == 1
        N.call("lema_mm_is_layer_in_ram", mm.h, 2, C.byref(flag))
        assert flag.value == 0
        a = np.arange(10, dtype=np.uint8)
        b = np.arange(100, 105, dtype=np.uint8)
        srcs = (C.c_void_p * 2)(a.ctypes.data, b.ctypes.data)
        sizes = (C.c_size_t * 2)(a.nbytes, b.nbytes)
        N.call("lema_mm_pack_layer_to_ram", mm.h, 1000, srcs, sizes, 2)
        assert list(buf[:15]) == list(range(10)) + list(range(100, 105))
        offs = (C.c_size_t * 2)()
        buf[:] = 0
        N.call("lema_mm_pack_layer_to_ram_aligned", mm.h, 1000, srcs, sizes, 2, 32, offs)
        assert list(offs) == [0, 32]
        assert list(buf[32:37]) == list(range(100, 105))
        # overflow and unregistered buffers are reported, not crashed on
        big = (C.c_size_t * 2)(60, 10)
        with pytest.raises(N.LemaError) as e:
            N.call("lema_mm_pack_layer_to_ram", mm.h, 1000, srcs, big, 2)
        assert e.value.code == N.LEMA_ERR_OVERFLOW
        with pytest.raises(N.LemaError) as e:
            N.call("lema_mm_pack_layer_to_ram", mm.h, 7, srcs, sizes, 2)
        assert e.value.code == N.LEMA_ERR_NOT_REGISTERED
        # transfers need a device
        ev = C.c_int64(-1)
        with pytest.raises(N.LemaError):
            N.call("lema_mm_async_transfer_to_vram", mm.h, 1000, 0, 0, C.byref(ev))
        # invalid event ids are no-ops, as in the reference
        N.call("lema_mm_wait_vram_transfer", mm.h, -5)
        done = C.c_int32(0)
        N.call("lema_mm_is_transfer_complete", mm.h, 4096, C.byref(done))
        assert done.value == 1
    finally:
        mm.close()


def test_manager_prefetch_jobs_and_bounded_wait():
    mm = HostManager()
    gate = threading.Event()
    ran = []

    @N.JOB_FN
    def job(user):
        gate.wait(5.0)
        ran.append(user)

    try:
        jid = C.c_int64(0)
        N.call("lema_mm_submit_prefetch_job", mm.h, job, C.c_void_p(7), C.byref(jid))
        done = C.c_int32(1)
        N.call("lema_mm_is_prefetch_complete", mm.h, jid.value, C.byref(done))
        assert done.value == 0
        t0 = time.time()
        with pytest.raises(N.LemaError) as e:
            N.call("lema_mm_wait_for_prefetch_timeout", mm.h, jid.value, 50)
        assert e.value.code == N.LEMA_ERR_TIMEOUT
        assert time.time() - t0 < 2.0
        gate.set()
        N.call("lema_mm_wait_for_prefetch", mm.h, jid.value)
        N.call("lema_mm_is_prefetch_complete", mm.h, jid.value, C.byref(done))
        assert done.value == 1 and ran == [7]
        # unknown job ids count as complete (reference semantics)
        N.call("lema_mm_is_prefetch_complete", mm.h, 123456, C.byref(done))
        assert done.value == 1
    finally:
        mm.close()


def test_noalloc_size_checks_cannot_overflow():
    """The allocation-free forward rejects sizes past its fixed workspace before
    forming any product of them, so a huge K cannot wrap around the check."""
    lib = N.lib()
    huge = (1 << 63) - 3
    for M, K in ((1, huge), (2, huge), (1, (1 << 24) + 1), (65536, 512)):
        rc = lib.lema_w8a8_linear_fwd_noalloc(None, 16, None, 16, None, None, None, 16,
                                              M, 16, K, None)
        assert rc == N.LEMA_ERR_UNSUPPORTED and "16 MiB" in N.last_error(), (M, K)
    rc = lib.lema_w8a8_linear_fwd_noalloc(None, 16, None, 16, None, None, None, 16,
                                          65537, 16, 16, None)
    assert rc == N.LEMA_ERR_UNSUPPORTED and "65536" in N.last_error()
