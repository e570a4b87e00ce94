"""ctypes binding of ``liblema_b200.so`` (the C ABI declared in include/lema_b200.h).

The library is built in-tree (``python -m lema_b200.build``). There is no
fallback: if the library is missing or a call fails, a ``LemaError`` is
raised with the library's own message.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblema_b200.so"

_lib = None
_lock = threading.Lock()

i64 = C.c_int64
i32 = C.c_int32
vp = C.c_void_p
sz = C.c_size_t

JOB_FN = C.CFUNCTYPE(None, vp)

# name -> argument types (all return int status unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "lema_last_error": [],
    "lema_version": [],
    "lema_device_error": [C.POINTER(i32)],
    "lema_device_error_async": [vp, vp],
    "lema_gemm_workspace_count": [C.POINTER(i64)],
    "lema_gemm_set_test_hooks": [i32, i64],
    "lema_num_sms": [C.POINTER(i32)],
    "lema_quantize_rows": [vp, i64, i64, i64, vp, i64, vp, vp],
    "lema_quantize_rows_f32": [vp, i64, i64, i64, vp, i64, vp, vp],
    "lema_quantize_per_token": [vp, i64, i64, i64, vp, i64, vp, vp],
    "lema_w8a8_gemm": [vp, i64, vp, vp, i64, vp, vp, vp, i64, vp, i64, i64, i64, i64, vp],
    "lema_w8a8_linear_fwd": [vp, i64, vp, i64, vp, vp, vp, i64, vp, i64, vp, i64, i64, i64, vp],
    "lema_w8a8_linear_fwd_noalloc": [vp, i64, vp, i64, vp, vp, vp, i64, i64, i64, i64, vp],
    "lema_dequant_transpose": [vp, i64, vp, i64, i64, vp, i64, vp],
    "lema_bf16_gemm_tn": [vp, i64, vp, i64, vp, i64, i64, i64, i64, vp],
    "lema_bf16_gemm_tn_f32": [vp, i64, vp, i64, vp, i64, i64, i64, i64, vp],
    "lema_w8a8_dgrad": [vp, i64, vp, i64, vp, vp, i64, vp, i64, i64, i64, i64, vp],
    "lema_quantize_rows_colscaled": [vp, vp, i64, i64, i64, vp, i64, vp, vp],
    "lema_transpose_i8": [vp, i64, i64, i64, vp, i64, vp],
    "lema_w8a8_dgrad_int8": [vp, i64, vp, i64, vp, vp, i64, vp, i64, vp, i64, vp, i64, i64, i64,
                             vp],
    "lema_adamw_requant_rows": [vp, i64, vp, i64, vp, vp, i64, i64, i64, C.c_float, C.c_float,
                                C.c_float, C.c_float, C.c_float, C.c_float, C.c_float,
                                C.c_float, i32, vp, i64, vp, vp],
    "lema_gemm_timer_start": [i64],
    "lema_gemm_timer_stop": [C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(i64),
                             C.POINTER(i64)],
    "lema_grouped_w8a8_gemm": [vp, i64, vp, vp, i64, vp, vp, vp, i64, vp, i32, i64, i64, vp],
    "lema_grouped_bf16_gemm_tn": [vp, i64, vp, i64, vp, i64, vp, i32, i64, i64, vp],
    "lema_grouped_w8a8_dgrad": [vp, i64, vp, i64, vp, vp, i64, vp, i64, vp, i32, i64, i64, vp],
    "lema_rmsnorm_quant": [vp, i64, vp, i64, i64, C.c_float, vp, i64, vp, i64, vp, vp, vp],
    "lema_rmsnorm_bwd": [vp, i64, vp, vp, vp, i64, i64, i64, vp, i64, vp],
    "lema_rope": [vp, i64, vp, i64, vp, vp, i64, i32, i32, i32, i32, vp, vp, i32, vp],
    "lema_rope_qkv": [vp, i64, vp, i64, vp, i64, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32,
                      vp, vp, vp, i32, vp],
    "lema_swiglu_quant": [vp, i64, i64, i64, vp, i64, vp, vp, i64, vp],
    "lema_swiglu_bwd": [vp, i64, vp, i64, i64, i64, vp, i64, vp],
    "lema_attn_fwd": [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, i64, i64, i64, i64,
                      C.c_float, vp],
    "lema_attn_bwd": [vp, i64, vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, vp, vp, i64, vp,
                      i64, vp, i64, i64, i64, i64, i64, i64, C.c_float, vp],
    "lema_attn_set_wait_budget": [i64],
    "lema_ckpt_save": [vp, vp, sz, i32, vp, vp, vp],
    "lema_ckpt_restore": [vp, vp, sz, vp, vp, vp],
    "lema_mm_create": [i64, i64, i32, C.POINTER(vp)],
    "lema_mm_destroy": [vp],
    "lema_mm_register_ram_buffer": [vp, i64, vp, sz],
    "lema_mm_register_vram_slot": [vp, i64, vp, sz],
    "lema_mm_pack_layer_to_ram": [vp, i64, C.POINTER(vp), C.POINTER(sz), i64],
    "lema_mm_pack_layer_to_ram_aligned": [vp, i64, C.POINTER(vp), C.POINTER(sz), i64, sz,
                                          C.POINTER(sz)],
    "lema_mm_async_transfer_to_vram": [vp, i64, i64, sz, C.POINTER(i64)],
    "lema_mm_stream_wait_transfer": [vp, i64, vp],
    "lema_mm_release_vram_slot": [vp, i64, vp],
    "lema_mm_wait_vram_transfer": [vp, i64],
    "lema_mm_wait_vram_transfer_timeout": [vp, i64, i64],
    "lema_mm_is_transfer_complete": [vp, i64, C.POINTER(i32)],
    "lema_mm_synchronize_all": [vp],
    "lema_mm_submit_prefetch_job": [vp, JOB_FN, vp, C.POINTER(i64)],
    "lema_mm_is_prefetch_complete": [vp, i64, C.POINTER(i32)],
    "lema_mm_wait_for_prefetch": [vp, i64],
    "lema_mm_wait_for_prefetch_timeout": [vp, i64, i64],
    "lema_mm_is_layer_in_ram": [vp, i64, C.POINTER(i32)],
    "lema_mm_copy_stream": [vp, C.POINTER(vp)],
}
_RESTYPES = {"lema_last_error": C.c_char_p, "lema_version": C.c_char_p}

# Status codes (enum lema_status).
LEMA_OK = 0
LEMA_ERR_INVALID_ARGUMENT = 1
LEMA_ERR_MISALIGNED = 2
LEMA_ERR_UNSUPPORTED = 3
LEMA_ERR_CUDA = 4
LEMA_ERR_NOT_REGISTERED = 5
LEMA_ERR_OVERFLOW = 6
LEMA_ERR_TIMEOUT = 7
LEMA_ERR_DEVICE = 8


class LemaError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, code: int, message: str, call: str = ""):
        self.code = code
        super().__init__(f"{call}: [{code}] {message}" if call else f"[{code}] {message}")


def lib() -> C.CDLL:
    """Loads the native library once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"lema_b200 native library not found at {LIB_PATH}; "
                    "build it with `python -m lema_b200.build` (needs nvcc)")
            handle = C.CDLL(str(LIB_PATH))
            for name, args in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = handle
    return _lib


def last_error() -> str:
    return lib().lema_last_error().decode()


# Kernels each entry point launches (the checkpoint save launches one only in
# its SM-store mode 1; its copy-engine mode and the restore launch none).
KERNELS_PER_CALL = {
    "lema_quantize_rows": 1, "lema_quantize_rows_f32": 1, "lema_quantize_per_token": 1,
    "lema_w8a8_gemm": 1, "lema_w8a8_linear_fwd": 2, "lema_w8a8_linear_fwd_noalloc": 2,
    "lema_dequant_transpose": 1, "lema_bf16_gemm_tn": 1, "lema_bf16_gemm_tn_f32": 1,
    "lema_w8a8_dgrad": 2, "lema_grouped_w8a8_gemm": 1, "lema_grouped_bf16_gemm_tn": 1,
    "lema_quantize_rows_colscaled": 1, "lema_transpose_i8": 1, "lema_w8a8_dgrad_int8": 3,
    "lema_grouped_w8a8_dgrad": 2, "lema_rmsnorm_quant": 1, "lema_rmsnorm_bwd": 1,
    "lema_rope": 1, "lema_rope_qkv": 1, "lema_swiglu_quant": 1, "lema_swiglu_bwd": 1,
    "lema_adamw_requant_rows": 1, "lema_device_error_async": 1, "lema_attn_fwd": 1,
    "lema_attn_bwd": 3,
}
# Running count of this library's kernel launches issued by this process.
kernel_launches = 0


def call(name: str, *args) -> None:
    """Invokes a status-returning entry point and raises LemaError on failure."""
    global kernel_launches
    rc = getattr(lib(), name)(*args)
    if rc != LEMA_OK:
        raise LemaError(rc, last_error(), name)
    if name == "lema_ckpt_save":
        kernel_launches += 1 if args[3] == 1 else 0
    else:
        kernel_launches += KERNELS_PER_CALL.get(name, 0)


def version() -> str:
    return lib().lema_version().decode()


def device_error() -> int:
    """Synchronises the current device and returns (and clears) its device error word."""
    out = i32(0)
    call("lema_device_error", C.byref(out))
    return out.value


def num_sms() -> int:
    out = i32(0)
    call("lema_num_sms", C.byref(out))
    return out.value


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def gemm_workspace_count() -> int:
    """(device, stream) stream-K workspaces the library has allocated."""
    out = i64(0)
    call("lema_gemm_workspace_count", C.byref(out))
    return out.value


def gemm_set_test_hooks(skip_publish: bool = False, wait_budget_cycles: int = 0) -> None:
    """Test hooks of the GEMMs' bounded waits (0 cycles = the default budget)."""
    call("lema_gemm_set_test_hooks", int(bool(skip_publish)), int(wait_budget_cycles))


DEVICE_ERROR_NAMES = {
    0x101: "a GEMM's TMA producer timed out waiting for a free stage",
    0x102: "a GEMM's MMA issuer timed out waiting for operands or accumulators",
    0x103: "a GEMM's epilogue timed out waiting for accumulators",
    0x104: "a split GEMM tile's partial accumulators never arrived",
    0x105: "an attention kernel timed out waiting for a tile, a score buffer or P",
}


class DeviceErrorWatch:
    """Watches the library's device error word across training steps without a
    host synchronisation: ``arm(stream)`` enqueues a one-thread kernel that
    moves a nonzero word into a pinned host int (``lema_device_error_async``);
    ``check()`` reads that int on the host and raises ``LemaError`` when a
    kernel recorded a failure (a bounded wait that ran out leaves a wrong
    tile behind, so the step's results must not be used)."""

    def __init__(self, host=None):
        import torch
        self.host = host if host is not None else torch.zeros(1, dtype=torch.int32).pin_memory()

    def arm(self, stream) -> None:
        call("lema_device_error_async", self.host.data_ptr(), stream)

    def check(self) -> None:
        code = int(self.host[0])
        if code:
            self.host[0] = 0
            what = DEVICE_ERROR_NAMES.get(code, "a kernel recorded a device-side failure")
            raise LemaError(LEMA_ERR_DEVICE,
                            f"device error 0x{code:x}: {what}; the last step's results are "
                            "invalid", "train_step")
