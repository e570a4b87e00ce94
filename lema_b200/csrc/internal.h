// internal.h — host-side helpers shared by the C-ABI translation units:
// thread-local error messages, argument checks, device properties.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/lema_b200.h"

namespace lema {

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();

// Wraps a CUDA runtime call: on failure records "<what>: <cuda message>".
int cuda_check(cudaError_t e, const char* what);

// SM count of the current device (cached per device).
int device_sm_count();
int current_device();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-translation-unit device error words: each .cu that launches kernels with
// bounded waits exposes a reader that fetches and clears its word.
int gemm_read_device_error(int32_t* out);
// Device address of the GEMM's error word (also used by the attention kernels),
// or null when it cannot be resolved on the current device.
int32_t* gemm_error_word();
int quant_read_device_error(int32_t* out);

// Device-side error codes written into the error words.
enum DeviceErr : int32_t {
  kDevErrNone = 0,
  kDevErrProducerTimeout = 0x101,
  kDevErrMmaTimeout = 0x102,
  kDevErrEpilogueTimeout = 0x103,
  kDevErrSplitTimeout = 0x104,  // a split tile's partial accumulators never arrived
  kDevErrAttnTimeout = 0x105,   // an attention kernel's wait ran out
};

// While alive, GEMMs issued by this thread run every tile whole (no split-K
// tail, so no workspace is allocated): the allocation-free entry point.
struct ScopedNoGemmWorkspace {
  ScopedNoGemmWorkspace();
  ~ScopedNoGemmWorkspace();
  bool prev;
};

}  // namespace lema

#define LEMA_CUDA_TRY(expr)                                   \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::lema::cuda_check(_e, #expr); \
  } while (0)
