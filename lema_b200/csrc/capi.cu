// capi.cu — error reporting, device queries and K5 (boundary-activation
// checkpoint save / restore between device memory and pinned host slots).
#include <algorithm>
#include <mutex>
#include <string>

#include "internal.h"

namespace lema {

namespace {
thread_local std::string t_last_error;
}

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

void clear_error() { t_last_error.clear(); }

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LEMA_OK;
  (void)cudaGetLastError();  // clear the sticky-less error state for the next call
  return set_error(LEMA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int device_sm_count() {
  static int cache[64] = {};
  const int d = current_device();
  if (d < 0 || d >= 64) return 148;
  if (cache[d] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0)
      n = 148;
    cache[d] = n;
  }
  return cache[d];
}

namespace {

// Zero-copy store of device bytes into mapped pinned host memory, 16 bytes
// per thread per iteration; a scalar head/tail covers unaligned ends.
__global__ void ckpt_store_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                  size_t bytes) {
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t nvec = bytes / 16;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (size_t i = tid; i < nvec; i += stride) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(s4 + i));
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(d4 + i), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
  for (size_t i = nvec * 16 + tid; i < bytes; i += stride) dst[i] = src[i];
}

}  // namespace

}  // namespace lema

using namespace lema;

extern "C" const char* lema_last_error(void) { return t_last_error.c_str(); }

extern "C" const char* lema_version(void) { return "lema_b200 0.1.0 sm_100a"; }

extern "C" int lema_device_error(int32_t* code_out) {
  clear_error();
  if (code_out == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null code_out");
  LEMA_CUDA_TRY(cudaDeviceSynchronize());
  int32_t a = 0, b = 0;
  int rc = gemm_read_device_error(&a);
  if (rc) return rc;
  rc = quant_read_device_error(&b);
  if (rc) return rc;
  *code_out = a ? a : b;
  return LEMA_OK;
}

extern "C" int lema_num_sms(int32_t* out) {
  clear_error();
  if (out == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null out");
  *out = device_sm_count();
  return LEMA_OK;
}

extern "C" int lema_ckpt_save(const void* src, void* pinned_dst, size_t bytes, int32_t mode,
                              void* copy_stream, void* after_event, void* done_event) {
  clear_error();
  if (bytes == 0) return LEMA_OK;
  if (src == nullptr || pinned_dst == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  auto s = static_cast<cudaStream_t>(copy_stream);
  if (after_event) LEMA_CUDA_TRY(cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(after_event), 0));
  if (mode == 0) {
    LEMA_CUDA_TRY(cudaMemcpyAsync(pinned_dst, src, bytes, cudaMemcpyDeviceToHost, s));
  } else if (mode == 1) {
    // The destination must be page-locked host memory mapped into the device
    // address space; anything else is rejected before a kernel touches it.
    cudaPointerAttributes attr;
    LEMA_CUDA_TRY(cudaPointerGetAttributes(&attr, pinned_dst));
    if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr)
      return set_error(LEMA_ERR_INVALID_ARGUMENT,
                       "mode 1 needs pinned (cudaHostAlloc / pin_memory) host memory");
    cudaPointerAttributes sattr;
    LEMA_CUDA_TRY(cudaPointerGetAttributes(&sattr, src));
    if (sattr.type != cudaMemoryTypeDevice)
      return set_error(LEMA_ERR_INVALID_ARGUMENT, "mode 1 needs a device source pointer");
    const int grid = std::max(1, std::min(2 * device_sm_count(),
                                          static_cast<int>((bytes / 16 + 255) / 256)));
    ckpt_store_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(src),
                                           static_cast<uint8_t*>(attr.devicePointer), bytes);
    LEMA_CUDA_TRY(cudaGetLastError());
  } else {
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "mode must be 0 (copy engine) or 1 (kernel)");
  }
  if (done_event) LEMA_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(done_event), s));
  return LEMA_OK;
}

extern "C" int lema_ckpt_restore(const void* pinned_src, void* dst, size_t bytes,
                                 void* copy_stream, void* after_event, void* done_event) {
  clear_error();
  if (bytes == 0) return LEMA_OK;
  if (pinned_src == nullptr || dst == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  auto s = static_cast<cudaStream_t>(copy_stream);
  if (after_event) LEMA_CUDA_TRY(cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(after_event), 0));
  LEMA_CUDA_TRY(cudaMemcpyAsync(dst, pinned_src, bytes, cudaMemcpyHostToDevice, s));
  if (done_event) LEMA_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(done_event), s));
  return LEMA_OK;
}
