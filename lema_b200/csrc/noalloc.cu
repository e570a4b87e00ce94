// noalloc.cu — an allocation-free variant of the W8A8 forward (K1 + K2/K3).
//
// lema_w8a8_linear_fwd needs a workspace for the quantised activations (int8
// [M, ldq]) and their per-token scales (fp32 [M]), and its callers allocate
// it. Some callers cannot: a host program that binds this C ABI from a
// language runtime with no CUDA allocator of its own, or a training process
// whose device memory is owned by a framework's caching allocator under a
// fixed VRAM budget (LEMA's per-kind TensorStore budgets), where a raw
// cudaMalloc would go around the budget's accounting and synchronise the
// device. lema_w8a8_linear_fwd_noalloc takes only the inputs and the output
// and keeps its workspace in fixed device arrays of this library.
//
// Limits and behaviour:
//   * the workspace is a file-scope __device__ array of 16 MiB for the int8
//     activations plus 65536 fp32 row scales (256 KiB); every GPU that loads
//     this library holds both until the process exits;
//   * M * round_up(K, 16) must be <= 16 MiB and M <= 65536, else the call
//     returns LEMA_ERR_UNSUPPORTED and nothing is launched;
//   * the first call on a device resolves the arrays' device addresses
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture on the device;
//   * every call on a device shares the same arrays and leaves the last
//     call's quantised activations in them. Nothing in them needs to start at
//     zero: each call rewrites rows [0, M) x columns [0, K) before reading
//     them, and the GEMM never reads the padding columns. Calls whose kernels
//     overlap on the GPU (different streams, or different host threads with
//     no ordering between them) race on the arrays and must be serialised by
//     the caller.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#include <algorithm>
#include <mutex>

#include "internal.h"

namespace {

constexpr size_t kNoallocXqBytes = size_t(16) << 20;
constexpr int64_t kNoallocMaxRows = 65536;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int8_t g_noalloc_xq[kNoallocXqBytes];
static __device__ __align__(256) float g_noalloc_sx[kNoallocMaxRows];

struct NoallocScratch {
  int8_t* xq = nullptr;
  float* sx = nullptr;
};

std::mutex g_noalloc_mu;
NoallocScratch g_noalloc_dev[kMaxDevices];

// Device addresses of the two arrays on the current device, resolved once per
// device. In host code the array names are host-side stand-ins, not device
// addresses, so the addresses must come from cudaGetSymbolAddress.
int noalloc_scratch(NoallocScratch* out) {
  const int dev = lema::current_device();
  if (dev < 0 || dev >= kMaxDevices)
    return lema::set_error(LEMA_ERR_CUDA, "no current CUDA device (or device index >= 64)");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocScratch& s = g_noalloc_dev[dev];
  if (s.xq == nullptr || s.sx == nullptr) {
    void* xq = nullptr;
    void* sx = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&xq, g_noalloc_xq);
    if (e != cudaSuccess) return lema::cuda_check(e, "cudaGetSymbolAddress(noalloc xq)");
    e = cudaGetSymbolAddress(&sx, g_noalloc_sx);
    if (e != cudaSuccess) return lema::cuda_check(e, "cudaGetSymbolAddress(noalloc sx)");
    s.xq = static_cast<int8_t*>(xq);
    s.sx = static_cast<float*>(sx);
  }
  *out = s;
  return LEMA_OK;
}

}  // namespace

extern "C" int lema_w8a8_linear_fwd_noalloc(const void* x_bf16, int64_t ldx, const int8_t* wq,
                                            int64_t ldw, const float* sw, const void* bias_bf16,
                                            void* y_bf16, int64_t ldy, int64_t M, int64_t N,
                                            int64_t K, void* stream) {
  lema::clear_error();
  if (M < 0 || N < 0 || K < 0) return lema::set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (M > kNoallocMaxRows)
    return lema::set_error(LEMA_ERR_UNSUPPORTED,
                           "lema_w8a8_linear_fwd_noalloc: M = " + std::to_string(M) +
                               " rows exceeds the fixed workspace limit of 65536 rows");
  // K is checked before it is rounded up, and the product is never formed, so
  // no size can overflow past the check.
  const int64_t limit = static_cast<int64_t>(kNoallocXqBytes);
  if (K > limit)
    return lema::set_error(LEMA_ERR_UNSUPPORTED,
                           "lema_w8a8_linear_fwd_noalloc: K = " + std::to_string(K) +
                               " exceeds the fixed 16 MiB activation workspace");
  const int64_t ldq = K > 0 ? (K + 15) / 16 * 16 : 16;
  if (ldq > limit / std::max<int64_t>(M, 1))
    return lema::set_error(LEMA_ERR_UNSUPPORTED,
                           "lema_w8a8_linear_fwd_noalloc: M = " + std::to_string(M) +
                               " rows of round_up(K, 16) = " + std::to_string(ldq) +
                               " bytes exceed the fixed 16 MiB activation workspace");
  NoallocScratch s;
  int rc = noalloc_scratch(&s);
  if (rc) return rc;
  // every GEMM tile runs whole: the split-K tail's per-stream workspace would
  // be a device allocation
  lema::ScopedNoGemmWorkspace no_workspace;
  return lema_w8a8_linear_fwd(x_bf16, ldx, wq, ldw, sw, bias_bf16, y_bf16, ldy, s.xq, ldq, s.sx,
                              M, N, K, stream);
}
