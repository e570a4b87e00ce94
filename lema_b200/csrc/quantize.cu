// quantize.cu — K1: per-row dynamic symmetric int8 quantisation (per token for
// activations, per output channel for weights), the int8 -> bf16 dequant +
// transpose that feeds the dgrad GEMM, and the C-ABI front ends that chain
// K1 -> K2/K3 (forward) and dequant -> bf16 GEMM (dgrad). The opt-in int8-dy
// dgrad chains a column-scaled quantiser (rows of dy * sw), an int8 transpose
// of wq and the int8 GEMM with unit column scales.
//
// K1 is HBM-bound: one CTA of 128 threads owns one row, reads it once with
// 128-bit loads into registers (up to 16 vectors per thread = 16384 bf16),
// reduces |x| with warp shuffles + a 4-entry shared array, then quantises from
// registers and writes int8 with 64-bit stores. For 4096-column rows twelve
// such CTAs fit an SM (~100 KB of loads in flight per SM). Rows longer than the
// register budget, unaligned rows and ragged column counts take a two-pass
// scalar path. The result is the operator contract's: rint (half to even) of
// the IEEE fp32 quotient x / s, clamped to [-127, 127]; the element arithmetic
// is in quant_core.cuh (reciprocal product, exact division near ties).
#include <cuda_bf16.h>

#include <algorithm>

#include "internal.h"
#include "quant_core.cuh"

namespace lema {

extern "C" int lema_w8a8_gemm(const int8_t*, int64_t, const float*, const int8_t*, int64_t,
                              const float*, const void*, void*, int64_t, int32_t*, int64_t,
                              int64_t, int64_t, int64_t, void*);
extern "C" int lema_bf16_gemm_tn(const void*, int64_t, const void*, int64_t, void*, int64_t,
                                 int64_t, int64_t, int64_t, void*);
extern "C" int lema_grouped_bf16_gemm_tn(const void*, int64_t, const void*, int64_t, void*,
                                         int64_t, const int64_t*, int32_t, int64_t, int64_t,
                                         void*);

namespace {

constexpr int kQThreads = 128;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Max over the CTA (128 threads = 4 warps); every thread gets the result.
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  return r;
}

template <typename T>
struct Vec;
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int kElems = 8;  // 8 x bf16 per 16-byte vector
  __device__ static float absmax(const uint4& v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    __nv_bfloat162 m = __hmax2(__habs2(h[0]), __habs2(h[1]));
    m = __hmax2(m, __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__bfloat162float(m.x), __bfloat162float(m.y));
  }
  // 8 int8 packed little-endian
  __device__ static uint2 quant(const uint4& v, float s, float inv_s) {
    return quant8_bf16(v, s, inv_s);
  }
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
};
template <>
struct Vec<float> {
  static constexpr int kElems = 4;
  __device__ static float absmax(const uint4& v) {
    return fmaxf(fmaxf(fabsf(__uint_as_float(v.x)), fabsf(__uint_as_float(v.y))),
                 fmaxf(fabsf(__uint_as_float(v.z)), fabsf(__uint_as_float(v.w))));
  }
  // 4 int8 packed little-endian
  __device__ static uint32_t quant(const uint4& v, float s, float inv_s) {
    return quant4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z),
                  __uint_as_float(v.w), s, inv_s);
  }
  __device__ static float to_f(float x) { return x; }
};

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Register-resident path: cols % kElems == 0, 16-byte aligned rows, and
// cols <= VPT * 128 * kElems.
template <typename T, int VPT>
__global__ void __launch_bounds__(kQThreads) quant_rows_vec_kernel(const T* __restrict__ x,
                                                                   int64_t ldx, int cols,
                                                                   int8_t* __restrict__ q,
                                                                   int64_t ldq,
                                                                   float* __restrict__ scale) {
  constexpr int E = Vec<T>::kElems;
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const int nvec = cols / E;
  uint4 v[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kQThreads;
    v[i] = idx < nvec ? ld_stream(xr + idx) : make_uint4(0u, 0u, 0u, 0u);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i)
    if (threadIdx.x + i * kQThreads < nvec) amax = fmaxf(amax, Vec<T>::absmax(v[i]));
  amax = block_max(amax, red);
  const float s = quant_row_scale(amax);
  const float inv_s = quant_row_inv_scale(s);
  int8_t* qr = q + row * ldq;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kQThreads;
    if (idx < nvec)
      *reinterpret_cast<decltype(Vec<T>::quant(v[i], s, inv_s))*>(
          qr + static_cast<int64_t>(idx) * E) = Vec<T>::quant(v[i], s, inv_s);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// Max over a CTA of W warps (called once per CTA); every thread gets the result.
template <int W>
__device__ __forceinline__ float block_max_w(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < W; ++w) r = fmaxf(r, red[w]);
  return r;
}

// Rows of x[r, c] * cs[c] (bf16 x, fp32 column scales; each product rounded to
// fp32) quantised by the contract: one CTA of THREADS threads per row, the row
// held as bf16 vectors (VPT 16-byte vectors per thread, loads issued before
// use), the products formed twice (for |max| and for the quantiser), the
// scales read through L1. THREADS grows with the row so that VPT stays <= 6
// (rows up to 24576 columns at 512 threads).
template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS) quant_rows_colscaled_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const float* __restrict__ cs, int cols,
    int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale) {
  __shared__ float red[THREADS / 32];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const float4* cs4 = reinterpret_cast<const float4*>(cs);
  const int nvec = cols / 8;
  uint4 v[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * THREADS;
    if (idx < nvec) v[i] = ld_stream(xr + idx);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * THREADS;
    if (idx < nvec) {
      const float4 c0 = __ldg(cs4 + 2 * idx), c1 = __ldg(cs4 + 2 * idx + 1);
      const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        amax = fmaxf(amax, fabsf(__fmul_rn(bf16_lo(w[j]), c[2 * j])));
        amax = fmaxf(amax, fabsf(__fmul_rn(bf16_hi(w[j]), c[2 * j + 1])));
      }
    }
  }
  amax = block_max_w<THREADS / 32>(amax, red);
  const float s = quant_row_scale(amax);
  const float inv_s = quant_row_inv_scale(s);
  int8_t* qr = q + row * ldq;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * THREADS;
    if (idx < nvec) {
      const float4 c0 = __ldg(cs4 + 2 * idx), c1 = __ldg(cs4 + 2 * idx + 1);
      const float f[8] = {__fmul_rn(bf16_lo(v[i].x), c0.x), __fmul_rn(bf16_hi(v[i].x), c0.y),
                          __fmul_rn(bf16_lo(v[i].y), c0.z), __fmul_rn(bf16_hi(v[i].y), c0.w),
                          __fmul_rn(bf16_lo(v[i].z), c1.x), __fmul_rn(bf16_hi(v[i].z), c1.y),
                          __fmul_rn(bf16_lo(v[i].w), c1.z), __fmul_rn(bf16_hi(v[i].w), c1.w)};
      *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(idx) * 8) = quant8(f, s, inv_s);
    }
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// Any alignment / length: two passes over the row, exact division.
__global__ void __launch_bounds__(kQThreads) quant_rows_colscaled_generic_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const float* __restrict__ cs,
    int64_t cols, int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale) {
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  float amax = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += kQThreads)
    amax = fmaxf(amax, fabsf(__fmul_rn(__bfloat162float(xr[c]), cs[c])));
  amax = block_max(amax, red);
  const float s = quant_row_scale(amax);
  int8_t* qr = q + row * ldq;
  for (int64_t c = threadIdx.x; c < cols; c += kQThreads)
    qr[c] = static_cast<int8_t>(quant_exact(__fmul_rn(__bfloat162float(xr[c]), cs[c]), s));
  if (threadIdx.x == 0) scale[row] = s;
}

// wqT[k, n] = wq[n, k] in 128 (n) x 128 (k) tiles, 256 threads. Each thread
// loads 16 bytes along k from four consecutive rows (4 x 16 bytes), transposes
// the 4 x 16 block in registers with byte permutes into 16 words of four
// n-values, and stores them as 32-bit words to tile[k][n / 4] (a warp covers
// one k row: 32 distinct banks). Then each quarter-warp copies one 128-byte
// k row of the tile to wqT with 16-byte loads and stores.
constexpr int kTT = 128;
__global__ void __launch_bounds__(256) transpose_i8_kernel(const int8_t* __restrict__ wq,
                                                           int64_t ldw, int64_t n_rows,
                                                           int64_t k_cols,
                                                           int8_t* __restrict__ out, int64_t ldt,
                                                           bool vec_in, bool vec_out) {
  __shared__ __align__(16) uint32_t tile[kTT][kTT / 4];
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kTT;
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * kTT;
  const int g = threadIdx.x & 31, b = threadIdx.x >> 5;  // rows 4g..4g+3, k 16b..16b+15
  const int64_t kb = k0 + 16 * b;
  uint32_t w[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t n = n0 + 4 * g + r;
    if (vec_in && n < n_rows && kb + 16 <= k_cols) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(wq + n * ldw + kb));
      w[r][0] = v.x;
      w[r][1] = v.y;
      w[r][2] = v.z;
      w[r][3] = v.w;
    } else {
      uint32_t t[4] = {0u, 0u, 0u, 0u};
      for (int j = 0; j < 16; ++j)
        if (n < n_rows && kb + j < k_cols)
          t[j >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(wq[n * ldw + kb + j]))
                       << (8 * (j & 3));
#pragma unroll
      for (int m = 0; m < 4; ++m) w[r][m] = t[m];
    }
  }
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    // bytes e of rows 0..3 -> word (a_e, b_e, c_e, d_e), little-endian
    const uint32_t ab_lo = __byte_perm(w[0][m], w[1][m], 0x5140);
    const uint32_t ab_hi = __byte_perm(w[0][m], w[1][m], 0x7362);
    const uint32_t cd_lo = __byte_perm(w[2][m], w[3][m], 0x5140);
    const uint32_t cd_hi = __byte_perm(w[2][m], w[3][m], 0x7362);
    const int row = 16 * b + 4 * m;
    tile[row + 0][g] = __byte_perm(ab_lo, cd_lo, 0x5410);
    tile[row + 1][g] = __byte_perm(ab_lo, cd_lo, 0x7632);
    tile[row + 2][g] = __byte_perm(ab_hi, cd_hi, 0x5410);
    tile[row + 3][g] = __byte_perm(ab_hi, cd_hi, 0x7632);
  }
  __syncthreads();
  const int c = threadIdx.x & 7;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kl = (threadIdx.x >> 3) + 32 * i;
    const int64_t k = k0 + kl;
    const int64_t n = n0 + 16 * c;
    if (k >= k_cols || n >= n_rows) continue;
    int8_t* dst = out + k * ldt + n;
    const uint4 v = *reinterpret_cast<const uint4*>(&tile[kl][4 * c]);
    if (vec_out && n + 16 <= n_rows) {
      *reinterpret_cast<uint4*>(dst) = v;
    } else {
      const uint8_t* bytes = reinterpret_cast<const uint8_t*>(&v);
      for (int j = 0; j < 16 && n + j < n_rows; ++j) dst[j] = static_cast<int8_t>(bytes[j]);
    }
  }
}

// General path: any alignment / length; reads the row twice.
template <typename T>
__global__ void __launch_bounds__(kQThreads) quant_rows_generic_kernel(const T* __restrict__ x,
                                                                       int64_t ldx, int64_t cols,
                                                                       int8_t* __restrict__ q,
                                                                       int64_t ldq,
                                                                       float* __restrict__ scale) {
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  float amax = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += kQThreads)
    amax = fmaxf(amax, fabsf(Vec<T>::to_f(xr[c])));
  amax = block_max(amax, red);
  const float s = quant_row_scale(amax);
  int8_t* qr = q + row * ldq;
  for (int64_t c = threadIdx.x; c < cols; c += kQThreads)
    qr[c] = static_cast<int8_t>(quant_exact(Vec<T>::to_f(xr[c]), s));
  if (threadIdx.x == 0) scale[row] = s;
}

template <typename T>
int quantize_rows_impl(const T* x, int64_t rows, int64_t cols, int64_t ldx, int8_t* q,
                       int64_t ldq, float* scale, cudaStream_t s) {
  clear_error();
  if (rows < 0 || cols < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0) return LEMA_OK;
  if (x == nullptr || q == nullptr || scale == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldx < cols || ldq < cols) return set_error(LEMA_ERR_INVALID_ARGUMENT, "ld < cols");
  if (rows > INT32_MAX) return set_error(LEMA_ERR_UNSUPPORTED, "rows exceed 2^31-1");
  constexpr int E = Vec<T>::kElems;
  const bool vec_ok = cols > 0 && cols % E == 0 && aligned16(x) && (ldx * sizeof(T)) % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(q) % E) == 0 && ldq % E == 0;
  const int64_t per_thread = (cols / E + kQThreads - 1) / kQThreads;
  const dim3 grid(static_cast<unsigned>(rows));
  if (vec_ok && per_thread <= 16) {
    if (per_thread <= 1)
      quant_rows_vec_kernel<T, 1><<<grid, kQThreads, 0, s>>>(x, ldx, (int)cols, q, ldq, scale);
    else if (per_thread <= 2)
      quant_rows_vec_kernel<T, 2><<<grid, kQThreads, 0, s>>>(x, ldx, (int)cols, q, ldq, scale);
    else if (per_thread <= 4)
      quant_rows_vec_kernel<T, 4><<<grid, kQThreads, 0, s>>>(x, ldx, (int)cols, q, ldq, scale);
    else if (per_thread <= 8)
      quant_rows_vec_kernel<T, 8><<<grid, kQThreads, 0, s>>>(x, ldx, (int)cols, q, ldq, scale);
    else if (per_thread <= 12)
      quant_rows_vec_kernel<T, 12><<<grid, kQThreads, 0, s>>>(x, ldx, (int)cols, q, ldq, scale);
    else
      quant_rows_vec_kernel<T, 16><<<grid, kQThreads, 0, s>>>(x, ldx, (int)cols, q, ldq, scale);
  } else {
    quant_rows_generic_kernel<T><<<grid, kQThreads, 0, s>>>(x, ldx, cols, q, ldq, scale);
  }
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

// wdT[k, n] = bf16(float(wq[n, k]) * sw[n]). One CTA transposes a 64 (n) x
// 128 (k) tile through shared memory: 16-byte loads of 16 int8 per thread
// (consecutive threads take consecutive rows, so the shared-memory writes of a
// warp hit consecutive bf16), then 16-byte stores of 8 bf16 along n.
constexpr int kDTN = 64;
constexpr int kDTK = 128;
__global__ void __launch_bounds__(256) dequant_transpose_kernel(const int8_t* __restrict__ wq,
                                                                int64_t ldw,
                                                                const float* __restrict__ sw,
                                                                int64_t n_rows, int64_t k_cols,
                                                                __nv_bfloat16* __restrict__ out,
                                                                int64_t ldt, bool vec_in,
                                                                bool vec_out) {
  __shared__ __align__(16) __nv_bfloat16 tile[kDTK][kDTN + 8];  // [k][n], 144-byte rows
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kDTN;
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * kDTK;
  for (int c = threadIdx.x; c < kDTN * (kDTK / 16); c += 256) {
    const int r = c % kDTN, q = c / kDTN;  // row of the tile, 16-byte chunk along k
    const int64_t n = n0 + r;
    const int64_t kb = k0 + q * 16;
    __align__(16) int8_t v[16];
    if (vec_in && n < n_rows && kb + 16 <= k_cols) {
      *reinterpret_cast<uint4*>(v) =
          __ldg(reinterpret_cast<const uint4*>(wq + n * ldw + kb));
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        v[j] = (n < n_rows && kb + j < k_cols) ? wq[n * ldw + kb + j] : static_cast<int8_t>(0);
    }
    const float s = n < n_rows ? sw[n] : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      tile[q * 16 + j][r] = __float2bfloat16_rn(__fmul_rn(static_cast<float>(v[j]), s));
  }
  __syncthreads();
  for (int c = threadIdx.x; c < kDTK * (kDTN / 8); c += 256) {
    const int r = c / (kDTN / 8), q = c % (kDTN / 8);
    const int64_t k = k0 + r;
    const int64_t n = n0 + q * 8;
    if (k >= k_cols || n >= n_rows) continue;
    __nv_bfloat16* dst = out + k * ldt + n;
    if (vec_out && n + 8 <= n_rows) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&tile[r][q * 8]);
    } else {
      for (int j = 0; j < 8 && n + j < n_rows; ++j) dst[j] = tile[r][q * 8 + j];
    }
  }
}

}  // namespace

int quant_read_device_error(int32_t* out) {
  *out = 0;  // no kernel of this file waits on anything
  return LEMA_OK;
}

}  // namespace lema

using namespace lema;

extern "C" int lema_quantize_rows(const void* x_bf16, int64_t rows, int64_t cols, int64_t ldx,
                                  int8_t* q, int64_t ldq, float* scale, void* stream) {
  return quantize_rows_impl(static_cast<const __nv_bfloat16*>(x_bf16), rows, cols, ldx, q, ldq,
                            scale, static_cast<cudaStream_t>(stream));
}

extern "C" int lema_quantize_rows_f32(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                                      int8_t* q, int64_t ldq, float* scale, void* stream) {
  return quantize_rows_impl(x, rows, cols, ldx, q, ldq, scale, static_cast<cudaStream_t>(stream));
}

extern "C" int lema_quantize_per_token(const void* x_bf16, int64_t M, int64_t K, int64_t ldx,
                                       int8_t* xq, int64_t ldq, float* sx, void* stream) {
  return lema_quantize_rows(x_bf16, M, K, ldx, xq, ldq, sx, stream);
}

extern "C" int lema_w8a8_linear_fwd(const void* x_bf16, int64_t ldx, const int8_t* wq,
                                    int64_t ldw, const float* sw, const void* bias_bf16,
                                    void* y_bf16, int64_t ldy, int8_t* xq_ws, int64_t ldq,
                                    float* sx_ws, int64_t M, int64_t N, int64_t K, void* stream) {
  int rc = lema_quantize_rows(x_bf16, M, K, ldx, xq_ws, ldq, sx_ws, stream);
  if (rc) return rc;
  return lema_w8a8_gemm(xq_ws, ldq, sx_ws, wq, ldw, sw, bias_bf16, y_bf16, ldy, nullptr, 0, M, N,
                        K, stream);
}

extern "C" int lema_dequant_transpose(const int8_t* wq, int64_t ldw, const float* sw, int64_t N,
                                      int64_t K, void* wdT_bf16, int64_t ldt, void* stream) {
  clear_error();
  if (N < 0 || K < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (N == 0 || K == 0) return LEMA_OK;
  if (wq == nullptr || sw == nullptr || wdT_bf16 == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldw < K || ldt < N) return set_error(LEMA_ERR_INVALID_ARGUMENT, "ld too small");
  if ((K + kDTK - 1) / kDTK > INT32_MAX || (N + kDTN - 1) / kDTN > 65535)
    return set_error(LEMA_ERR_UNSUPPORTED, "matrix too large for the transpose grid");
  dim3 grid(static_cast<unsigned>((K + kDTK - 1) / kDTK),
            static_cast<unsigned>((N + kDTN - 1) / kDTN));
  const bool vec_in = aligned16(wq) && ldw % 16 == 0;
  const bool vec_out = aligned16(wdT_bf16) && ldt % 8 == 0;
  dequant_transpose_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      wq, ldw, sw, N, K, static_cast<__nv_bfloat16*>(wdT_bf16), ldt, vec_in, vec_out);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_w8a8_dgrad(const void* dy_bf16, int64_t lddy, const int8_t* wq, int64_t ldw,
                               const float* sw, void* dx_bf16, int64_t lddx, void* wdT_ws,
                               int64_t ldt, int64_t M, int64_t N, int64_t K, void* stream) {
  clear_error();
  if (ldt < N || ldt % 8 != 0)
    return set_error(LEMA_ERR_MISALIGNED, "workspace ld must be >= N and a multiple of 8");
  int rc = lema_dequant_transpose(wq, ldw, sw, N, K, wdT_ws, ldt, stream);
  if (rc) return rc;
  // dx[M, K] = dy[M, N] . wdT[K, N]^T
  return lema_bf16_gemm_tn(dy_bf16, lddy, wdT_ws, ldt, dx_bf16, lddx, M, K, N, stream);
}

extern "C" int lema_grouped_w8a8_dgrad(const void* dy_bf16, int64_t lddy, const int8_t* wq,
                                       int64_t ldw, const float* sw, void* dx_bf16,
                                       int64_t lddx, void* wdT_ws, int64_t ldt,
                                       const int64_t* offsets_host, int32_t E, int64_t N,
                                       int64_t K, void* stream) {
  clear_error();
  if (ldt < N || ldt % 8 != 0)
    return set_error(LEMA_ERR_MISALIGNED, "workspace ld must be >= N and a multiple of 8");
  if (offsets_host == nullptr || E <= 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "offsets must hold E+1 entries, E >= 1");
  auto* ws = static_cast<__nv_bfloat16*>(wdT_ws);
  for (int e = 0; e < E; ++e) {
    if (offsets_host[e + 1] == offsets_host[e]) continue;  // expert without tokens
    int rc = lema_dequant_transpose(wq + static_cast<int64_t>(e) * N * ldw, ldw, sw + e * N, N, K,
                                    ws + static_cast<int64_t>(e) * K * ldt, ldt, stream);
    if (rc) return rc;
  }
  // rows of expert e: dx = dy . wdT_e^T, wdT_e = ws[e] ([K, ldt])
  return lema_grouped_bf16_gemm_tn(dy_bf16, lddy, wdT_ws, ldt, dx_bf16, lddx, offsets_host, E,
                                   K, N, stream);
}

extern "C" int lema_quantize_rows_colscaled(const void* x_bf16, const float* cs, int64_t rows,
                                            int64_t cols, int64_t ldx, int8_t* q, int64_t ldq,
                                            float* scale, void* stream) {
  clear_error();
  if (rows < 0 || cols < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0) return LEMA_OK;
  if (x_bf16 == nullptr || cs == nullptr || q == nullptr || scale == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldx < cols || ldq < cols) return set_error(LEMA_ERR_INVALID_ARGUMENT, "ld < cols");
  if (rows > INT32_MAX) return set_error(LEMA_ERR_UNSUPPORTED, "rows exceed 2^31-1");
  const auto* x = static_cast<const __nv_bfloat16*>(x_bf16);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec_ok = cols > 0 && cols % 8 == 0 && aligned16(x) && (ldx * 2) % 16 == 0 &&
                      aligned16(cs) && (reinterpret_cast<uintptr_t>(q) % 8) == 0 && ldq % 8 == 0;
  const int64_t nvec = cols / 8;
  const dim3 grid(static_cast<unsigned>(rows));
  const int c = static_cast<int>(cols);
  if (vec_ok && nvec <= 128 * 2) {
    quant_rows_colscaled_kernel<128, 2><<<grid, 128, 0, s>>>(x, ldx, cs, c, q, ldq, scale);
  } else if (vec_ok && nvec <= 128 * 4) {
    quant_rows_colscaled_kernel<128, 4><<<grid, 128, 0, s>>>(x, ldx, cs, c, q, ldq, scale);
  } else if (vec_ok && nvec <= 256 * 4) {
    quant_rows_colscaled_kernel<256, 4><<<grid, 256, 0, s>>>(x, ldx, cs, c, q, ldq, scale);
  } else if (vec_ok && nvec <= 256 * 6) {
    quant_rows_colscaled_kernel<256, 6><<<grid, 256, 0, s>>>(x, ldx, cs, c, q, ldq, scale);
  } else if (vec_ok && nvec <= 512 * 6) {
    quant_rows_colscaled_kernel<512, 6><<<grid, 512, 0, s>>>(x, ldx, cs, c, q, ldq, scale);
  } else {
    quant_rows_colscaled_generic_kernel<<<grid, kQThreads, 0, s>>>(x, ldx, cs, cols, q, ldq,
                                                                    scale);
  }
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_transpose_i8(const int8_t* wq, int64_t ldw, int64_t N, int64_t K,
                                 int8_t* wqT, int64_t ldt, void* stream) {
  clear_error();
  if (N < 0 || K < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (N == 0 || K == 0) return LEMA_OK;
  if (wq == nullptr || wqT == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldw < K || ldt < N) return set_error(LEMA_ERR_INVALID_ARGUMENT, "ld too small");
  if ((K + kTT - 1) / kTT > INT32_MAX || (N + kTT - 1) / kTT > 65535)
    return set_error(LEMA_ERR_UNSUPPORTED, "matrix too large for the transpose grid");
  dim3 grid(static_cast<unsigned>((K + kTT - 1) / kTT), static_cast<unsigned>((N + kTT - 1) / kTT));
  const bool vec_in = aligned16(wq) && ldw % 16 == 0;
  const bool vec_out = aligned16(wqT) && ldt % 16 == 0;
  transpose_i8_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(wq, ldw, N, K, wqT,
                                                                           ldt, vec_in, vec_out);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_w8a8_dgrad_int8(const void* dy_bf16, int64_t lddy, const int8_t* wq,
                                    int64_t ldw, const float* sw, void* dx_bf16, int64_t lddx,
                                    int8_t* wqT_ws, int64_t ldt, int8_t* dq_ws, int64_t ldq,
                                    float* sd_ws, int64_t M, int64_t N, int64_t K,
                                    void* stream) {
  clear_error();
  if (ldt < N || ldt % 16 != 0 || ldq < N || ldq % 16 != 0)
    return set_error(LEMA_ERR_MISALIGNED, "workspace lds must be >= N and multiples of 16");
  if (sw == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null weight scales");
  int rc = lema_quantize_rows_colscaled(dy_bf16, sw, M, N, lddy, dq_ws, ldq, sd_ws, stream);
  if (rc) return rc;
  rc = lema_transpose_i8(wq, ldw, N, K, wqT_ws, ldt, stream);
  if (rc) return rc;
  // dx[M, K] = bf16(sd[m] * sum_n dq[m, n] * wqT[k, n]) (no column scales)
  return lema_w8a8_gemm(dq_ws, ldq, sd_ws, wqT_ws, ldt, nullptr, nullptr, dx_bf16, lddx, nullptr,
                        0, M, K, N, stream);
}
