// adamw.cu — the optimizer step of one trainable W8A8 projection under
// selective full fine-tuning, fused with the re-quantisation of its new weight.
//
// Per element, the reference's per-layer AdamW (src/lema/_full_ft.py:204-229:
// decoupled weight decay, bias-corrected moments, the update in fp32, the
// weight stored back in the model dtype), each fp32 operation rounded once in
// this order:
//   w  = f32(w_bf16) * decay                       decay = f32(1 - lr * wd)
//   m  = m * beta1 + g * c1                        c1 = f32(1 - beta1)
//   v  = v * beta2 + (g * g) * c2                  c2 = f32(1 - beta2)
//   d  = sqrt(v) / sqrt_bc2 + eps                  sqrt_bc2 = f32(sqrt(1 - beta2^t))
//   w' = bf16_rne(w + step_size * (m / d))         step_size = f32(-lr / (1 - beta1^t))
// then the row of w' is quantised per output channel by the K1 contract
// (quant_core.cuh) into the int8 row and scale that the streamed segment holds,
// and the gradient accumulator is optionally cleared.
//
// One CTA of 256 threads per weight row. Pass 1 reads w, g, m, v once (16-byte
// vectors when aligned), writes w', m, v (and zeros into g) and reduces |w'|;
// pass 2 re-reads each thread's own w' (L2) and writes the int8 row. HBM-bound:
// 2 + 4 + 8 bytes in, 2 + 8 (+ 4) + 1 bytes out per element.
#include <cuda_bf16.h>

#include "internal.h"
#include "quant_core.cuh"

namespace lema {
namespace {

constexpr int kAThreads = 256;

struct AdamWCoef {
  float decay, beta1, c1, beta2, c2, sqrt_bc2, step_size, eps;
};

__device__ __forceinline__ float adamw_elem(float w, float g, float& m, float& v,
                                            const AdamWCoef& k) {
  w = __fmul_rn(w, k.decay);
  m = __fadd_rn(__fmul_rn(m, k.beta1), __fmul_rn(g, k.c1));
  v = __fadd_rn(__fmul_rn(v, k.beta2), __fmul_rn(__fmul_rn(g, g), k.c2));
  const float d = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), k.sqrt_bc2), k.eps);
  return __fadd_rn(w, __fmul_rn(k.step_size, __fdiv_rn(m, d)));
}

__device__ __forceinline__ float adamw_block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kAThreads / 32; ++w) r = fmaxf(r, red[w]);
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat16 a = __float2bfloat16_rn(lo), b = __float2bfloat16_rn(hi);
  return static_cast<uint32_t>(__bfloat16_as_ushort(a)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
}

// VEC: cols % 8 == 0, 16-byte aligned rows of w, g, m, v and 8-byte aligned q rows.
template <bool VEC>
__global__ void __launch_bounds__(kAThreads) adamw_requant_rows_kernel(
    __nv_bfloat16* __restrict__ w, int64_t ldw, float* __restrict__ g, int64_t ldg,
    float* __restrict__ m, float* __restrict__ v, int64_t ldmv, int64_t cols, AdamWCoef k,
    int zero_grad, int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale) {
  __shared__ float red[kAThreads / 32];
  const int64_t row = blockIdx.x;
  __nv_bfloat16* wr = w + row * ldw;
  float* gr = g + row * ldg;
  float* mr = m + row * ldmv;
  float* vr = v + row * ldmv;
  int8_t* qr = q + row * ldq;
  float amax = 0.f;
  if (VEC) {
    const int64_t nvec = cols / 8;
    for (int64_t i = threadIdx.x; i < nvec; i += kAThreads) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + 8 * i);
      float4* g4 = reinterpret_cast<float4*>(gr + 8 * i);
      float4* m4 = reinterpret_cast<float4*>(mr + 8 * i);
      float4* v4 = reinterpret_cast<float4*>(vr + 8 * i);
      const float4 g0 = g4[0], g1 = g4[1];
      float4 m0 = m4[0], m1 = m4[1], v0 = v4[0], v1 = v4[1];
      const float wf[8] = {bf16_lo(wv.x), bf16_hi(wv.x), bf16_lo(wv.y), bf16_hi(wv.y),
                           bf16_lo(wv.z), bf16_hi(wv.z), bf16_lo(wv.w), bf16_hi(wv.w)};
      const float gf[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      float mf[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      float vf[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      float nw[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) nw[j] = adamw_elem(wf[j], gf[j], mf[j], vf[j], k);
      uint4 out;
      out.x = pack_bf16x2(nw[0], nw[1]);
      out.y = pack_bf16x2(nw[2], nw[3]);
      out.z = pack_bf16x2(nw[4], nw[5]);
      out.w = pack_bf16x2(nw[6], nw[7]);
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(bf16_lo(out.x)), fabsf(bf16_hi(out.x))),
                               fmaxf(fabsf(bf16_lo(out.y)), fabsf(bf16_hi(out.y)))));
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(bf16_lo(out.z)), fabsf(bf16_hi(out.z))),
                               fmaxf(fabsf(bf16_lo(out.w)), fabsf(bf16_hi(out.w)))));
      *reinterpret_cast<uint4*>(wr + 8 * i) = out;
      m4[0] = make_float4(mf[0], mf[1], mf[2], mf[3]);
      m4[1] = make_float4(mf[4], mf[5], mf[6], mf[7]);
      v4[0] = make_float4(vf[0], vf[1], vf[2], vf[3]);
      v4[1] = make_float4(vf[4], vf[5], vf[6], vf[7]);
      if (zero_grad) {
        g4[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        g4[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += kAThreads) {
      float mc = mr[c], vc = vr[c];
      const float nw = adamw_elem(__bfloat162float(wr[c]), gr[c], mc, vc, k);
      const __nv_bfloat16 b = __float2bfloat16_rn(nw);
      amax = fmaxf(amax, fabsf(__bfloat162float(b)));
      wr[c] = b;
      mr[c] = mc;
      vr[c] = vc;
      if (zero_grad) gr[c] = 0.f;
    }
  }
  amax = adamw_block_max(amax, red);
  const float s = quant_row_scale(amax);
  const float inv_s = quant_row_inv_scale(s);
  // each thread quantises the elements it wrote above (its own stores: no barrier)
  if (VEC) {
    const int64_t nvec = cols / 8;
    for (int64_t i = threadIdx.x; i < nvec; i += kAThreads) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + 8 * i);
      *reinterpret_cast<uint2*>(qr + 8 * i) = quant8_bf16(wv, s, inv_s);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += kAThreads)
      qr[c] = static_cast<int8_t>(quant_exact(__bfloat162float(wr[c]), s));
  }
  if (threadIdx.x == 0) scale[row] = s;
}

}  // namespace
}  // namespace lema

using namespace lema;

extern "C" int lema_adamw_requant_rows(void* w_bf16, int64_t ldw, float* g, int64_t ldg,
                                       float* m, float* v, int64_t ldmv, int64_t rows,
                                       int64_t cols, float decay, float beta1, float c1,
                                       float beta2, float c2, float sqrt_bc2, float step_size,
                                       float eps, int32_t zero_grad, int8_t* q, int64_t ldq,
                                       float* scale, void* stream) {
  clear_error();
  if (rows < 0 || cols < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0) return LEMA_OK;
  if (w_bf16 == nullptr || g == nullptr || m == nullptr || v == nullptr || q == nullptr ||
      scale == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldw < cols || ldg < cols || ldmv < cols || ldq < cols)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "leading dimension < cols");
  if (rows > INT32_MAX) return set_error(LEMA_ERR_UNSUPPORTED, "rows exceed 2^31-1");
  auto* w = static_cast<__nv_bfloat16*>(w_bf16);
  const AdamWCoef k{decay, beta1, c1, beta2, c2, sqrt_bc2, step_size, eps};
  const bool vec = cols % 8 == 0 && aligned16(w) && (ldw * 2) % 16 == 0 && aligned16(g) &&
                   (ldg * 4) % 16 == 0 && aligned16(m) && aligned16(v) && (ldmv * 4) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(q) % 8) == 0 && ldq % 8 == 0;
  const dim3 grid(static_cast<unsigned>(rows));
  const auto s = static_cast<cudaStream_t>(stream);
  if (vec)
    adamw_requant_rows_kernel<true><<<grid, kAThreads, 0, s>>>(w, ldw, g, ldg, m, v, ldmv, cols,
                                                               k, zero_grad, q, ldq, scale);
  else
    adamw_requant_rows_kernel<false><<<grid, kAThreads, 0, s>>>(w, ldw, g, ldg, m, v, ldmv,
                                                                cols, k, zero_grad, q, ldq,
                                                                scale);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}
