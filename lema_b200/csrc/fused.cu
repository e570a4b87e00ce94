// fused.cu — producers that feed the W8A8 GEMMs of a decoder block without
// extra HBM round trips, and their backward kernels:
//
//   rmsnorm_quant   hn = bf16(g * bf16(x * rsqrt(mean(x^2) + eps))) per row
//                   (the rounding sequence of HF LlamaRMSNorm in bf16), plus the
//                   per-row int8 quantisation of hn (the K1 rule) for the
//                   following projections, plus rstd for the backward.
//   rmsnorm_bwd     dx = rstd * (g*dhn - xhat * mean(g*dhn*xhat)), xhat = x*rstd (fp32).
//   rope            out = bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)) per head
//                   (torch's rounding of q*cos + rotate_half(q)*sin in bf16),
//                   reading strided q/k rows and writing contiguous rows; the
//                   backward applies the transposed rotation in fp32.
//   swiglu_quant    m = bf16(bf16(silu(gate)) * up) per row of [gate | up],
//                   quantised per row (K1 rule) for the down projection.
//   swiglu_bwd      d[gate | up] from dm and the saved [gate | up].
//
// All are HBM-bound; one CTA (128 threads) per row keeps the row in registers
// (16-byte vectors) so each input byte is read once.
#include <cuda_bf16.h>

#include "internal.h"
#include "quant_core.cuh"

namespace lema {
namespace {

constexpr int kThreads = 128;

// Block-wide reductions over NW warps (red holds NW floats); every thread gets
// the result. A leading barrier lets two reductions share one red array.
template <int NW = 4>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) r += red[w];
  return r;
}

template <int NW = 4>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) r = fmaxf(r, red[w]);
  return r;
}

__device__ __forceinline__ void row_scale(float amax, float& s, float& inv_s) {
  s = quant_row_scale(amax);
  inv_s = quant_row_inv_scale(s);
}

union V8 {
  uint4 u;
  __nv_bfloat16 h[8];
};

// 16-byte load of data read once (not kept in L1).
__device__ __forceinline__ uint4 ld_stream16(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------- RMSNorm
template <int VPT>
__global__ void __launch_bounds__(kThreads) rmsnorm_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ g,
    int cols, float eps, __nv_bfloat16* __restrict__ hn, int64_t ldh, int8_t* __restrict__ q,
    int64_t ldq, float* __restrict__ scale, float* __restrict__ rstd_out) {
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const int nvec = cols / 8;
  uint4 v[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    v[i] = idx < nvec ? ld_stream16(reinterpret_cast<const uint4*>(x + row * ldx) + idx)
                      : make_uint4(0u, 0u, 0u, 0u);
  }
  // sum of squares in two fp32 lanes (even / odd columns), packed
  uint64_t ss2 = f2_splat(0.f);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const uint64_t a = f2_from_bf16x2(v[i].x), b = f2_from_bf16x2(v[i].y);
    const uint64_t c = f2_from_bf16x2(v[i].z), d = f2_from_bf16x2(v[i].w);
    ss2 = f2_fma(d, d, f2_fma(c, c, f2_fma(b, b, f2_fma(a, a, ss2))));
  }
  float ss_lo, ss_hi;
  f2_unpack(ss2, ss_lo, ss_hi);
  const float ss = block_sum(ss_lo + ss_hi, red);
  const float rstd = rsqrtf(ss / static_cast<float>(cols) + eps);
  const uint64_t rstd2 = f2_splat(rstd);
  // hn = bf16(g * bf16(x * rstd)): the bf16 x bf16 product is exact in fp32, so
  // one bf16x2 multiply rounds it as the fp32 product followed by RN to bf16 does
  __nv_bfloat162 amax2 = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < nvec) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g) + idx);
      uint32_t* w = reinterpret_cast<uint32_t*>(&v[i]);
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t xh = bf16x2_from_f2(f2_mul(f2_from_bf16x2(w[j]), rstd2));
        const __nv_bfloat162 o = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&gw[j]),
                                         *reinterpret_cast<const __nv_bfloat162*>(&xh));
        amax2 = __hmax2(amax2, __habs2(o));
        w[j] = *reinterpret_cast<const uint32_t*>(&o);
      }
      reinterpret_cast<uint4*>(hn + row * ldh)[idx] = v[i];
    }
  }
  if (q != nullptr) {
    const float amax = block_max(
        fmaxf(__bfloat162float(__low2bfloat16(amax2)), __bfloat162float(__high2bfloat16(amax2))),
        red);
    float s, inv_s;
    row_scale(amax, s, inv_s);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      if (idx < nvec)
        *reinterpret_cast<uint2*>(q + row * ldq + static_cast<int64_t>(idx) * 8) =
            quant8_bf16(v[i], s, inv_s);
    }
    if (threadIdx.x == 0) scale[row] = s;
  }
  if (threadIdx.x == 0 && rstd_out != nullptr) rstd_out[row] = rstd;
}

template <int VPT>
__global__ void __launch_bounds__(kThreads) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ g,
    const float* __restrict__ rstd_in, const __nv_bfloat16* __restrict__ dhn, int64_t ldd,
    int cols, __nv_bfloat16* __restrict__ dx, int64_t lddx) {
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const int nvec = cols / 8;
  const float rstd = rstd_in[row];
  V8 xv[VPT], dv[VPT];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < nvec) {
      xv[i].u = __ldg(reinterpret_cast<const uint4*>(x + row * ldx) + idx);
      dv[i].u = __ldg(reinterpret_cast<const uint4*>(dhn + row * ldd) + idx);
      V8 gv;
      gv.u = __ldg(reinterpret_cast<const uint4*>(g) + idx);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float gd = __bfloat162float(gv.h[j]) * __bfloat162float(dv[i].h[j]);
        dot = fmaf(gd, __bfloat162float(xv[i].h[j]) * rstd, dot);
      }
    }
  }
  dot = block_sum(dot, red) / static_cast<float>(cols);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < nvec) {
      V8 gv, out;
      gv.u = __ldg(reinterpret_cast<const uint4*>(g) + idx);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xhat = __bfloat162float(xv[i].h[j]) * rstd;
        const float gd = __bfloat162float(gv.h[j]) * __bfloat162float(dv[i].h[j]);
        out.h[j] = __float2bfloat16_rn(rstd * (gd - xhat * dot));
      }
      reinterpret_cast<uint4*>(dx + row * lddx)[idx] = out.u;
    }
  }
}

// ---------------------------------------------------------------- RoPE
// One thread handles 8 consecutive dims i..i+7 of the first half of one head
// and their partners i+d/2.. of one token. Heads [0, hq) are q, [hq, hq+hk) k,
// [hq+hk, hq+2hk) v (when v_in is given; v is not rotated). An optional addend
// per tensor (contiguous rows, e.g. a LoRA output) is added first with bf16
// rounding, as torch's `t + lora` does. mode 0: forward with torch's bf16
// roundings; mode 1: backward (transposed rotation, fp32, one rounding; addends
// and v are not used).
struct RopeArgs {
  const __nv_bfloat16* in[3];
  int64_t ld[3];
  const __nv_bfloat16* add[3];
  __nv_bfloat16* out[3];
  int heads[3];
};

__global__ void rope_kernel(const __grid_constant__ RopeArgs a,
                            const __nv_bfloat16* __restrict__ cosv,
                            const __nv_bfloat16* __restrict__ sinv, int64_t tokens, int seq,
                            int d, int mode) {
  const int half = d / 2;
  const int groups = half / 8;
  const int htot = a.heads[0] + a.heads[1] + a.heads[2];
  const int per_token = htot * groups;
  const int64_t gid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (gid >= tokens * per_token) return;
  const int64_t t = gid / per_token;
  int r = static_cast<int>(gid % per_token);
  int which = 0;
  while (which < 2 && r >= a.heads[which] * groups) {
    r -= a.heads[which] * groups;
    ++which;
  }
  const int head = r / groups, grp = r % groups;
  const int s = static_cast<int>(t % seq);
  const __nv_bfloat16* src = a.in[which] + t * a.ld[which];
  const int64_t orow = t * static_cast<int64_t>(a.heads[which]) * d;
  __nv_bfloat16* dst = a.out[which] + orow;
  const int i0 = head * d + grp * 8;
  V8 va, vb, oa, ob;
  va.u = *reinterpret_cast<const uint4*>(src + i0);
  vb.u = *reinterpret_cast<const uint4*>(src + i0 + half);
  if (mode == 0 && a.add[which] != nullptr) {
    V8 pa, pb;
    pa.u = *reinterpret_cast<const uint4*>(a.add[which] + orow + i0);
    pb.u = *reinterpret_cast<const uint4*>(a.add[which] + orow + i0 + half);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      va.h[j] = __float2bfloat16_rn(__bfloat162float(va.h[j]) + __bfloat162float(pa.h[j]));
      vb.h[j] = __float2bfloat16_rn(__bfloat162float(vb.h[j]) + __bfloat162float(pb.h[j]));
    }
  }
  if (which == 2) {  // v: no rotation
    *reinterpret_cast<uint4*>(dst + i0) = va.u;
    *reinterpret_cast<uint4*>(dst + i0 + half) = vb.u;
    return;
  }
  V8 c1, s1, c2, s2;
  c1.u = *reinterpret_cast<const uint4*>(cosv + static_cast<int64_t>(s) * d + grp * 8);
  s1.u = *reinterpret_cast<const uint4*>(sinv + static_cast<int64_t>(s) * d + grp * 8);
  c2.u = *reinterpret_cast<const uint4*>(cosv + static_cast<int64_t>(s) * d + half + grp * 8);
  s2.u = *reinterpret_cast<const uint4*>(sinv + static_cast<int64_t>(s) * d + half + grp * 8);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float xa = __bfloat162float(va.h[j]), xb = __bfloat162float(vb.h[j]);
    if (mode == 0) {
      // out[i] = x[i]c[i] + (-x[i+h]) s[i];  out[i+h] = x[i+h]c[i+h] + x[i] s[i+h]
      const float ta = __bfloat162float(__float2bfloat16_rn(xa * __bfloat162float(c1.h[j])));
      const float tb = __bfloat162float(__float2bfloat16_rn(-xb * __bfloat162float(s1.h[j])));
      oa.h[j] = __float2bfloat16_rn(ta + tb);
      const float tc = __bfloat162float(__float2bfloat16_rn(xb * __bfloat162float(c2.h[j])));
      const float td = __bfloat162float(__float2bfloat16_rn(xa * __bfloat162float(s2.h[j])));
      ob.h[j] = __float2bfloat16_rn(tc + td);
    } else {
      // dx[i] = dout[i]c[i] + dout[i+h]s[i+h];  dx[i+h] = dout[i+h]c[i+h] - dout[i]s[i]
      oa.h[j] = __float2bfloat16_rn(xa * __bfloat162float(c1.h[j]) +
                                    xb * __bfloat162float(s2.h[j]));
      ob.h[j] = __float2bfloat16_rn(xb * __bfloat162float(c2.h[j]) -
                                    xa * __bfloat162float(s1.h[j]));
    }
  }
  *reinterpret_cast<uint4*>(dst + i0) = oa.u;
  *reinterpret_cast<uint4*>(dst + i0 + half) = ob.u;
}

// ---------------------------------------------------------------- SwiGLU
// silu(x) = x / (1 + 2^(-x log2 e)) with the hardware's approximate base-2
// exponential and reciprocal (a few ulps of fp32 from the IEEE expression; the
// result is rounded to bf16 next), two columns at a time where the arithmetic
// has a packed fp32 form.
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

constexpr float kNegLog2E = -1.4426950408889634f;

// bf16(silu(g)) for the two bf16 of a word, low half first.
__device__ __forceinline__ uint32_t silu_bf16x2(uint32_t gw) {
  const uint64_t g2 = f2_from_bf16x2(gw);
  float a, b;
  f2_unpack(f2_mul(g2, f2_splat(kNegLog2E)), a, b);
  f2_unpack(f2_add(f2_pack(ex2_approx(a), ex2_approx(b)), f2_splat(1.f)), a, b);
  return bf16x2_from_f2(f2_mul(g2, f2_pack(rcp_approx(a), rcp_approx(b))));
}

constexpr int kSwThreads = 256;  // wide rows (I = 11008 / 14336): 256 threads per row

// Resident 256-thread blocks per SM asked of the register allocator. VPT 6 (I = 11008)
// fits in 48 registers, 5 blocks instead of the 4 that its unconstrained 55 allow; VPT 8
// (I = 14336) keeps its 64 registers (4 blocks: its 16 uint4 of row data would spill
// below that) but is scheduled differently under the hint. Measured at M = 4096 with
// the L2 flushed: 55.3 -> 51 us at I = 11008, 68.5 -> 60 us at I = 14336. Omitting the
// hint is not the same as 1: a 1 lets ptxas grow VPT 8 to 148 registers (1 block per
// SM, 1.75x slower).
constexpr int sw_min_blocks(int vpt) { return vpt <= 2 ? 8 : vpt <= 6 ? 5 : 4; }

template <int VPT>
__global__ void __launch_bounds__(kSwThreads, sw_min_blocks(VPT)) swiglu_quant_kernel(
    const __nv_bfloat16* __restrict__ gu, int64_t ldgu, int inter, int8_t* __restrict__ q,
    int64_t ldq, float* __restrict__ scale, __nv_bfloat16* __restrict__ m_out, int64_t ldm) {
  __shared__ float red[kSwThreads / 32];
  const int64_t row = blockIdx.x;
  const int nvec = inter / 8;
  const __nv_bfloat16* gate = gu + row * ldgu;
  const __nv_bfloat16* up = gate + inter;
  uint4 mv[VPT], uv[VPT];
  // every load is issued before any is used: one memory round trip per row
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kSwThreads;
    mv[i] = uv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (idx < nvec) {
      mv[i] = ld_stream16(reinterpret_cast<const uint4*>(gate) + idx);
      uv[i] = ld_stream16(reinterpret_cast<const uint4*>(up) + idx);
    }
  }
  // m = bf16(bf16(silu(gate)) * up): the bf16 x bf16 product is exact in fp32,
  // so one bf16x2 multiply rounds it as the fp32 product followed by RN does
  __nv_bfloat162 amax2 = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    uint32_t* w = reinterpret_cast<uint32_t*>(&mv[i]);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&uv[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a = silu_bf16x2(w[j]);
      const __nv_bfloat162 m = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                       *reinterpret_cast<const __nv_bfloat162*>(&u[j]));
      amax2 = __hmax2(amax2, __habs2(m));
      w[j] = *reinterpret_cast<const uint32_t*>(&m);
    }
    const int idx = threadIdx.x + i * kSwThreads;
    if (m_out != nullptr && idx < nvec) reinterpret_cast<uint4*>(m_out + row * ldm)[idx] = mv[i];
  }
  const float amax = block_max<kSwThreads / 32>(
      fmaxf(__bfloat162float(__low2bfloat16(amax2)), __bfloat162float(__high2bfloat16(amax2))),
      red);
  float s, inv_s;
  row_scale(amax, s, inv_s);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * kSwThreads;
    if (idx < nvec)
      *reinterpret_cast<uint2*>(q + row * ldq + static_cast<int64_t>(idx) * 8) =
          quant8_bf16(mv[i], s, inv_s);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, int64_t ldgu,
                                  const __nv_bfloat16* __restrict__ dm, int64_t lddm,
                                  int64_t rows, int inter, __nv_bfloat16* __restrict__ dgu,
                                  int64_t lddgu) {
  const int per_row = inter / 8;
  const int64_t gid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (gid >= rows * per_row) return;
  const int64_t r = gid / per_row;
  const int c = static_cast<int>(gid % per_row) * 8;
  V8 gv, uv, dv, og, ou;
  gv.u = *reinterpret_cast<const uint4*>(gu + r * ldgu + c);
  uv.u = *reinterpret_cast<const uint4*>(gu + r * ldgu + inter + c);
  dv.u = *reinterpret_cast<const uint4*>(dm + r * lddm + c);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float g = __bfloat162float(gv.h[j]), u = __bfloat162float(uv.h[j]);
    const float d = __bfloat162float(dv.h[j]);
    const float sg = 1.f / (1.f + expf(-g));
    og.h[j] = __float2bfloat16_rn(d * u * (sg * (1.f + g * (1.f - sg))));
    ou.h[j] = __float2bfloat16_rn(d * g * sg);
  }
  *reinterpret_cast<uint4*>(dgu + r * lddgu + c) = og.u;
  *reinterpret_cast<uint4*>(dgu + r * lddgu + inter + c) = ou.u;
}

int vpt_for(int cols) {
  const int nv = (cols / 8 + kThreads - 1) / kThreads;
  if (nv <= 4) return 4;
  if (nv <= 8) return 8;
  if (nv <= 12) return 12;
  if (nv <= 16) return 16;
  return 0;
}

bool rows_ok(const void* p, int64_t ld) { return aligned16(p) && ld % 8 == 0; }

}  // namespace
}  // namespace lema

using namespace lema;

// Launches KERNEL<VPT> for the register-vector count chosen by vpt_for();
// ARGS is the parenthesised kernel argument list, the rest the launch config.
#define LEMA_VPT_LAUNCH(vpt, KERNEL, ARGS, ...)              \
  switch (vpt) {                                             \
    case 4: KERNEL<4><<<__VA_ARGS__>>> ARGS; break;          \
    case 8: KERNEL<8><<<__VA_ARGS__>>> ARGS; break;          \
    case 12: KERNEL<12><<<__VA_ARGS__>>> ARGS; break;        \
    default: KERNEL<16><<<__VA_ARGS__>>> ARGS; break;        \
  }

extern "C" int lema_rmsnorm_quant(const void* x_bf16, int64_t ldx, const void* g_bf16,
                                  int64_t rows, int64_t cols, float eps, void* hn_bf16,
                                  int64_t ldh, int8_t* q, int64_t ldq, float* scale, float* rstd,
                                  void* stream) {
  clear_error();
  if (rows < 0 || cols <= 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad size");
  if (rows == 0) return LEMA_OK;
  if (!x_bf16 || !g_bf16 || !hn_bf16 || (q && !scale))
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  const int vpt = vpt_for(static_cast<int>(cols));
  if (cols % 8 != 0 || vpt == 0 || cols > INT32_MAX || rows > INT32_MAX)
    return set_error(LEMA_ERR_UNSUPPORTED, "rmsnorm_quant needs cols % 8 == 0, cols <= 16384");
  if (!rows_ok(x_bf16, ldx) || !rows_ok(hn_bf16, ldh) || !aligned16(g_bf16) ||
      (q && (reinterpret_cast<uintptr_t>(q) % 8 != 0 || ldq % 8 != 0)))
    return set_error(LEMA_ERR_MISALIGNED, "rmsnorm_quant needs 16-byte aligned rows");
  auto s = static_cast<cudaStream_t>(stream);
  LEMA_VPT_LAUNCH(vpt, rmsnorm_quant_kernel, (
      static_cast<const __nv_bfloat16*>(x_bf16), ldx, static_cast<const __nv_bfloat16*>(g_bf16),
      static_cast<int>(cols), eps, static_cast<__nv_bfloat16*>(hn_bf16), ldh, q, ldq, scale,
      rstd),
                  static_cast<unsigned>(rows), kThreads, 0, s);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_rmsnorm_bwd(const void* x_bf16, int64_t ldx, const void* g_bf16,
                                const float* rstd, const void* dhn_bf16, int64_t ldd,
                                int64_t rows, int64_t cols, void* dx_bf16, int64_t lddx,
                                void* stream) {
  clear_error();
  if (rows < 0 || cols <= 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad size");
  if (rows == 0) return LEMA_OK;
  if (!x_bf16 || !g_bf16 || !rstd || !dhn_bf16 || !dx_bf16)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  const int vpt = vpt_for(static_cast<int>(cols));
  if (cols % 8 != 0 || vpt == 0)
    return set_error(LEMA_ERR_UNSUPPORTED, "rmsnorm_bwd needs cols % 8 == 0, cols <= 16384");
  if (!rows_ok(x_bf16, ldx) || !rows_ok(dhn_bf16, ldd) || !rows_ok(dx_bf16, lddx) ||
      !aligned16(g_bf16))
    return set_error(LEMA_ERR_MISALIGNED, "rmsnorm_bwd needs 16-byte aligned rows");
  auto s = static_cast<cudaStream_t>(stream);
  LEMA_VPT_LAUNCH(vpt, rmsnorm_bwd_kernel, (
      static_cast<const __nv_bfloat16*>(x_bf16), ldx, static_cast<const __nv_bfloat16*>(g_bf16),
      rstd, static_cast<const __nv_bfloat16*>(dhn_bf16), ldd, static_cast<int>(cols),
      static_cast<__nv_bfloat16*>(dx_bf16), lddx),
                  static_cast<unsigned>(rows), kThreads, 0, s);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_rope_qkv(const void* q_in, int64_t ldq, const void* k_in, int64_t ldk,
                             const void* v_in, int64_t ldv, const void* q_add, const void* k_add,
                             const void* v_add, const void* cos_bf16, const void* sin_bf16,
                             int64_t tokens, int32_t seq, int32_t heads_q, int32_t heads_k,
                             int32_t head_dim, void* q_out, void* k_out, void* v_out,
                             int32_t mode, void* stream) {
  clear_error();
  if (tokens < 0 || seq <= 0 || heads_q < 0 || heads_k < 0 || head_dim <= 0 ||
      (mode != 0 && mode != 1))
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad size or mode");
  if (tokens == 0) return LEMA_OK;
  if (head_dim % 16 != 0)
    return set_error(LEMA_ERR_UNSUPPORTED, "rope needs head_dim % 16 == 0");
  if (!q_in || !k_in || !cos_bf16 || !sin_bf16 || !q_out || !k_out || (v_in && !v_out))
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  const void* ptrs[] = {q_out, k_out, v_out, q_add, k_add, v_add, cos_bf16, sin_bf16};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return set_error(LEMA_ERR_MISALIGNED, "rope needs 16-byte aligned rows");
  if (!rows_ok(q_in, ldq) || !rows_ok(k_in, ldk) || (v_in && !rows_ok(v_in, ldv)))
    return set_error(LEMA_ERR_MISALIGNED, "rope needs 16-byte aligned rows");
  RopeArgs a;
  a.in[0] = static_cast<const __nv_bfloat16*>(q_in);
  a.in[1] = static_cast<const __nv_bfloat16*>(k_in);
  a.in[2] = static_cast<const __nv_bfloat16*>(v_in);
  a.ld[0] = ldq;
  a.ld[1] = ldk;
  a.ld[2] = ldv;
  a.add[0] = static_cast<const __nv_bfloat16*>(q_add);
  a.add[1] = static_cast<const __nv_bfloat16*>(k_add);
  a.add[2] = static_cast<const __nv_bfloat16*>(v_add);
  a.out[0] = static_cast<__nv_bfloat16*>(q_out);
  a.out[1] = static_cast<__nv_bfloat16*>(k_out);
  a.out[2] = static_cast<__nv_bfloat16*>(v_out);
  a.heads[0] = heads_q;
  a.heads[1] = heads_k;
  a.heads[2] = (v_in && mode == 0) ? heads_k : 0;
  const int64_t work = tokens * (a.heads[0] + a.heads[1] + a.heads[2]) * (head_dim / 16);
  const int64_t blocks = (work + 255) / 256;
  if (blocks > INT32_MAX) return set_error(LEMA_ERR_UNSUPPORTED, "too many tokens");
  rope_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, static_cast<const __nv_bfloat16*>(cos_bf16), static_cast<const __nv_bfloat16*>(sin_bf16),
      tokens, seq, head_dim, mode);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_rope(const void* q_in, int64_t ldq_in, const void* k_in, int64_t ldk_in,
                         const void* cos_bf16, const void* sin_bf16, int64_t tokens, int32_t seq,
                         int32_t heads_q, int32_t heads_k, int32_t head_dim, void* q_out,
                         void* k_out, int32_t mode, void* stream) {
  return lema_rope_qkv(q_in, ldq_in, k_in, ldk_in, nullptr, 0, nullptr, nullptr, nullptr,
                       cos_bf16, sin_bf16, tokens, seq, heads_q, heads_k, head_dim, q_out, k_out,
                       nullptr, mode, stream);
}

extern "C" int lema_swiglu_quant(const void* gu_bf16, int64_t ldgu, int64_t rows, int64_t inter,
                                 int8_t* q, int64_t ldq, float* scale, void* m_bf16, int64_t ldm,
                                 void* stream) {
  clear_error();
  if (rows < 0 || inter <= 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad size");
  if (rows == 0) return LEMA_OK;
  if (!gu_bf16 || !q || !scale) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  const int64_t nv = (inter / 8 + kSwThreads - 1) / kSwThreads;
  if (inter % 8 != 0 || nv > 8)
    return set_error(LEMA_ERR_UNSUPPORTED, "swiglu_quant needs inter % 8 == 0, <= 16384");
  if (!rows_ok(gu_bf16, ldgu) || reinterpret_cast<uintptr_t>(q) % 8 != 0 || ldq % 8 != 0 ||
      (m_bf16 && !rows_ok(m_bf16, ldm)))
    return set_error(LEMA_ERR_MISALIGNED, "swiglu_quant needs 16-byte aligned rows");
  auto s = static_cast<cudaStream_t>(stream);
  const int vpt = nv <= 2 ? 2 : (nv <= 4 ? 4 : (nv <= 6 ? 6 : 8));
  auto args = [&](auto kern) {
    kern<<<static_cast<unsigned>(rows), kSwThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(gu_bf16), ldgu, static_cast<int>(inter), q, ldq, scale,
        static_cast<__nv_bfloat16*>(m_bf16), ldm);
  };
  switch (vpt) {
    case 2: args(swiglu_quant_kernel<2>); break;
    case 4: args(swiglu_quant_kernel<4>); break;
    case 6: args(swiglu_quant_kernel<6>); break;
    default: args(swiglu_quant_kernel<8>); break;
  }
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_swiglu_bwd(const void* gu_bf16, int64_t ldgu, const void* dm_bf16,
                               int64_t lddm, int64_t rows, int64_t inter, void* dgu_bf16,
                               int64_t lddgu, void* stream) {
  clear_error();
  if (rows < 0 || inter <= 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad size");
  if (rows == 0) return LEMA_OK;
  if (!gu_bf16 || !dm_bf16 || !dgu_bf16) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null pointer");
  if (inter % 8 != 0) return set_error(LEMA_ERR_UNSUPPORTED, "swiglu_bwd needs inter % 8 == 0");
  if (!rows_ok(gu_bf16, ldgu) || !rows_ok(dm_bf16, lddm) || !rows_ok(dgu_bf16, lddgu))
    return set_error(LEMA_ERR_MISALIGNED, "swiglu_bwd needs 16-byte aligned rows");
  const int64_t work = rows * (inter / 8);
  swiglu_bwd_kernel<<<static_cast<unsigned>((work + 255) / 256), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gu_bf16), ldgu, static_cast<const __nv_bfloat16*>(dm_bf16),
      lddm, rows, static_cast<int>(inter), static_cast<__nv_bfloat16*>(dgu_bf16), lddgu);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}
