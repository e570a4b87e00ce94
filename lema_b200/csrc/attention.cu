// attention.cu — causal self-attention (head_dim 128, GQA) on the 5th-generation
// tensor cores: forward and backward, bf16 in / bf16 out, fp32 softmax and
// accumulators. It replaces the block's scaled-dot-product attention
// (torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True,
// scale=head_dim ** -0.5, enable_gqa=...)), which the reference's Llama adapter
// runs through HF's attention (src/lema/adapters/_llama.py:236-252).
//
// Layout in HBM: the token-major projections the block already produces —
// q [B*S, H*128], k and v [B*S, Hkv*128], o [B*S, H*128] (row strides given),
// addressed by 3-D tensor maps {columns, S, B} so that a 128-token tile never
// reads into the next sequence (TMA zero-fills past S and clips stores there).
// lse [B, H, S] fp32 holds each query row's log2-domain log-sum-exp of the
// scaled scores; delta [B, H, S] fp32 holds rowsum(dO * O) for the backward.
//
// Forward (attn_fwd_kernel): one CTA per (b, h, pair of 128-query tiles A and B),
// heaviest pairs first; the pair shares every K / V tile it loads (one tile per
// CTA when the pairs would be fewer than the SMs). Warp 0 loads
// Q of both tiles once and K / V tiles into two-slot rings (two producer
// threads; TMA, 128-byte swizzle); warp 1 issues S = Q K^T (M = N = 128, K = 128)
// into each tile's TMEM score block and O += P V into each tile's TMEM
// accumulator, P read from TMEM as the A operand and V read MN-major straight
// from its token-major tile, in the order P_A V, S_A(next), P_B V, S_B(next), so
// that one tile's softmax runs while the tensor core works on the other's. Four
// softmax warps per tile, one thread per query row: each masks the diagonal tile,
// keeps its row's running max and sum (online softmax; O is rescaled in TMEM only
// when the max grows by more than 2^8, so P stays below 256), writes P as bf16
// over its own scores in TMEM, and finally normalises O into a TMA store and
// records the row's log-sum-exp.
//
// Backward (three or four kernels, no atomics, deterministic): attn_delta_kernel
// (rowsum(dO * O)), then
//   attn_bwd_dkdv_kernel: one CTA per (b, kv head, 128-key tile), heaviest
//     first; for every query head of the group and every causal query tile (Q / dO
//     double-buffered) it forms S^T = K Q^T and dP^T = V dO^T in TMEM, P^T =
//     exp2(S^T c - lse), dS^T = P^T (dP^T - delta), and accumulates dV += P^T dO
//     and dK += dS^T Q (Q, dO read MN-major from the tiles the first two MMAs used
//     K-major; P^T and dS^T share one shared tile in turn). When
//     those CTAs would not fill the GPU (GQA, few sequences or heads), one CTA per
//     query head instead writes its head's fp32 dK / dV share and
//     attn_dkv_reduce_kernel sums a group's shares in head order into the bf16
//     dK / dV of its kv head.
//   attn_bwd_dq_kernel: one CTA per (b, h, 128-query tile); for every causal key
//     tile (K / V double-buffered) it forms S = Q K^T and dP = dO V^T, dS = P (dP
//     - delta), and accumulates dQ += dS K (K read MN-major); its 16 row warps
//     free the score TMEM as soon as they have read it.
// dK, dQ carry the softmax scale; dK / dV of a kv head sum over its query heads.
//
// Every wait is bounded (clock64 budget) and also ends when another role of the
// CTA has given up: a timeout records an error word and the CTA drains its
// copies and MMAs in flight before TMEM is released.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include <cudaTypedefs.h>

#include "internal.h"
#include "ptx.cuh"
#include "quant_core.cuh"

namespace lema {
namespace {

constexpr int kHd = 128;          // head dim
constexpr int kTile = 128;        // query / key rows per tile
constexpr int kBox = 16384;       // one TMA box: 128 rows x 64 bf16 (128 B), swizzled
constexpr int kTileBytes = 2 * kBox;  // a 128 x 128 bf16 tile = two boxes
constexpr uint32_t kIdescKK = ptx::idesc_bf16_f32_major(128, 128, false, false);
constexpr uint32_t kIdescKMn = ptx::idesc_bf16_f32_major(128, 128, false, true);
constexpr float kRescaleLog2 = 8.f;  // O is rescaled when a row max grows by more

struct AttnParams {
  int B, S, H, Hkv, q_tiles;
  float scale;       // softmax scale (head_dim ** -0.5)
  float scale_log2;  // scale * log2(e)
  float* lse;        // [B, H, S]
  const float* delta;  // [B, H, S] (backward)
  float* dkv_ws;       // split GQA backward: fp32 dK / dV shares per query head, or null
  int64_t ws_half;     // floats in each half of dkv_ws (B * S * H * 128)
  int heads_per_cta;   // dK/dV kernel: the whole group (bf16 out) or 1 (shares into dkv_ws)
  int fwd_tiles_per_cta;  // forward: 2 (pairs of query tiles) or 1 (grids below the SM count)
  int32_t* err;
  long long budget;
};

__device__ __forceinline__ void record_err(int32_t* err, int32_t code, int* abort_flag) {
  atomicCAS(err, 0, code);
  *reinterpret_cast<volatile int*>(abort_flag) = 1;
}

__device__ __forceinline__ bool is_aborted(const int* abort_flag) {
  return *reinterpret_cast<const volatile int*>(abort_flag) != 0;
}

// mbar_wait that also gives up when another role of the CTA has aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, long long budget,
                                         const int* abort_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (is_aborted(abort_flag) || clock64() - t0 > budget) return false;
  }
}

// Byte offset of the 16-byte chunk holding columns [col, col + 8) (col a
// multiple of 8, < 128) of row r (< 128) in a 128 x 128 bf16 tile stored as two
// 128-byte-swizzled boxes of 64 columns (TMA's layout): box col / 64, row r at
// 128 B, chunk (col / 8) % 8 exchanged with r % 8. Always < 32768.
__device__ __forceinline__ uint32_t swz_chunk(int r, int col) {
  return static_cast<uint32_t>((col >> 6) * kBox + r * 128 +
                               ((((col >> 3) & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void st_shared_v4(uint32_t saddr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Named barrier 1 over the N row threads of a kernel (warps 2 ..).
template <int N>
__device__ __forceinline__ void sync_softmax_n() {
  asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// S or dP = A B^T over head_dim: A, B both [128 x 128] K-major tiles.
__device__ __forceinline__ void mma_tile_kk(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr,
                                            bool accumulate_first) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t off = static_cast<uint32_t>((k >> 2) * kBox + (k & 3) * 32);
    ptx::mma_bf16(d_tmem, ptx::desc_kmajor_sw128(a_addr + off),
                  ptx::desc_kmajor_sw128(b_addr + off), kIdescKK,
                  (accumulate_first || k > 0) ? 1u : 0u);
  }
}

// D += A B over 128 inner rows: A [128 x 128] K-major (written by threads),
// B a token-major [128 rows x 128 dims] tile read MN-major (N = dims).
__device__ __forceinline__ void mma_tile_kmn(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr,
                                             bool accumulate_first) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t aoff = static_cast<uint32_t>((k >> 2) * kBox + (k & 3) * 32);
    ptx::mma_bf16(d_tmem, ptx::desc_kmajor_sw128(a_addr + aoff),
                  ptx::desc_mnmajor_sw128(b_addr + k * 2048, kBox, 1024), kIdescKMn,
                  (accumulate_first || k > 0) ? 1u : 0u);
  }
}

// wait_bar whose result is the same for every lane of the warp (the warp then
// takes the same path into warp-collective tcgen05 loads and stores).
__device__ __forceinline__ bool wait_bar_warp(uint64_t* bar, uint32_t parity, long long budget,
                                              const int* abort_flag) {
  const bool r = wait_bar(bar, parity, budget, abort_flag);
  return __all_sync(0xffffffffu, r);
}

// ------------------------------------------------------------------ forward
constexpr int kFwdThreads = 320;  // producer warp, MMA warp, 2 x 4 softmax warps
constexpr bool kPolyExp = true;
constexpr int kFwdBars = 16;
constexpr int kFwdSmem = 6 * kTileBytes + kFwdBars * 8 + 16 + 1024;

// O += P V over 128 keys: P [128 rows x 128 keys] bf16 in TMEM (64 columns from
// p_tmem, two keys per column), V a token-major [128 keys x 128 dims] tile read
// MN-major (N = dims).
__device__ __forceinline__ void mma_tile_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_addr,
                                            bool accumulate_first) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    ptx::mma_bf16_tmem_a(d_tmem, p_tmem + static_cast<uint32_t>(k * 8),
                         ptx::desc_mnmajor_sw128(v_addr + k * 2048, kBox, 1024), kIdescKMn,
                         (accumulate_first || k > 0) ? 1u : 0u);
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mo,
                    const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem;                   // Q of tiles A and B; O staging at the end
  uint8_t* sk = smem + 2 * kTileBytes;  // K ring, 2 slots
  uint8_t* sv = smem + 4 * kTileBytes;  // V ring, 2 slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // 2 slots
  uint64_t* k_empty = bars + 3;  // 2 slots
  uint64_t* v_full = bars + 5;   // 2 slots
  uint64_t* v_empty = bars + 7;  // 2 slots
  uint64_t* s_full = bars + 9;   // per query tile
  uint64_t* p_full = bars + 11;  // per query tile
  uint64_t* o_done = bars + 13;  // per query tile
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kFwdBars);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int bh_count = p.B * p.H;
  const int per = p.fwd_tiles_per_cta;  // 2, or 1 when pairs would leave SMs idle
  const int groups = (p.q_tiles + per - 1) / per;
  const int grp = groups - 1 - static_cast<int>(blockIdx.x) / bh_count;  // heaviest first
  const int bh = static_cast<int>(blockIdx.x) % bh_count;
  const int b = bh / p.H, h = bh % p.H;
  const int kvh = h / (p.H / p.Hkv);
  const int qa = per * grp;  // query tile A; B is qa + 1
  // one tile per CTA, or an odd tile count's last pair: no tile B
  const bool has_b = per == 2 && qa + 1 < p.q_tiles;
  const int n_a = qa + 1;                 // key tiles of A (causal)
  const int n_kv = has_b ? qa + 2 : n_a;  // key tiles of the pair

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&mq);
    ptx::prefetch_tmap(&mk);
    ptx::prefetch_tmap(&mv);
    ptx::prefetch_tmap(&mo);
    for (int i = 0; i < kFwdBars; ++i) ptx::mbar_init(&bars[i], 1);
    ptx::mbar_init(&p_full[0], 128);  // every row thread of the tile arrives
    ptx::mbar_init(&p_full[1], 128);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);  // S/P of A [0,128), of B [128,256); O of A, B [256,512)
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  ptx::griddep_wait();

  if (warp == 0) {
    // ---------------- TMA producers: lane 0 Q and K, lane 1 V ----------------
    if (lane == 0) {
      int k_issued = 0;
      bool ok = true;
      ptx::mbar_arrive_expect_tx(q_full, (has_b ? 2 : 1) * kTileBytes);
      ptx::tma_load_3d(sq, &mq, q_full, h * kHd, qa * kTile, b);
      ptx::tma_load_3d(sq + kBox, &mq, q_full, h * kHd + 64, qa * kTile, b);
      if (has_b) {
        ptx::tma_load_3d(sq + kTileBytes, &mq, q_full, h * kHd, (qa + 1) * kTile, b);
        ptx::tma_load_3d(sq + kTileBytes + kBox, &mq, q_full, h * kHd + 64, (qa + 1) * kTile, b);
      }
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !wait_bar(&k_empty[s], ((j - 2) >> 1) & 1, p.budget, abort_flag)) {
          ok = false;
          break;
        }
        ptx::mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        ptx::tma_load_3d(sk + s * kTileBytes, &mk, &k_full[s], kvh * kHd, j * kTile, b);
        ptx::tma_load_3d(sk + s * kTileBytes + kBox, &mk, &k_full[s], kvh * kHd + 64, j * kTile,
                         b);
        ++k_issued;
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      // every issued load lands before this CTA's shared memory is released
      (void)ptx::mbar_wait(q_full, 0, p.budget);
      for (int i = k_issued - 1; i >= 0 && i >= k_issued - 2; --i)
        (void)ptx::mbar_wait(&k_full[i & 1], (i >> 1) & 1, p.budget);
    } else if (lane == 1) {
      int v_issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !wait_bar(&v_empty[s], ((j - 2) >> 1) & 1, p.budget, abort_flag)) {
          ok = false;
          break;
        }
        ptx::mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        ptx::tma_load_3d(sv + s * kTileBytes, &mv, &v_full[s], kvh * kHd, j * kTile, b);
        ptx::tma_load_3d(sv + s * kTileBytes + kBox, &mv, &v_full[s], kvh * kHd + 64, j * kTile,
                         b);
        ++v_issued;
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      for (int i = v_issued - 1; i >= 0 && i >= v_issued - 2; --i)
        (void)ptx::mbar_wait(&v_full[i & 1], (i >> 1) & 1, p.budget);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      // Order: S_A(0), S_B(0), then for every key tile j: O_A += P_A(j) V_j, S_A(j+1),
      // O_B += P_B(j) V_j, S_B(j+1). S_X(j+1) overwrites P_X(j) in TMEM after the
      // P V MMA that reads it (MMAs of one thread run in issue order), and one
      // tile's softmax runs while the tensor core works on the other tile.
      bool ok = wait_bar(q_full, 0, p.budget, abort_flag) &&
                wait_bar(&k_full[0], 0, p.budget, abort_flag);
      bool issued = false;
      if (ok) {
        ptx::tc_fence_after();
        mma_tile_kk(tmem, ptx::smem_u32(sq), ptx::smem_u32(sk), false);
        ptx::mma_commit(&s_full[0]);
        if (has_b) {
          mma_tile_kk(tmem + 128, ptx::smem_u32(sq + kTileBytes), ptx::smem_u32(sk), false);
          ptx::mma_commit(&s_full[1]);
        }
        ptx::mma_commit(&k_empty[0]);
        issued = true;
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j & 1, nx = j + 1, ns = nx & 1;
        const uint32_t v_addr = ptx::smem_u32(sv + s * kTileBytes);
        const uint32_t k_addr = ptx::smem_u32(sk + ns * kTileBytes);
        bool k_ready = false;
        if (!wait_bar(&v_full[s], (j >> 1) & 1, p.budget, abort_flag)) {
          ok = false;
          break;
        }
        if (j < n_a) {
          if (!wait_bar(&p_full[0], j & 1, p.budget, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_pv(tmem + 256, tmem, v_addr, j > 0);
          if (nx < n_a) {
            if (!wait_bar(&k_full[ns], (nx >> 1) & 1, p.budget, abort_flag)) {
              ok = false;
              break;
            }
            k_ready = true;
            ptx::tc_fence_after();
            mma_tile_kk(tmem, ptx::smem_u32(sq), k_addr, false);
            ptx::mma_commit(&s_full[0]);
          } else {
            ptx::mma_commit(&o_done[0]);
          }
        }
        if (has_b) {
          if (!wait_bar(&p_full[1], j & 1, p.budget, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_pv(tmem + 384, tmem + 128, v_addr, j > 0);
          if (nx < n_kv) {
            if (!k_ready && !wait_bar(&k_full[ns], (nx >> 1) & 1, p.budget, abort_flag)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            mma_tile_kk(tmem + 128, ptx::smem_u32(sq + kTileBytes), k_addr, false);
            ptx::mma_commit(&s_full[1]);
          } else {
            ptx::mma_commit(&o_done[1]);
          }
        }
        ptx::mma_commit(&v_empty[s]);
        if (nx < n_kv) ptx::mma_commit(&k_empty[ns]);
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      if (issued) {  // all MMAs complete before TMEM is released
        ptx::mma_commit(drain);
        (void)ptx::mbar_wait(drain, 0, p.budget);
      }
    }
  } else {
    // ---------------- softmax: warps 2..5 tile A, 6..9 tile B, one thread per query row ----------------
    // A thread holds its row's 128 scores, so the row max and sum never leave it.
    // O is rescaled in TMEM only when the row max grows by more than 2^8 (P stays
    // below 256); P (bf16) is written over the row's scores, where the P V MMA reads
    // it. The thread's O row is quiescent then: S_X(j) completing implies that
    // every earlier MMA of the issuer, P_X(j-1) V included, has completed.
    const int tile = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qx = qa + tile;
    const int n_x = tile == 0 ? n_a : n_kv;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_col = static_cast<uint32_t>(tile * 128);
    const uint32_t o_col = 256 + s_col;
    if (tile == 0 || has_b) {
      const uint64_t c2 = f2_splat(p.scale_log2);
      float m_run = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n_x; ++j) {
        if (!wait_bar_warp(&s_full[tile], j & 1, p.budget, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          ptx::tmem_ld_32x32b_x32(trow + s_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
        ptx::tmem_ld_wait();
        if (j == qx) {  // diagonal tile: keys after the query are masked
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > row) v[i] = 0xff800000u;  // -inf
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 128; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(v[i]));
        const float smax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        const float tmax = smax * p.scale_log2;  // scale > 0: max commutes with it
        const bool need = tmax > m_run + kRescaleLog2;
        const float m_new = need ? tmax : m_run;
        const float alpha = need ? ex2(m_run - m_new) : 1.f;
        l *= alpha;
        m_run = m_new;
        // P = 2^(s c - m), written over the scores in quarters of 32 keys: the
        // scaling and the sum two columns per instruction
        const uint64_t negm2 = f2_splat(-m_run);
        uint64_t acc0 = f2_splat(0.f), acc1 = f2_splat(0.f);
#pragma unroll
        for (int qtr = 0; qtr < 4; ++qtr) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = qtr * 32 + 2 * i;
            const uint64_t x2 =
                f2_fma(f2_pack(__uint_as_float(v[c]), __uint_as_float(v[c + 1])), c2, negm2);
            float ea, eb;
            f2_unpack(x2, ea, eb);
            ea = ex2(ea);
            eb = ex2(eb);
            if (i & 1)
              acc1 = f2_add(acc1, f2_pack(ea, eb));
            else
              acc0 = f2_add(acc0, f2_pack(ea, eb));
            pk[i] = pack_bf16x2(ea, eb);
          }
          ptx::tmem_st_32x32b_x16(trow + s_col + qtr * 16, pk);
        }
        float s0, s1, s2, s3;
        f2_unpack(acc0, s0, s1);
        f2_unpack(acc1, s2, s3);
        l += (s0 + s1) + (s2 + s3);
        // O *= alpha on this thread's row, after the scores are no longer held
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            ptx::tmem_ld_32x32b_x32(trow + o_col + c * 32, o);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            ptx::tmem_st_32x32b_x32(trow + o_col + c * 32, o);
          }
        }
        ptx::tmem_st_wait();
        ptx::tc_fence_before();
        ptx::mbar_arrive(&p_full[tile]);
      }
      // ---------------- epilogue: O / l -> bf16 -> TMA store; lse ----------------
      if (ok && !wait_bar_warp(&o_done[tile], 0, p.budget, abort_flag)) ok = false;
      if (!ok) {
        record_err(p.err, kDevErrAttnTimeout, abort_flag);
      } else {
        ptx::tc_fence_after();
        const float inv_l = 1.f / l;
        // Q_X is free: its last S MMA completed before the last P V of the tile
        const uint32_t obase = ptx::smem_u32(sq + tile * kTileBytes);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          ptx::tmem_ld_32x32b_x32(trow + o_col + c * 32, o);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t* e = &o[i * 8];
            st_shared_v4(obase + swz_chunk(row, c * 32 + i * 8),
                         pack_bf16x2(__uint_as_float(e[0]) * inv_l, __uint_as_float(e[1]) * inv_l),
                         pack_bf16x2(__uint_as_float(e[2]) * inv_l, __uint_as_float(e[3]) * inv_l),
                         pack_bf16x2(__uint_as_float(e[4]) * inv_l, __uint_as_float(e[5]) * inv_l),
                         pack_bf16x2(__uint_as_float(e[6]) * inv_l, __uint_as_float(e[7]) * inv_l));
          }
        }
        const int q = qx * kTile + row;
        if (q < p.S) p.lse[(static_cast<int64_t>(b) * p.H + h) * p.S + q] = m_run + log2f(l);
      }
      ptx::fence_proxy_async_smem();
      asm volatile("bar.sync %0, 128;" ::"r"(1 + tile) : "memory");  // the tile's 4 warps
      if (quarter == 2 && lane == 0 && !is_aborted(abort_flag)) {  // first warp of the tile
        ptx::tma_store_3d(&mo, sq + tile * kTileBytes, h * kHd, qx * kTile, b);
        ptx::tma_store_3d(&mo, sq + tile * kTileBytes + kBox, h * kHd + 64, qx * kTile, b);
        ptx::bulk_commit_group();
        ptx::bulk_wait_group_all();
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- backward

// delta[b, h, q] = sum_d dO[b, q, h, d] * O[b, q, h, d] (fp32), one warp per
// (token, head): 4 columns per lane.
__global__ void __launch_bounds__(256) attn_delta_kernel(const __nv_bfloat16* __restrict__ o,
                                                         int64_t ldo,
                                                         const __nv_bfloat16* __restrict__ dout,
                                                         int64_t lddo, float* __restrict__ delta,
                                                         int B, int S, int H) {
  const int lane = threadIdx.x % 32;
  const int64_t pairs = static_cast<int64_t>(B) * S * H;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
       w < pairs; w += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const int64_t tok = w / H;  // b * S + q
    const int h = static_cast<int>(w % H);
    const uint2 a = *reinterpret_cast<const uint2*>(o + tok * ldo + h * kHd + lane * 4);
    const uint2 g = *reinterpret_cast<const uint2*>(dout + tok * lddo + h * kHd + lane * 4);
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 af = __bfloat1622float2(a2[i]), gf = __bfloat1622float2(g2[i]);
      s = fmaf(af.x, gf.x, s);
      s = fmaf(af.y, gf.y, s);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      const int64_t b = tok / S, q = tok % S;
      delta[(b * H + h) * S + q] = s;
    }
  }
}

// Loads the 128 (lse, delta) values of query tile q0 of head (b, h) into shared
// memory; rows past S get lse = +inf (P = 0 there) and delta = 0.
__device__ __forceinline__ void stage_rows(const AttnParams& p, int b, int h, int q0, int tid,
                                           float* lse_s, float* delta_s) {
  const int q = q0 + tid;
  const int64_t i = (static_cast<int64_t>(b) * p.H + h) * p.S + q;
  lse_s[tid] = q < p.S ? p.lse[i] : INFINITY;
  delta_s[tid] = q < p.S ? p.delta[i] : 0.f;
}

// Writes 32 fp32 values (columns [col, col + 32) of row r) as bf16 into a
// swizzled 128 x 128 tile, each multiplied by mul.
__device__ __forceinline__ void store_row32(uint32_t tile, int r, int col, const float (&x)[32],
                                            float mul) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    st_shared_v4(tile + swz_chunk(r, col + i * 8),
                 pack_bf16x2(x[i * 8 + 0] * mul, x[i * 8 + 1] * mul),
                 pack_bf16x2(x[i * 8 + 2] * mul, x[i * 8 + 3] * mul),
                 pack_bf16x2(x[i * 8 + 4] * mul, x[i * 8 + 5] * mul),
                 pack_bf16x2(x[i * 8 + 6] * mul, x[i * 8 + 7] * mul));
}

constexpr int kDqThreads = 576;  // producer, MMA issuer, 16 row warps
constexpr int kDkdvThreads = 320;  // producer, MMA issuer, 8 row warps
constexpr int kDkdvBars = 11;
constexpr int kDkdvSmem = 7 * kTileBytes + 1024 + kDkdvBars * 8 + 16 + 1024;

// dK, dV of one (b, kv head, 128-key tile), or one query head's share of them.
// Eight row warps: warps w and w + 4 share TMEM lane quarter w % 4 and take
// query columns [64 half, 64 half + 64) of their key rows.
// The Q / dO tiles of the items are double-buffered, so the next item's loads
// overlap this one; P^T and dS^T share one tile: P^T is written, dV += P^T dO
// reads it, then dS^T (kept in registers meanwhile) replaces it for
// dK += dS^T Q. MMA issue order per item i: dV(i - 1), S^T(i) and dP^T(i),
// dK(i - 1). A row thread whose wait fails keeps passing the named barriers
// with its work skipped.
__global__ void __launch_bounds__(kDkdvThreads, 1)
    attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap mq,
                         const __grid_constant__ CUtensorMap mk,
                         const __grid_constant__ CUtensorMap mv,
                         const __grid_constant__ CUtensorMap mdo,
                         const __grid_constant__ CUtensorMap mdk,
                         const __grid_constant__ CUtensorMap mdv,
                         const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sk = smem;
  uint8_t* sv = smem + kTileBytes;
  uint8_t* sq = smem + 2 * kTileBytes;   // 2 slots (item % 2); dV, dK staging at the end
  uint8_t* sdo = smem + 4 * kTileBytes;  // 2 slots
  uint8_t* spd = smem + 6 * kTileBytes;  // P^T, then dS^T (bf16)
  float* lse_s = reinterpret_cast<float*>(smem + 7 * kTileBytes);
  float* delta_s = lse_s + kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * kTileBytes + 1024);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;   // 2 slots
  uint64_t* qd_empty = bars + 3;  // 2 slots: the item's dV and dK MMAs are complete
  uint64_t* st_full = bars + 5;   // S^T and dP^T are in TMEM
  uint64_t* st_free = bars + 6;   // the rows have read them (256 arrivals)
  uint64_t* p_ready = bars + 7;   // P^T is in shared memory (256 arrivals)
  uint64_t* dv_done = bars + 8;   // dV += P^T dO is complete: the tile is free
  uint64_t* ds_ready = bars + 9;  // dS^T is in shared memory (256 arrivals)
  uint64_t* drain = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDkdvBars);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int groups = p.H / p.heads_per_cta;  // head groups per sequence
  const int bg_count = p.B * groups;
  const int kt = static_cast<int>(blockIdx.x) / bg_count;  // key tile 0 (the heaviest) first
  const int b = (static_cast<int>(blockIdx.x) % bg_count) / groups;
  const int h0 = (static_cast<int>(blockIdx.x) % groups) * p.heads_per_cta;
  const int kvh = h0 / (p.H / p.Hkv);
  const int per_head = p.q_tiles - kt;  // causal query tiles kt .. q_tiles - 1
  const int n_items = p.heads_per_cta * per_head;

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&mq);
    ptx::prefetch_tmap(&mk);
    ptx::prefetch_tmap(&mv);
    ptx::prefetch_tmap(&mdo);
    for (int i = 0; i < kDkdvBars; ++i) ptx::mbar_init(&bars[i], 1);
    ptx::mbar_init(st_free, 256);
    ptx::mbar_init(p_ready, 256);
    ptx::mbar_init(ds_ready, 256);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);  // S^T [0,128), dP^T [128,256), dV [256,384), dK [384,512)
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  ptx::griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int issued = 0;
      bool ok = true;
      ptx::mbar_arrive_expect_tx(kv_full, 2 * kTileBytes);
      ptx::tma_load_3d(sk, &mk, kv_full, kvh * kHd, kt * kTile, b);
      ptx::tma_load_3d(sk + kBox, &mk, kv_full, kvh * kHd + 64, kt * kTile, b);
      ptx::tma_load_3d(sv, &mv, kv_full, kvh * kHd, kt * kTile, b);
      ptx::tma_load_3d(sv + kBox, &mv, kv_full, kvh * kHd + 64, kt * kTile, b);
      for (int it = 0; it < n_items; ++it) {
        const int slot = it & 1;
        const int h = h0 + it / per_head;
        const int q0 = (kt + it % per_head) * kTile;
        if (it >= 2 && !wait_bar(&qd_empty[slot], ((it - 2) >> 1) & 1, p.budget, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* q_dst = sq + slot * kTileBytes;
        uint8_t* do_dst = sdo + slot * kTileBytes;
        ptx::mbar_arrive_expect_tx(&qd_full[slot], 2 * kTileBytes);
        ptx::tma_load_3d(q_dst, &mq, &qd_full[slot], h * kHd, q0, b);
        ptx::tma_load_3d(q_dst + kBox, &mq, &qd_full[slot], h * kHd + 64, q0, b);
        ptx::tma_load_3d(do_dst, &mdo, &qd_full[slot], h * kHd, q0, b);
        ptx::tma_load_3d(do_dst + kBox, &mdo, &qd_full[slot], h * kHd + 64, q0, b);
        ++issued;
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      // every issued load lands before this CTA's shared memory is released
      (void)ptx::mbar_wait(kv_full, 0, p.budget);
      for (int i = issued - 1; i >= 0 && i >= issued - 2; --i)
        (void)ptx::mbar_wait(&qd_full[i & 1], (i >> 1) & 1, p.budget);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = wait_bar(kv_full, 0, p.budget, abort_flag);
      bool issued = false;
      for (int it = 0; ok && it <= n_items; ++it) {
        if (it >= 1) {  // dV += P^T dO of item it - 1
          const int j = it - 1;
          if (!wait_bar(p_ready, j & 1, p.budget, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_kmn(tmem + 256, ptx::smem_u32(spd), ptx::smem_u32(sdo + (j & 1) * kTileBytes),
                       j > 0);
          ptx::mma_commit(dv_done);
        }
        if (it < n_items) {  // S^T = K Q^T, dP^T = V dO^T of item it
          const int slot = it & 1;
          if (!wait_bar(&qd_full[slot], (it >> 1) & 1, p.budget, abort_flag) ||
              (it >= 1 && !wait_bar(st_free, (it - 1) & 1, p.budget, abort_flag))) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_kk(tmem, ptx::smem_u32(sk), ptx::smem_u32(sq + slot * kTileBytes), false);
          mma_tile_kk(tmem + 128, ptx::smem_u32(sv), ptx::smem_u32(sdo + slot * kTileBytes),
                      false);
          issued = true;
          ptx::mma_commit(st_full);
        }
        if (it >= 1) {  // dK += dS^T Q of item it - 1
          const int j = it - 1;
          if (!wait_bar(ds_ready, j & 1, p.budget, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_kmn(tmem + 384, ptx::smem_u32(spd), ptx::smem_u32(sq + (j & 1) * kTileBytes),
                       j > 0);
          ptx::mma_commit(&qd_empty[j & 1]);
        }
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      if (issued) {
        ptx::mma_commit(drain);
        (void)ptx::mbar_wait(drain, 0, p.budget);
      }
    }
  } else {
    // ---------------- elementwise rows (warps 2..9): two threads per key row ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int tid = threadIdx.x - 64;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t pd_base = ptx::smem_u32(spd);
    bool ok = true;
    for (int it = 0; it < n_items; ++it) {
      const int h = h0 + it / per_head;
      const int qi = kt + it % per_head;
      sync_softmax_n<256>();  // every row is done with the previous item's (lse, delta)
      if (tid < kTile) stage_rows(p, b, h, qi * kTile, tid, lse_s, delta_s);
      sync_softmax_n<256>();
      if (!ok) continue;
      if (!wait_bar_warp(st_full, it & 1, p.budget, abort_flag) ||
          (it >= 1 &&
           !wait_bar_warp(&qd_empty[(it - 1) & 1], ((it - 1) >> 1) & 1, p.budget, abort_flag))) {
        ok = false;  // the shared P / dS tile is free once dK of item it - 1 is done
        continue;
      }
      ptx::tc_fence_after();
      const bool diag = qi == kt;
      uint32_t dsk[32];  // this half row's dS^T, bf16 pairs, until dV has read P^T
#pragma unroll
      for (int cq = 0; cq < 2; ++cq) {
        const int c4 = 2 * half + cq;
        uint32_t sv32[32], dp32[32];
        ptx::tmem_ld_32x32b_x32(trow + c4 * 32, sv32);
        ptx::tmem_ld_32x32b_x32(trow + 128 + c4 * 32, dp32);
        ptx::tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float pr[2], dr[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = c4 * 32 + 2 * i + e;  // query column
            float pv = ex2(__uint_as_float(sv32[2 * i + e]) * p.scale_log2 - lse_s[c]);
            if (diag && c < row) pv = 0.f;  // key after query
            pr[e] = pv;
            dr[e] = pv * (__uint_as_float(dp32[2 * i + e]) - delta_s[c]);
          }
          pk[i] = pack_bf16x2(pr[0], pr[1]);
          dsk[cq * 16 + i] = pack_bf16x2(dr[0], dr[1]);
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          st_shared_v4(pd_base + swz_chunk(row, c4 * 32 + cc * 8), pk[cc * 4], pk[cc * 4 + 1],
                       pk[cc * 4 + 2], pk[cc * 4 + 3]);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(st_free);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(p_ready);
      if (!wait_bar_warp(dv_done, it & 1, p.budget, abort_flag)) {
        ok = false;
        continue;
      }
#pragma unroll
      for (int cc = 0; cc < 8; ++cc)
        st_shared_v4(pd_base + swz_chunk(row, half * 64 + cc * 8), dsk[cc * 4], dsk[cc * 4 + 1],
                     dsk[cc * 4 + 2], dsk[cc * 4 + 3]);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(ds_ready);
    }
    // ---------------- epilogue: dV, scale * dK -> bf16 -> TMA store, or (split
    // heads) this head's fp32 share into the workspace ----------------
    if (ok && !wait_bar_warp(&qd_empty[(n_items - 1) & 1], ((n_items - 1) >> 1) & 1, p.budget,
                             abort_flag))
      ok = false;
    const uint32_t dv_stage = ptx::smem_u32(sq), dk_stage = ptx::smem_u32(sq + kTileBytes);
    if (!ok) {
      record_err(p.err, kDevErrAttnTimeout, abort_flag);
    } else if (p.dkv_ws != nullptr) {
      ptx::tc_fence_after();
      const int key = kt * kTile + row;
      float* wk = p.dkv_ws + (static_cast<int64_t>(b) * p.S + key) * (p.H * kHd) + h0 * kHd;
      float* wv = wk + p.ws_half;
#pragma unroll 1
      for (int c4 = 2 * half; c4 < 2 * half + 2; ++c4) {
        uint32_t a[32], g[32];
        ptx::tmem_ld_32x32b_x32(trow + 256 + c4 * 32, a);
        ptx::tmem_ld_32x32b_x32(trow + 384 + c4 * 32, g);
        ptx::tmem_ld_wait();
        if (key < p.S) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            reinterpret_cast<float4*>(wv + c4 * 32)[i] =
                make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                            __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
            reinterpret_cast<float4*>(wk + c4 * 32)[i] = make_float4(
                __uint_as_float(g[4 * i]) * p.scale, __uint_as_float(g[4 * i + 1]) * p.scale,
                __uint_as_float(g[4 * i + 2]) * p.scale, __uint_as_float(g[4 * i + 3]) * p.scale);
          }
        }
      }
    } else {
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c4 = 2 * half; c4 < 2 * half + 2; ++c4) {
        uint32_t a[32], g[32];
        ptx::tmem_ld_32x32b_x32(trow + 256 + c4 * 32, a);
        ptx::tmem_ld_32x32b_x32(trow + 384 + c4 * 32, g);
        ptx::tmem_ld_wait();
        float af[32], gf[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          af[i] = __uint_as_float(a[i]);
          gf[i] = __uint_as_float(g[i]);
        }
        store_row32(dv_stage, row, c4 * 32, af, 1.f);
        store_row32(dk_stage, row, c4 * 32, gf, p.scale);
      }
    }
    ptx::fence_proxy_async_smem();
    sync_softmax_n<256>();
    if (threadIdx.x == 64 && p.dkv_ws == nullptr && !is_aborted(abort_flag)) {
      ptx::tma_store_3d(&mdv, sq, kvh * kHd, kt * kTile, b);
      ptx::tma_store_3d(&mdv, sq + kBox, kvh * kHd + 64, kt * kTile, b);
      ptx::tma_store_3d(&mdk, sq + kTileBytes, kvh * kHd, kt * kTile, b);
      ptx::tma_store_3d(&mdk, sq + kTileBytes + kBox, kvh * kHd + 64, kt * kTile, b);
      ptx::bulk_commit_group();
      ptx::bulk_wait_group_all();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// dk / dv [b, s, kvh, :] (bf16) = the sum over the group's query heads, in head
// order, of their fp32 shares in the workspace ([2][B * S][H * 128]: dK, dV).
// One thread per 4 columns of one (token, kv head, dK or dV).
__global__ void __launch_bounds__(256) attn_dkv_reduce_kernel(
    const float* __restrict__ ws, int64_t ws_half, int64_t tokens, int H, int Hkv,
    __nv_bfloat16* __restrict__ dk, int64_t lddk, __nv_bfloat16* __restrict__ dv, int64_t lddv) {
  const int rep = H / Hkv;
  const int64_t units = tokens * Hkv * 2 * (kHd / 4);
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(u % (kHd / 4)) * 4;
    const int which = static_cast<int>((u / (kHd / 4)) % 2);
    const int64_t rest = u / (kHd / 4) / 2;
    const int kvh = static_cast<int>(rest % Hkv);
    const int64_t tok = rest / Hkv;
    const float* src = ws + which * ws_half + tok * (static_cast<int64_t>(H) * kHd) +
                       static_cast<int64_t>(kvh) * rep * kHd + c;
    float4 acc = *reinterpret_cast<const float4*>(src);
    for (int r = 1; r < rep; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(src + r * kHd);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    __nv_bfloat16* dst = (which == 0 ? dk + tok * lddk : dv + tok * lddv) + kvh * kHd + c;
    const uint2 pk = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
    *reinterpret_cast<uint2*>(dst) = pk;
  }
}

constexpr int kDqBars = 11;
constexpr int kDqSmem = 7 * kTileBytes + kDqBars * 8 + 16 + 1024;

// dQ of one (b, h, 128-query tile).
__global__ void __launch_bounds__(kDqThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap mq,
                       const __grid_constant__ CUtensorMap mk,
                       const __grid_constant__ CUtensorMap mv,
                       const __grid_constant__ CUtensorMap mdo,
                       const __grid_constant__ CUtensorMap mdq,
                       const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem;                   // Q; dQ staging at the end
  uint8_t* sdo = smem + kTileBytes;
  uint8_t* sk = smem + 2 * kTileBytes;  // K ring, 2 slots
  uint8_t* sv = smem + 4 * kTileBytes;  // V ring, 2 slots
  uint8_t* sds = smem + 6 * kTileBytes; // dS (bf16)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * kTileBytes);
  uint64_t* qd_full = bars;
  uint64_t* kv_full = bars + 1;   // 2
  uint64_t* kv_empty = bars + 3;  // 2
  uint64_t* sd_full = bars + 5;   // S and dP are in TMEM
  uint64_t* sd_free = bars + 6;   // the rows have read them (512 arrivals)
  uint64_t* ds_full = bars + 7;   // dS is in shared memory (512 arrivals)
  uint64_t* dq_done = bars + 8;   // dQ += dS K complete
  uint64_t* drain = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDqBars);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int bh_count = p.B * p.H;
  const int qi = p.q_tiles - 1 - static_cast<int>(blockIdx.x) / bh_count;
  const int bh = static_cast<int>(blockIdx.x) % bh_count;
  const int b = bh / p.H, h = bh % p.H;
  const int kvh = h / (p.H / p.Hkv);
  const int n_kv = qi + 1;
  const int q0 = qi * kTile;

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&mq);
    ptx::prefetch_tmap(&mk);
    ptx::prefetch_tmap(&mv);
    ptx::prefetch_tmap(&mdo);
    for (int i = 0; i < kDqBars; ++i) ptx::mbar_init(&bars[i], 1);
    ptx::mbar_init(sd_free, 512);
    ptx::mbar_init(ds_full, 512);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);  // S [0,128), dP [128,256), dQ [256,384)
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  ptx::griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int issued = 0;
      bool ok = true;
      ptx::mbar_arrive_expect_tx(qd_full, 2 * kTileBytes);
      ptx::tma_load_3d(sq, &mq, qd_full, h * kHd, q0, b);
      ptx::tma_load_3d(sq + kBox, &mq, qd_full, h * kHd + 64, q0, b);
      ptx::tma_load_3d(sdo, &mdo, qd_full, h * kHd, q0, b);
      ptx::tma_load_3d(sdo + kBox, &mdo, qd_full, h * kHd + 64, q0, b);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !wait_bar(&kv_empty[s], ((j - 2) >> 1) & 1, p.budget, abort_flag)) {
          ok = false;
          break;
        }
        ptx::mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
        ptx::tma_load_3d(sk + s * kTileBytes, &mk, &kv_full[s], kvh * kHd, j * kTile, b);
        ptx::tma_load_3d(sk + s * kTileBytes + kBox, &mk, &kv_full[s], kvh * kHd + 64, j * kTile, b);
        ptx::tma_load_3d(sv + s * kTileBytes, &mv, &kv_full[s], kvh * kHd, j * kTile, b);
        ptx::tma_load_3d(sv + s * kTileBytes + kBox, &mv, &kv_full[s], kvh * kHd + 64, j * kTile, b);
        ++issued;
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      (void)ptx::mbar_wait(qd_full, 0, p.budget);
      for (int i = issued - 1; i >= 0 && i >= issued - 2; --i)
        (void)ptx::mbar_wait(&kv_full[i & 1], (i >> 1) & 1, p.budget);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = wait_bar(qd_full, 0, p.budget, abort_flag);
      bool issued = false;
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (j < n_kv) {  // S_j = Q K_j^T, dP_j = dO V_j^T
          const int s = j & 1;
          if (!wait_bar(&kv_full[s], (j >> 1) & 1, p.budget, abort_flag) ||
              (j >= 1 && !wait_bar(sd_free, (j - 1) & 1, p.budget, abort_flag))) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_kk(tmem, ptx::smem_u32(sq), ptx::smem_u32(sk + s * kTileBytes), false);
          mma_tile_kk(tmem + 128, ptx::smem_u32(sdo), ptx::smem_u32(sv + s * kTileBytes), false);
          issued = true;
          ptx::mma_commit(sd_full);
        }
        if (j >= 1) {  // dQ += dS_{j-1} K_{j-1}
          const int jj = j - 1, s = jj & 1;
          if (!wait_bar(ds_full, jj & 1, p.budget, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          mma_tile_kmn(tmem + 256, ptx::smem_u32(sds), ptx::smem_u32(sk + s * kTileBytes), jj > 0);
          ptx::mma_commit(dq_done);
          ptx::mma_commit(&kv_empty[s]);
        }
      }
      if (!ok) record_err(p.err, kDevErrAttnTimeout, abort_flag);
      if (issued) {
        ptx::mma_commit(drain);
        (void)ptx::mbar_wait(drain, 0, p.budget);
      }
    }
  } else {
    // ---------------- elementwise rows (warps 2..17): four threads per query row ----------------
    // Warps w, w + 4, w + 8, w + 12 share TMEM lane quarter w % 4 and take key
    // columns [32 sub, 32 sub + 32). Each reads its S and dP columns and frees
    // them at once (the next key tile's MMAs then overlap this one's dS).
    const int quarter = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int c0 = sub * 32;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t ds_base = ptx::smem_u32(sds);
    const int q = q0 + row;
    const int64_t ri = (static_cast<int64_t>(b) * p.H + h) * p.S + q;
    const float lse_r = q < p.S ? p.lse[ri] : INFINITY;
    const float delta_r = q < p.S ? p.delta[ri] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!wait_bar_warp(sd_full, j & 1, p.budget, abort_flag)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t sv32[32], dp32[32];
      ptx::tmem_ld_32x32b_x32(trow + c0, sv32);
      ptx::tmem_ld_32x32b_x32(trow + 128 + c0, dp32);
      ptx::tmem_ld_wait();
      ptx::tc_fence_before();
      ptx::mbar_arrive(sd_free);
      const bool diag = j == qi;
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float d2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float pv = ex2(__uint_as_float(sv32[2 * i + e]) * p.scale_log2 - lse_r);
          if (diag && c0 + 2 * i + e > row) pv = 0.f;  // key after query
          d2[e] = pv * (__uint_as_float(dp32[2 * i + e]) - delta_r);
        }
        pk[i] = pack_bf16x2(d2[0], d2[1]);
      }
      // dS_j goes into the one dS tile once dQ += dS_{j-1} K_{j-1} has read it
      if (j >= 1 && !wait_bar_warp(dq_done, (j - 1) & 1, p.budget, abort_flag)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        st_shared_v4(ds_base + swz_chunk(row, c0 + cc * 8), pk[cc * 4], pk[cc * 4 + 1],
                     pk[cc * 4 + 2], pk[cc * 4 + 3]);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(ds_full);
    }
    // ---------------- epilogue: scale * dQ -> bf16 -> TMA store ----------------
    if (ok && !wait_bar_warp(dq_done, (n_kv - 1) & 1, p.budget, abort_flag)) ok = false;
    if (!ok) {
      record_err(p.err, kDevErrAttnTimeout, abort_flag);
    } else {
      ptx::tc_fence_after();
      uint32_t a[32];
      ptx::tmem_ld_32x32b_x32(trow + 256 + c0, a);
      ptx::tmem_ld_wait();
      float af[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) af[i] = __uint_as_float(a[i]);
      store_row32(ptx::smem_u32(sq), row, c0, af, p.scale);
    }
    ptx::fence_proxy_async_smem();
    sync_softmax_n<512>();
    if (threadIdx.x == 64 && !is_aborted(abort_flag)) {
      ptx::tma_store_3d(&mdq, sq, h * kHd, q0, b);
      ptx::tma_store_3d(&mdq, sq + kBox, h * kHd + 64, q0, b);
      ptx::bulk_commit_group();
      ptx::bulk_wait_group_all();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host side

// 3-D map over a token-major bf16 tensor [B, S, cols] with row stride ld
// elements: box = 64 columns (128 B) x 128 tokens x 1 sequence, 128-byte
// swizzle, zero fill past S (loads) and clipping past S (stores).
int make_seq_map(CUtensorMap* map, const void* base, int64_t B, int64_t S, int64_t cols,
                 int64_t ld) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (encode == nullptr)
    return set_error(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2,
                           static_cast<cuuint64_t>(ld) * 2 * static_cast<cuuint64_t>(S)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kTile), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (code " +
                                        std::to_string(static_cast<int>(r)) + ")");
  return LEMA_OK;
}

std::atomic<long long> g_attn_budget{ptx::kWaitBudgetCycles};

// Shape and pointer checks shared by the entry points.
int check_attn(int64_t B, int64_t S, int64_t H, int64_t Hkv, int64_t head_dim) {
  if (head_dim != kHd) return set_error(LEMA_ERR_INVALID_ARGUMENT, "head_dim must be 128");
  if (B < 0 || S < 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad B / S / heads (H must be a multiple of Hkv)");
  if (B > 65535 || S > (1 << 24) || H > 1024)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "B, S or H out of range");
  return LEMA_OK;
}

int check_tensor(const void* ptr, int64_t ld, int64_t cols, const char* name) {
  if (ptr == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, std::string("null ") + name);
  if (!aligned16(ptr) || ld % 8 != 0 || ld < cols)
    return set_error(LEMA_ERR_INVALID_ARGUMENT,
                     std::string(name) + ": 16-byte aligned base and row stride >= columns, "
                                         "a multiple of 8 elements, required");
  return LEMA_OK;
}

AttnParams make_params(int64_t B, int64_t S, int64_t H, int64_t Hkv, float scale) {
  AttnParams p{};
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.H = static_cast<int>(H);
  p.Hkv = static_cast<int>(Hkv);
  p.q_tiles = static_cast<int>((S + kTile - 1) / kTile);
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.fwd_tiles_per_cta = 2;
  p.err = gemm_error_word();
  p.budget = g_attn_budget.load();
  return p;
}

template <typename Kern>
int set_smem(Kern kern, int bytes, bool* done) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(LEMA_ERR_CUDA, "bad device");
  if (!done[dev]) {
    LEMA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev] = true;
  }
  return LEMA_OK;
}

}  // namespace
}  // namespace lema

using namespace lema;

extern "C" int lema_attn_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk,
                             const void* v, int64_t ldv, void* o, int64_t ldo, float* lse,
                             int64_t B, int64_t S, int64_t H, int64_t Hkv, int64_t head_dim,
                             float scale, void* stream) {
  clear_error();
  int rc = check_attn(B, S, H, Hkv, head_dim);
  if (rc) return rc;
  if (B == 0 || S == 0) return LEMA_OK;
  if ((rc = check_tensor(q, ldq, H * kHd, "q")) || (rc = check_tensor(k, ldk, Hkv * kHd, "k")) ||
      (rc = check_tensor(v, ldv, Hkv * kHd, "v")) || (rc = check_tensor(o, ldo, H * kHd, "o")))
    return rc;
  if (lse == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null lse");
  AttnParams p = make_params(B, S, H, Hkv, scale);
  if (p.err == nullptr) return set_error(LEMA_ERR_CUDA, "cannot resolve device error word");
  p.lse = lse;
  CUtensorMap mq, mk, mv, mo;
  if ((rc = make_seq_map(&mq, q, B, S, H * kHd, ldq)) ||
      (rc = make_seq_map(&mk, k, B, S, Hkv * kHd, ldk)) ||
      (rc = make_seq_map(&mv, v, B, S, Hkv * kHd, ldv)) ||
      (rc = make_seq_map(&mo, o, B, S, H * kHd, ldo)))
    return rc;
  static bool done[64] = {};
  if ((rc = set_smem(attn_fwd_kernel, kFwdSmem, done))) return rc;
  // pairs of query tiles share their K / V loads and overlap each other's softmax with
  // the other's MMAs; below one CTA per SM, single tiles keep twice the SMs busy
  if (B * H * ((p.q_tiles + 1) / 2) < static_cast<int64_t>(device_sm_count()))
    p.fwd_tiles_per_cta = 1;
  const int64_t ctas =
      B * H * ((p.q_tiles + p.fwd_tiles_per_cta - 1) / p.fwd_tiles_per_cta);
  if (ctas > 0x7fffffff) return set_error(LEMA_ERR_INVALID_ARGUMENT, "too many tiles");
  attn_fwd_kernel<<<static_cast<unsigned>(ctas), kFwdThreads, kFwdSmem,
                    static_cast<cudaStream_t>(stream)>>>(mq, mk, mv, mo, p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_attn_set_wait_budget(int64_t cycles) {
  clear_error();
  if (cycles < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "cycles must be >= 0");
  g_attn_budget.store(cycles == 0 ? ptx::kWaitBudgetCycles : static_cast<long long>(cycles));
  return LEMA_OK;
}

extern "C" int lema_attn_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk,
                             const void* v, int64_t ldv, const void* o, int64_t ldo,
                             const void* dout, int64_t lddo, const float* lse, float* delta,
                             float* dkv_ws, void* dq, int64_t lddq, void* dk, int64_t lddk,
                             void* dv, int64_t lddv, int64_t B, int64_t S, int64_t H,
                             int64_t Hkv, int64_t head_dim, float scale, void* stream) {
  clear_error();
  int rc = check_attn(B, S, H, Hkv, head_dim);
  if (rc) return rc;
  if (B == 0 || S == 0) return LEMA_OK;
  if ((rc = check_tensor(q, ldq, H * kHd, "q")) || (rc = check_tensor(k, ldk, Hkv * kHd, "k")) ||
      (rc = check_tensor(v, ldv, Hkv * kHd, "v")) || (rc = check_tensor(o, ldo, H * kHd, "o")) ||
      (rc = check_tensor(dout, lddo, H * kHd, "dout")) ||
      (rc = check_tensor(dq, lddq, H * kHd, "dq")) ||
      (rc = check_tensor(dk, lddk, Hkv * kHd, "dk")) ||
      (rc = check_tensor(dv, lddv, Hkv * kHd, "dv")))
    return rc;
  if (lse == nullptr || delta == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null lse or delta");
  AttnParams p = make_params(B, S, H, Hkv, scale);
  if (p.err == nullptr) return set_error(LEMA_ERR_CUDA, "cannot resolve device error word");
  p.lse = const_cast<float*>(lse);
  p.delta = delta;
  // dK/dV CTAs per kv head (the group's heads in one CTA, bf16 out) unless they
  // would leave SMs idle and a workspace for per-query-head shares was given
  p.heads_per_cta = static_cast<int>(H / Hkv);
  if (H != Hkv && dkv_ws != nullptr &&
      B * Hkv * p.q_tiles < static_cast<int64_t>(device_sm_count())) {
    if (!aligned16(dkv_ws))
      return set_error(LEMA_ERR_INVALID_ARGUMENT, "dkv_ws must be 16-byte aligned");
    p.dkv_ws = dkv_ws;
    p.ws_half = B * S * H * kHd;
    p.heads_per_cta = 1;
  }
  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  if ((rc = make_seq_map(&mq, q, B, S, H * kHd, ldq)) ||
      (rc = make_seq_map(&mk, k, B, S, Hkv * kHd, ldk)) ||
      (rc = make_seq_map(&mv, v, B, S, Hkv * kHd, ldv)) ||
      (rc = make_seq_map(&mdo, dout, B, S, H * kHd, lddo)) ||
      (rc = make_seq_map(&mdq, dq, B, S, H * kHd, lddq)) ||
      (rc = make_seq_map(&mdk, dk, B, S, Hkv * kHd, lddk)) ||
      (rc = make_seq_map(&mdv, dv, B, S, Hkv * kHd, lddv)))
    return rc;
  static bool done_kv[64] = {}, done_q[64] = {};
  if ((rc = set_smem(attn_bwd_dkdv_kernel, kDkdvSmem, done_kv)) ||
      (rc = set_smem(attn_bwd_dq_kernel, kDqSmem, done_q)))
    return rc;
  const int64_t q_ctas = B * H * p.q_tiles, kv_ctas = B * (H / p.heads_per_cta) * p.q_tiles;
  if (q_ctas > 0x7fffffff) return set_error(LEMA_ERR_INVALID_ARGUMENT, "too many tiles");
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t warps = B * S * H;
  const int delta_blocks =
      static_cast<int>(std::min<int64_t>((warps + 7) / 8, static_cast<int64_t>(device_sm_count()) * 16));
  attn_delta_kernel<<<delta_blocks, 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(o), ldo, static_cast<const __nv_bfloat16*>(dout), lddo,
      delta, static_cast<int>(B), static_cast<int>(S), static_cast<int>(H));
  LEMA_CUDA_TRY(cudaGetLastError());
  attn_bwd_dkdv_kernel<<<static_cast<unsigned>(kv_ctas), kDkdvThreads, kDkdvSmem, s>>>(
      mq, mk, mv, mdo, mdk, mdv, p);
  LEMA_CUDA_TRY(cudaGetLastError());
  if (p.dkv_ws != nullptr) {
    const int64_t units = B * S * Hkv * 2 * (kHd / 4);
    const int blocks = static_cast<int>(
        std::min<int64_t>((units + 255) / 256, static_cast<int64_t>(device_sm_count()) * 8));
    attn_dkv_reduce_kernel<<<blocks, 256, 0, s>>>(
        p.dkv_ws, p.ws_half, B * S, static_cast<int>(H), static_cast<int>(Hkv),
        static_cast<__nv_bfloat16*>(dk), lddk, static_cast<__nv_bfloat16*>(dv), lddv);
    LEMA_CUDA_TRY(cudaGetLastError());
  }
  attn_bwd_dq_kernel<<<static_cast<unsigned>(q_ctas), kDqThreads, kDqSmem, s>>>(mq, mk, mv, mdo,
                                                                                mdq, p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}
