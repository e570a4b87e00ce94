// gemm_sm100.cu — K2/K3 (int8 tcgen05 GEMM + fused dequant/bias/bf16 epilogue),
// the bf16 tcgen05 GEMM used by K4 (dgrad), and K6 (grouped int8 GEMM for MoE
// experts). Two persistent, warp-specialised kernel templates serve all three:
// a 1-SM kernel (128 x BN tiles) and a CTA-pair kernel (cluster of 2, 256 x 256
// tiles, cta_group::2 MMAs), with the same roles:
//
//   warp 0      TMA producer: one thread streams 128-byte-wide K slices of the
//               A tile (128 rows) and B tile (BN rows) into a STAGES-deep ring
//               of 128B-swizzled shared-memory buffers (plain TMA, no multicast).
//   warp 1      allocates TMEM (2 x BN columns: double-buffered accumulators);
//               one thread issues tcgen05.mma (K=32 bytes per instruction) and
//               tcgen05.commit to free smem stages / publish finished
//               accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, then
//               y = bf16((float(acc) * sx[m]) * sw[n] + bias[n]) (int8 kind) or
//               y = bf16(acc) (bf16 kind), staged in 64-byte-swizzled shared
//               memory and written by TMA stores (direct stores for raw
//               accumulator outputs and unaligned y), while the MMA warp already
//               accumulates the next tile into the other TMEM buffer.
//
// Tiles are ordered in panels of column tiles inside each group (decode_tile)
// so concurrently running CTAs share A rows and B columns through L2. A
// "group" is a contiguous row range of A that multiplies its own B matrix (MoE
// experts); the dense GEMM is one group. When the tile count leaves the last
// wave part-empty, a stream-K schedule gives every worker an equal range of
// K-slices instead (plan_schedule, WorkIter): split tiles' partial
// accumulators go through a per-stream workspace to the worker that owns the
// tile. Kernels are launched with programmatic stream serialisation: their
// set-up overlaps the previous kernel's tail and griddepcontrol.wait precedes
// every data read.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include <cudaTypedefs.h>

#include "internal.h"
#include "ptx.cuh"

namespace lema {

namespace {

constexpr int kBM = 128;
constexpr int kRowBytes = 128;  // K bytes per stage row (one 128B swizzle atom row)
constexpr int kMaxGroups = 64;
// Warps: 0 = TMA producer, 1 = MMA issuer and TMEM owner, then the epilogue
// warps: 4 in the 1-SM kernel (one per TMEM lane quarter), 8 in the pair kernel
// (two per lane quarter, each converting half of the tile's columns, so the
// last tile's epilogue, which nothing overlaps, takes half as long).
constexpr int kEpiWarps1 = 4;
constexpr int kEpiWarpsPair = 8;
constexpr int kMaxEpiWarps = 8;  // publish flags per workspace slot
constexpr int threads_for(int epi_warps) { return 64 + 32 * epi_warps; }

enum GemmKind : int { kKindI8 = 0, kKindBF16 = 1 };

struct GemmParams {
  int32_t num_kb;       // K slices of 128 bytes
  int32_t n;            // columns of every group's output
  int32_t num_n_tiles;  // ceil(n / BN)
  int32_t num_groups;
  int32_t total_tiles;
  int32_t row_start[kMaxGroups + 1];   // group g owns A rows [row_start[g], row_start[g+1])
  int32_t tile_start[kMaxGroups + 1];  // first linear tile index of group g
  const float* sx;                     // [rows] per-row scale (int8 kind)
  const float* sw;                     // [groups * n] per-column scale (int8 kind)
  const __nv_bfloat16* bias;           // [groups * n] or null
  __nv_bfloat16* y;                    // may be null
  int64_t ldy;
  int32_t* acc;                        // raw s32 accumulators or null (int8 kind)
  int64_t ldacc;
  int32_t* err;                        // device error word
  // Stream-K schedule (see WorkIter): tiles [0, sk_tiles) form a row of
  // sk_tiles * num_kb K-slice units cut into sk_workers contiguous ranges, one
  // per worker (CTA, or CTA pair) w < sk_workers, processed first; tiles
  // [sk_tiles, total_tiles) then run whole, round-robin over all workers.
  int32_t sk_tiles;
  int32_t sk_workers;
  int32_t* ws;        // partial accumulators: one kSlotElems slot per CTA
  int32_t* ws_flags;  // per slot and epilogue warp: the epoch of its last publish
  int32_t epoch;      // this launch's publish value (never 0; differs from the
                      // previous launches on the same workspace)
  int32_t raster;     // column tiles per raster panel (tile order, decode_tile)
  int32_t y_tma;      // y is written by TMA stores through the y tensor map
  int32_t total_rows; // rows of A (and of y)
  int32_t skip_publish;  // test hook: partial ranges are not published
  long long wait_budget; // clock64 cycles each bounded wait may spin
};

// A partial slot holds one CTA's 128 rows x 256 columns of 32-bit accumulators
// as four 32 KB blocks, one per TMEM lane quarter (32 rows each). Inside a
// block, element (row, col) of 32-column chunk c = col / 32 sits at
// c * 1024 + ((col % 32) / 4) * 128 + row * 4 + col % 4: each lane (row) moves
// four columns with one 16-byte access, and the 32 lanes of a warp together
// cover 512 contiguous bytes.
constexpr int kSlotElems = 128 * 256;
constexpr int kSlotWarpElems = 32 * 256;

enum WorkRole : int { kRoleWhole = 0, kRolePartial = 1, kRoleOwner = 2 };

struct Work {
  int tile;
  int kb0, kb1;        // K-slices [kb0, kb1) of the tile
  int role;
  int c_first, c_last; // owner: the workers holding the tile's other K-slices
};

// First stream-K unit of worker w: floor(w * U / S) for U units on S workers.
__device__ __forceinline__ int64_t sk_start(int64_t w, int64_t units, int64_t workers) {
  return w * units / workers;
}

// The worker whose stream-K range holds unit u: the largest w with
// sk_start(w) <= u, i.e. floor(((u + 1) * S - 1) / U).
__device__ __forceinline__ int sk_worker_of(int64_t u, int64_t units, int64_t workers) {
  return static_cast<int>(((u + 1) * workers - 1) / units);
}

// The work list of one worker, identical in its producer, MMA and epilogue
// roles. Stream-K first: worker w < sk_workers walks its contiguous range of
// the units of tiles [0, sk_tiles) in order. A range starting inside a tile
// begins with a partial item (its accumulators go to the worker's slot and are
// published); a range ending inside a tile ends with that tile's head, whose
// worker owns the tile: it adds the partials of the later workers that hold
// the rest of the tile and writes it. A partial is always its worker's first
// item and an owned head its worker's last stream-K item, so no owner waits on
// a worker that is itself waiting. Then whole tiles sk_tiles + w, + W, ...
struct WorkIter {
  int W;
  int64_t u, u_end, units;
  int next_dp;
  __device__ WorkIter(const GemmParams& p, int worker, int workers) : W(workers) {
    units = static_cast<int64_t>(p.sk_tiles) * p.num_kb;
    if (worker < p.sk_workers) {
      u = sk_start(worker, units, p.sk_workers);
      u_end = sk_start(worker + 1, units, p.sk_workers);
    } else {
      u = u_end = 0;
    }
    next_dp = p.sk_tiles + worker;
  }
  __device__ bool next(const GemmParams& p, Work& out) {
    if (u < u_end) {
      const int tile = static_cast<int>(u / p.num_kb);
      const int64_t tile_u0 = static_cast<int64_t>(tile) * p.num_kb;
      const int64_t tile_u1 = tile_u0 + p.num_kb;
      const int64_t stop = tile_u1 < u_end ? tile_u1 : u_end;
      out.tile = tile;
      out.kb0 = static_cast<int>(u - tile_u0);
      out.kb1 = static_cast<int>(stop - tile_u0);
      out.c_first = out.c_last = 0;
      if (out.kb0 > 0) {
        out.role = kRolePartial;
      } else if (stop == tile_u1) {
        out.role = kRoleWhole;
      } else {
        out.role = kRoleOwner;
        out.c_first = sk_worker_of(stop, units, p.sk_workers);
        out.c_last = sk_worker_of(tile_u1 - 1, units, p.sk_workers);
      }
      u = stop;
      return true;
    }
    if (next_dp < p.total_tiles) {
      out.tile = next_dp;
      out.kb0 = 0;
      out.kb1 = p.num_kb;
      out.role = kRoleWhole;
      out.c_first = out.c_last = 0;
      next_dp += W;
      return true;
    }
    return false;
  }
};

__device__ __forceinline__ int32_t ld_acquire_gpu(const int32_t* ptr) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(int32_t* ptr, int32_t v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// Bounded wait until a warp block's partial of this launch is published (its
// flag holds this launch's epoch; a flag left by an earlier launch, aborted or
// not, holds another value). Lane 0 polls and the outcome is broadcast, so the
// whole warp takes the same branch (the epilogue's tcgen05.ld needs the full
// warp); each lane then performs its own acquire load before it reads the
// block.
__device__ __forceinline__ bool warp_wait_published(const int32_t* flag, int32_t epoch,
                                                    long long budget, int lane) {
  int ok = 1;
  if (lane == 0 && ld_acquire_gpu(flag) != epoch) {
    const long long t0 = clock64();
    while (ld_acquire_gpu(flag) != epoch) {
      if (clock64() - t0 > budget) {
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)ld_acquire_gpu(flag);
  return ok != 0;
}

__device__ int32_t g_gemm_err = 0;

__device__ __forceinline__ void record_error(int32_t* err, int32_t code, int* abort_flag) {
  atomicCAS(err, 0, code);
  *reinterpret_cast<volatile int*>(abort_flag) = 1;
}

__device__ __forceinline__ bool aborted(const int* abort_flag) {
  return *reinterpret_cast<const volatile int*>(abort_flag) != 0;
}

// Linear tile index -> (group, first A row, end row of the group, column tile)
// for tiles TM rows high. Inside a group the tiles are ordered in panels of
// p.raster column tiles: panel by panel, and inside a panel row tile by row
// tile with the panel's column tiles fastest (the last panel may be narrower).
// Workers running consecutive tiles then cover a compact block of rows and
// columns, so the A rows and B columns they read stay in L2 between them.
template <int TM>
__device__ __forceinline__ void decode_tile(const GemmParams& p, int t, int& g, int& row0,
                                            int& row_end, int& n_tile) {
  g = 0;
  while (g + 1 < p.num_groups && t >= p.tile_start[g + 1]) ++g;
  const int local = t - p.tile_start[g];
  const int rows = p.row_start[g + 1] - p.row_start[g];
  const int m_tiles = (rows + TM - 1) / TM;
  const int panel = local / (m_tiles * p.raster);
  const int r = local - panel * m_tiles * p.raster;
  const int rest = p.num_n_tiles - panel * p.raster;
  const int width = rest < p.raster ? rest : p.raster;
  const int mt = r / width;
  const int nt = panel * p.raster + (r - mt * width);
  row0 = p.row_start[g] + mt * TM;
  row_end = p.row_start[g + 1];
  n_tile = nt;
}

// BROWS: B rows a CTA loads per stage; EPI: epilogue warps; ECOLS: output
// columns one epilogue warp converts per tile.
template <int BROWS, int STAGES, int EPI, int ECOLS>
struct SmemLayout {
  static constexpr int kABytes = kBM * kRowBytes;
  static constexpr int kBBytes = BROWS * kRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], then tmem addr + abort flag
  static constexpr int kBarBytes = (2 * STAGES + 4) * 8 + 16;
  // Per epilogue warp: two 2 KB staging buffers for TMA stores (32 rows x 64 B,
  // 64-byte swizzle, 1024-byte aligned), then the warp's ECOLS column scales
  // (fp32) and biases (bf16) of the current tile.
  static constexpr int kEpiOffset = (kBarOffset + kBarBytes + 1023) / 1024 * 1024;
  static constexpr int kEpiSwOffset = 4096;
  static constexpr int kEpiBiasOffset = kEpiSwOffset + ECOLS * 4;
  static constexpr int kEpiWarpBytes = (kEpiBiasOffset + ECOLS * 2 + 1023) / 1024 * 1024;
  static constexpr int kTotal = kEpiOffset + EPI * kEpiWarpBytes + 1024;  // + alignment slack
  static_assert(kTotal <= 227 * 1024, "shared memory per CTA");
};

constexpr int kEpiStageBytes = 2048;

// Other workers' K-ranges of a tile this worker owns: `count` partial blocks in
// the workspace, `stride` elements apart, each in the block layout above.
struct Partials {
  const int32_t* first;
  int count;
  int64_t stride;
};

// v[j] += the partials' column j of this lane's row in chunk `chunk`, for every
// partial block, in contributor order (exact for s32; one fp32 add each for
// bf16). The blocks were written by other SMs: the loads go to L2
// (ld.global.cg), past this SM's L1.
template <int KIND>
__device__ __forceinline__ void add_partials(uint32_t (&v)[32], const Partials& parts,
                                             int chunk, int lane) {
#pragma unroll 1
  for (int i = 0; i < parts.count; ++i) {
    const int4* pc = reinterpret_cast<const int4*>(parts.first + i * parts.stride +
                                                   chunk * 1024 + lane * 4);
    int32_t add[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int4 a = __ldcg(pc + q * 32);
      add[4 * q] = a.x;
      add[4 * q + 1] = a.y;
      add[4 * q + 2] = a.z;
      add[4 * q + 3] = a.w;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (KIND == kKindI8)
        v[j] = static_cast<uint32_t>(static_cast<int32_t>(v[j]) + add[j]);
      else
        v[j] = __float_as_uint(__fadd_rn(__uint_as_float(v[j]), __int_as_float(add[j])));
    }
  }
}

// Epilogue of one warp's 32 rows x (NCHUNK*32) columns of accumulators held in
// TMEM columns [col0, col0 + NCHUNK*32) of the warp's lane quarter. Row r of
// the output is this thread's row; columns start at n0. Chunk c of the warp is
// chunk chunk_base + c of the quarter's 32 x 256 partial block. slot != null
// (a partial K-range): the raw accumulators go to the warp's chunks of the slot
// block and nothing else is written. parts.count > 0 (the owner of a split
// tile): the other workers' partial chunks are added first.
template <int KIND, int NCHUNK>
__device__ __forceinline__ void epilogue_rows(const GemmParams& p, uint32_t tmem_row_base,
                                              uint32_t col0, int r, bool rvalid, int g, int n0,
                                              int chunk_base, bool y_vec, bool acc_vec, int lane,
                                              const Partials& parts, int32_t* slot) {
  float sxr = 0.f;
  if (KIND == kKindI8 && rvalid && p.sx != nullptr) sxr = p.sx[r];
  // no column scales (sw null): every column scale is 1
  const float* swg =
      (KIND == kKindI8 && p.sw != nullptr) ? p.sw + static_cast<int64_t>(g) * p.n : nullptr;
  const __nv_bfloat16* bg = p.bias != nullptr ? p.bias + static_cast<int64_t>(g) * p.n : nullptr;
#pragma unroll 1
  for (int c = 0; c < NCHUNK; ++c) {
    uint32_t v[32];
    __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp issues it together
    ptx::tmem_ld_32x32b_x32(tmem_row_base + col0 + static_cast<uint32_t>(c * 32), v);
    ptx::tmem_ld_wait();
    if (slot != nullptr) {
      int4* sc = reinterpret_cast<int4*>(slot + (chunk_base + c) * 1024 + lane * 4);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        sc[q * 32] = make_int4(static_cast<int32_t>(v[4 * q]), static_cast<int32_t>(v[4 * q + 1]),
                               static_cast<int32_t>(v[4 * q + 2]),
                               static_cast<int32_t>(v[4 * q + 3]));
      continue;
    }
    const int n = n0 + c * 32;
    if (!rvalid || n >= p.n) continue;
    if (parts.count > 0) add_partials<KIND>(v, parts, chunk_base + c, lane);
    const bool full_chunk = (n + 32) <= p.n;
    if (p.acc != nullptr) {  // raw accumulators: s32 (int8 kind) or fp32 bits (bf16 kind)
      int32_t* arow = p.acc + static_cast<int64_t>(r) * p.ldacc + n;
      if (full_chunk && acc_vec) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<uint4*>(arow + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < 32 && n + j < p.n; ++j) arow[j] = static_cast<int32_t>(v[j]);
      }
    }
    if (p.y == nullptr) continue;
    __align__(16) __nv_bfloat16 out[32];
    if (KIND == kKindI8) {
      if (full_chunk) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float f = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j])), sxr),
                              swg != nullptr ? __ldg(swg + n + j) : 1.f);
          if (bg != nullptr) f = __fadd_rn(f, __bfloat162float(bg[n + j]));
          out[j] = __float2bfloat16_rn(f);
        }
      } else {
        for (int j = 0; j < 32 && n + j < p.n; ++j) {
          float f = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j])), sxr),
                              swg != nullptr ? swg[n + j] : 1.f);
          if (bg != nullptr) f = __fadd_rn(f, __bfloat162float(bg[n + j]));
          out[j] = __float2bfloat16_rn(f);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float f = __uint_as_float(v[j]);
        if (bg != nullptr && n + j < p.n) f = __fadd_rn(f, __bfloat162float(bg[n + j]));
        out[j] = __float2bfloat16_rn(f);
      }
    }
    __nv_bfloat16* yrow = p.y + static_cast<int64_t>(r) * p.ldy + n;
    if (full_chunk && y_vec) {
      const uint4* src = reinterpret_cast<const uint4*>(out);
#pragma unroll
      for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(yrow)[j] = src[j];
    } else {
      for (int j = 0; j < 32 && n + j < p.n; ++j) yrow[j] = out[j];
    }
  }
}

// Stages one epilogue warp's ECOLS column scales (fp32; 1 without column
// scales) and biases (bf16) of a tile, from column n0 on, into its shared
// memory: issued before the warp waits for the tile's accumulators, so the
// global loads overlap the tile's MMAs. Columns >= n get zeros.
template <int KIND, int ECOLS>
__device__ __forceinline__ void stage_scales(const GemmParams& p, float* sw_s,
                                             __nv_bfloat16* bias_s, int g, int n0, int lane) {
  __syncwarp();  // every lane is done with the previous tile's scales
#pragma unroll
  for (int j = 0; j < ECOLS / 32; ++j) {
    const int c = lane * (ECOLS / 32) + j;
    const int n = n0 + c;
    const bool in = n < p.n;
    if (KIND == kKindI8)
      sw_s[c] = !in ? 0.f : p.sw != nullptr ? __ldg(p.sw + static_cast<int64_t>(g) * p.n + n) : 1.f;
    if (p.bias != nullptr)
      bias_s[c] = in ? p.bias[static_cast<int64_t>(g) * p.n + n] : __float2bfloat16_rn(0.f);
  }
  __syncwarp();
}

// Epilogue of one warp's 32 rows x (NCHUNK*32) columns through shared memory
// and TMA stores: per 32-column chunk, the warp's results (one row per lane,
// 64 B) go to a 64-byte-swizzled staging buffer (conflict-free 16-byte writes)
// and one lane stores the 32 x 32 block with cp.async.bulk.tensor; two buffers
// alternate so the next chunk is computed while the previous one is stored.
// The column scales and biases (stage_scales) are read from shared memory as
// warp-wide broadcasts; sxr is this lane's row scale. This keeps the
// epilogue's traffic through the SM's L1/shared-memory path small: that path
// also carries the main loop's TMA writes and MMA operand reads. Row
// r_base + lane of the output; rows past the tensor map's extent and columns
// >= n are clipped.
template <int KIND, int NCHUNK>
__device__ __forceinline__ void epilogue_tma(const GemmParams& p, const CUtensorMap* tmap_y,
                                             uint8_t* epi, const float* sw_s,
                                             const __nv_bfloat16* bias_s, float sxr,
                                             uint32_t& store_count, uint32_t tmem_row_base,
                                             uint32_t col0, int r_base, int lane, int n0,
                                             int chunk_base, const Partials& parts) {
  const bool has_bias = p.bias != nullptr;
#pragma unroll 1
  for (int c = 0; c < NCHUNK; ++c) {
    uint32_t v[32];
    __syncwarp();
    ptx::tmem_ld_32x32b_x32(tmem_row_base + col0 + static_cast<uint32_t>(c * 32), v);
    ptx::tmem_ld_wait();
    const int n = n0 + c * 32;
    if (n >= p.n) continue;  // uniform over the warp
    if (parts.count > 0) add_partials<KIND>(v, parts, chunk_base + c, lane);
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float f[4];
      if (KIND == kKindI8) {
        const float4 s4 = *reinterpret_cast<const float4*>(sw_s + c * 32 + j);
        f[0] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j])), sxr), s4.x);
        f[1] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j + 1])), sxr), s4.y);
        f[2] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j + 2])), sxr), s4.z);
        f[3] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j + 3])), sxr), s4.w);
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) f[t] = __uint_as_float(v[j + t]);
      }
      if (has_bias) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
          f[t] = __fadd_rn(f[t], __bfloat162float(bias_s[c * 32 + j + t]));
      }
      const __nv_bfloat162 lo = __floats2bfloat162_rn(f[0], f[1]);
      const __nv_bfloat162 hi = __floats2bfloat162_rn(f[2], f[3]);
      packed[j / 2] = *reinterpret_cast<const uint32_t*>(&lo);
      packed[j / 2 + 1] = *reinterpret_cast<const uint32_t*>(&hi);
    }
    uint8_t* buf = epi + (store_count & 1u) * kEpiStageBytes;
    if (lane == 0) ptx::bulk_wait_group_read<1>();  // this buffer's previous store has read it
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int phys = q ^ ((lane >> 1) & 3);  // 64-byte swizzle: 16-B chunk ^ row bits [1,3)
      *reinterpret_cast<uint4*>(buf + lane * 64 + phys * 16) =
          make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      ptx::tma_store_2d(tmap_y, buf, n, r_base);
      ptx::bulk_commit_group();
    }
    ++store_count;
  }
}

// Epilogue of one work item by one epilogue warp (CTAS = CTAs per worker,
// quarter = the warp's 32-row block of the CTA's 128 rows, ew = its index among
// the CTA's epilogue warps). The owner of a split tile first waits for the
// matching warp of every contributor to publish its chunks of this launch,
// then adds them while it converts the tile. Returns false when such a wait
// ran out (the error is recorded).
template <int KIND, int NCHUNK, int CTAS>
__device__ __forceinline__ bool epilogue_work(const GemmParams& p, const Work& w, int worker,
                                              int rank, const CUtensorMap* tmap_y, uint8_t* epi,
                                              const float* sw_s, const __nv_bfloat16* bias_s,
                                              float sxr, uint32_t& store_count,
                                              uint32_t tmem_row_base, uint32_t col0, int r_base,
                                              int row_end, int g, int n0, int chunk_base,
                                              bool y_vec, bool acc_vec, int quarter, int ew,
                                              int lane, int* abort_flag) {
  if (r_base >= row_end) return true;  // no row of this warp is in the tile (owner and
                                       // contributors agree: same tile, same rows)
  const int r = r_base + lane;
  const bool rvalid = r < row_end;
  Partials parts{nullptr, 0, static_cast<int64_t>(CTAS) * kSlotElems};
  int32_t* slot = nullptr;
  if (w.role == kRoleOwner) {
    for (int c = w.c_first; c <= w.c_last; ++c) {
      const int cslot = c * CTAS + rank;
      if (!warp_wait_published(p.ws_flags + cslot * kMaxEpiWarps + ew, p.epoch, p.wait_budget,
                               lane)) {
        record_error(p.err, kDevErrSplitTimeout, abort_flag);
        return false;
      }
    }
    parts.first = p.ws + static_cast<int64_t>(w.c_first * CTAS + rank) * kSlotElems +
                  quarter * kSlotWarpElems;
    parts.count = w.c_last - w.c_first + 1;
  } else if (w.role == kRolePartial) {
    slot = p.ws + static_cast<int64_t>(worker * CTAS + rank) * kSlotElems +
           quarter * kSlotWarpElems;
  }
  // TMA stores when the warp's 32 rows are all in the group, or the rows past
  // the group's end are past y's end too (the tensor map clips them).
  const bool tma = p.y_tma && p.acc == nullptr && slot == nullptr &&
                   (r_base + 32 <= row_end || row_end >= p.total_rows);
  if (tma)
    epilogue_tma<KIND, NCHUNK>(p, tmap_y, epi, sw_s, bias_s, sxr, store_count, tmem_row_base,
                               col0, r_base, lane, n0, chunk_base, parts);
  else
    epilogue_rows<KIND, NCHUNK>(p, tmem_row_base, col0, r, rvalid, g, n0, chunk_base, y_vec,
                                acc_vec, lane, parts, slot);
  return true;
}

// After the warp's part of a work item: a partial block is published (each
// lane's stores made visible, then the warp's flag set to this launch's
// epoch). Owners leave the flags as they are: the next launch on the same
// workspace publishes and waits for another epoch.
template <int CTAS>
__device__ __forceinline__ void epilogue_publish(const GemmParams& p, const Work& w, int worker,
                                                 int rank, int ew, int lane, bool active) {
  if (!active || w.role != kRolePartial || p.skip_publish) return;
  __threadfence();
  __syncwarp();
  if (lane == 0)
    st_release_gpu(p.ws_flags + (worker * CTAS + rank) * kMaxEpiWarps + ew, p.epoch);
}

// ------------------------------ 1-SM kernel --------------------------------

template <int KIND, int BN, int STAGES>
__global__ void __launch_bounds__(threads_for(kEpiWarps1), 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tma_a,
                      const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_y,
                      const __grid_constant__ GemmParams p) {
  using L = SmemLayout<BN, STAGES, kEpiWarps1, BN>;
  constexpr int kTmemCols = 2 * BN;  // 256 or 512: a power of two >= 32
  constexpr int kElemsPerRow = (KIND == kKindI8) ? 128 : 64;
  constexpr int kKStepBytes = 32;  // K=32 int8 or K=16 bf16 per MMA instruction
  constexpr uint32_t kIdesc =
      (KIND == kKindI8) ? ptx::idesc_i8_s32(kBM, BN) : ptx::idesc_bf16_f32(kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&tma_a);
    ptx::prefetch_tmap(&tma_b);
    if (p.y_tma) ptx::prefetch_tmap(&tma_y);
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&tmem_full[b], 1);
      ptx::mbar_init(&tmem_empty[b], 32 * kEpiWarps1);  // every epilogue thread arrives
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the set-up above overlaps the previous kernel's tail (programmatic launch);
  // operands, scales and the split workspace are read only after this
  ptx::griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;  // loads issued so far; load i used stage i % STAGES
      WorkIter it(p, blockIdx.x, gridDim.x);
      Work w;
      while (!aborted(abort_flag) && it.next(p, w)) {
        int g, row0, row_end, nt;
        decode_tile<kBM>(p, w.tile, g, row0, row_end, nt);
        const int b_row0 = g * p.n + nt * BN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, p.wait_budget)) {
            record_error(p.err, kDevErrProducerTimeout, abort_flag);
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          ptx::tma_load_2d(smem_a + stage * L::kABytes, &tma_a, &full[stage],
                           kb * kElemsPerRow, row0);
          ptx::tma_load_2d(smem_b + stage * L::kBBytes, &tma_b, &full[stage],
                           kb * kElemsPerRow, b_row0);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted(abort_flag)) {
        // Drain: the last (up to STAGES) issued loads must land before this
        // CTA's shared memory is released.
        for (int64_t i = issued - 1; i >= 0 && i >= issued - STAGES; --i)
          (void)ptx::mbar_wait(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1),
                              p.wait_budget);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued_any = false;
      WorkIter it(p, blockIdx.x, gridDim.x);
      Work w;
      while (!aborted(abort_flag) && it.next(p, w)) {
        if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.wait_budget)) {
          record_error(p.err, kDevErrMmaTimeout, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, p.wait_budget)) {
            record_error(p.err, kDevErrMmaTimeout, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(smem_a + stage * L::kABytes);
          const uint32_t b_addr = ptx::smem_u32(smem_b + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kRowBytes / kKStepBytes; ++k) {
            const uint64_t ad = ptx::desc_kmajor_sw128(a_addr + k * kKStepBytes);
            const uint64_t bd = ptx::desc_kmajor_sw128(b_addr + k * kKStepBytes);
            const uint32_t accumulate = (kb > w.kb0 || k > 0) ? 1u : 0u;
            if (KIND == kKindI8)
              ptx::mma_i8(d_tmem, ad, bd, kIdesc, accumulate);
            else
              ptx::mma_bf16(d_tmem, ad, bd, kIdesc, accumulate);
          }
          issued_any = true;
          ptx::mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::mma_commit(&tmem_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (aborted(abort_flag) && issued_any) {
        // Drain outstanding MMAs before TMEM is released.
        ptx::mma_commit(&tmem_full[acc]);
        (void)ptx::mbar_wait(&tmem_full[acc], acc_phase, p.wait_budget);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may read: [32q, 32q+32)
    const int ew = warp - 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool y_vec = p.y != nullptr && (p.ldy % 8) == 0 &&
                       (reinterpret_cast<uintptr_t>(p.y) & 15u) == 0;
    const bool acc_vec = p.acc != nullptr && (p.ldacc % 4) == 0 &&
                         (reinterpret_cast<uintptr_t>(p.acc) & 15u) == 0;
    uint8_t* epi = smem + L::kEpiOffset + ew * L::kEpiWarpBytes;
    float* sw_s = reinterpret_cast<float*>(epi + L::kEpiSwOffset);
    __nv_bfloat16* bias_s = reinterpret_cast<__nv_bfloat16*>(epi + L::kEpiBiasOffset);
    uint32_t store_count = 0;
    WorkIter it(p, blockIdx.x, gridDim.x);
    Work w;
    while (it.next(p, w)) {
      int g, row0, row_end, nt;
      decode_tile<kBM>(p, w.tile, g, row0, row_end, nt);
      const int r_base = row0 + quarter * 32;
      float sxr = 0.f;
      if (r_base < row_end) {  // scales first: their loads overlap the tile's MMAs
        stage_scales<KIND, BN>(p, sw_s, bias_s, g, nt * BN, lane);
        if (KIND == kKindI8 && r_base + lane < row_end) sxr = p.sx[r_base + lane];
      }
      if (!ptx::mbar_wait(&tmem_full[acc], acc_phase, p.wait_budget)) {
        record_error(p.err, kDevErrEpilogueTimeout, abort_flag);
        break;
      }
      if (aborted(abort_flag)) break;
      ptx::tc_fence_after();
      const bool ok = epilogue_work<KIND, BN / 32, 1>(
          p, w, blockIdx.x, 0, &tma_y, epi, sw_s, bias_s, sxr, store_count,
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16),
          static_cast<uint32_t>(acc * BN), r_base, row_end, g, nt * BN, 0, y_vec, acc_vec,
          quarter, ew, lane, abort_flag);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tmem_empty[acc]);
      if (!ok) break;
      epilogue_publish<1>(p, w, blockIdx.x, 0, ew, lane, r_base < row_end);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) ptx::bulk_wait_group_all();  // stores done before shared memory is released
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------ 2-SM kernel --------------------------------
// A CTA pair (cluster of 2) computes a 256 x 256 tile with cta_group::2 MMAs
// (M=256, N=256, K=32 bytes): CTA r loads A rows [256i + 128r, +128) and B rows
// [256j + 128r, +128) into its own shared memory; the even (leader) CTA's
// single MMA thread reads both CTAs' buffers, and each CTA's TMEM receives the
// accumulators of its own 128 A rows x all 256 columns. Per SM this halves
// the B bytes moved through L2 and shared memory compared with 128 x 256 tiles.
//
// Barriers: the leader's full[s] counts both CTAs' TMA bytes (the follower's
// loads name the leader's barrier); empty[s] and tmem_full[b] exist in both
// CTAs and receive the leader's multicast commits; the leader's tmem_empty[b]
// collects one arrival per epilogue warp of both CTAs (8).

template <int KIND, int STAGES>
__global__ void __launch_bounds__(threads_for(kEpiWarpsPair), 1)
    gemm_sm100_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                           const __grid_constant__ CUtensorMap tma_b,
                           const __grid_constant__ CUtensorMap tma_y,
                           const __grid_constant__ GemmParams p) {
  constexpr int kTM = 256, kTN = 256;
  constexpr int kSplit = kEpiWarpsPair / 4;      // epilogue warps per TMEM lane quarter
  constexpr int kWarpCols = kTN / kSplit;        // output columns per epilogue warp
  // per CTA: 128 A rows + 128 B rows per stage
  using L = SmemLayout<128, STAGES, kEpiWarpsPair, kWarpCols>;
  constexpr int kTmemCols = 2 * kTN;  // double-buffered 128 x 256 accumulators
  constexpr int kElemsPerRow = (KIND == kKindI8) ? 128 : 64;
  constexpr int kKStepBytes = 32;
  constexpr uint32_t kIdesc =
      (KIND == kKindI8) ? ptx::idesc_i8_s32(kTM, kTN) : ptx::idesc_bf16_f32(kTM, kTN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = (rank & 1u) == 0;
  const int pair = blockIdx.x / 2;
  const int npairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&tma_a);
    ptx::prefetch_tmap(&tma_b);
    if (p.y_tma) ptx::prefetch_tmap(&tma_y);
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&tmem_full[b], 1);
      ptx::mbar_init(&tmem_empty[b], 2 * kEpiWarpsPair);  // lane 0 of every epilogue warp
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  __syncwarp();
  ptx::cluster_sync();  // barriers of both CTAs initialised before any remote use
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the set-up above overlaps the previous kernel's tail (programmatic launch);
  // operands, scales and the split workspace are read only after this
  ptx::griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      WorkIter it(p, pair, npairs);
      Work w;
      while (!aborted(abort_flag) && it.next(p, w)) {
        int g, row0, row_end, nt;
        decode_tile<kTM>(p, w.tile, g, row0, row_end, nt);
        const int a_row = row0 + static_cast<int>(rank) * 128;
        const int b_row = g * p.n + nt * kTN + static_cast<int>(rank) * 128;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, p.wait_budget)) {
            record_error(p.err, kDevErrProducerTimeout, abort_flag);
            break;
          }
          if (leader) ptx::mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t lbar = ptx::smem_u32(&full[stage]) & ptx::kPeerBitMask;
          ptx::tma_load_2d_pair(smem_a + stage * L::kABytes, &tma_a, lbar, kb * kElemsPerRow,
                                a_row);
          ptx::tma_load_2d_pair(smem_b + stage * L::kBBytes, &tma_b, lbar, kb * kElemsPerRow,
                                b_row);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted(abort_flag) && leader) {
        // The leader's full barriers count both CTAs' bytes: drain them before
        // either CTA can pass the final cluster barrier.
        for (int64_t i = issued - 1; i >= 0 && i >= issued - STAGES; --i)
          (void)ptx::mbar_wait(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1),
                              p.wait_budget);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA only) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued_any = false;
      WorkIter it(p, pair, npairs);
      Work w;
      while (!aborted(abort_flag) && it.next(p, w)) {
        if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.wait_budget)) {
          record_error(p.err, kDevErrMmaTimeout, abort_flag);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTN);
        bool ok = true;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, p.wait_budget)) {
            record_error(p.err, kDevErrMmaTimeout, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(smem_a + stage * L::kABytes);
          const uint32_t b_addr = ptx::smem_u32(smem_b + stage * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kRowBytes / kKStepBytes; ++k) {
            const uint64_t ad = ptx::desc_kmajor_sw128(a_addr + k * kKStepBytes);
            const uint64_t bd = ptx::desc_kmajor_sw128(b_addr + k * kKStepBytes);
            const uint32_t accumulate = (kb > w.kb0 || k > 0) ? 1u : 0u;
            if (KIND == kKindI8)
              ptx::mma_i8_pair(d_tmem, ad, bd, kIdesc, accumulate);
            else
              ptx::mma_bf16_pair(d_tmem, ad, bd, kIdesc, accumulate);
          }
          issued_any = true;
          ptx::mma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ptx::mma_commit_pair(&tmem_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (aborted(abort_flag) && issued_any) {
        ptx::mma_commit_pair(&tmem_full[acc], 0x1);
        (void)ptx::mbar_wait(&tmem_full[acc], acc_phase, p.wait_budget);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may read: [32q, 32q+32)
    const int ew = warp - 2;
    const int half = ew / 4;       // which kWarpCols columns of the tile this warp converts
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool y_vec = p.y != nullptr && (p.ldy % 8) == 0 &&
                       (reinterpret_cast<uintptr_t>(p.y) & 15u) == 0;
    const bool acc_vec = p.acc != nullptr && (p.ldacc % 4) == 0 &&
                         (reinterpret_cast<uintptr_t>(p.acc) & 15u) == 0;
    const uint32_t leader_tmem_empty0 = ptx::mapa_shared(ptx::smem_u32(&tmem_empty[0]), rank & ~1u);
    const int crank = static_cast<int>(rank & 1u);
    uint8_t* epi = smem + L::kEpiOffset + ew * L::kEpiWarpBytes;
    float* sw_s = reinterpret_cast<float*>(epi + L::kEpiSwOffset);
    __nv_bfloat16* bias_s = reinterpret_cast<__nv_bfloat16*>(epi + L::kEpiBiasOffset);
    uint32_t store_count = 0;
    WorkIter it(p, pair, npairs);
    Work w;
    while (it.next(p, w)) {
      int g, row0, row_end, nt;
      decode_tile<kTM>(p, w.tile, g, row0, row_end, nt);
      const int r_base = row0 + crank * 128 + quarter * 32;
      const int n0 = nt * kTN + half * kWarpCols;
      float sxr = 0.f;
      if (r_base < row_end) {  // scales first: their loads overlap the tile's MMAs
        stage_scales<KIND, kWarpCols>(p, sw_s, bias_s, g, n0, lane);
        if (KIND == kKindI8 && r_base + lane < row_end) sxr = p.sx[r_base + lane];
      }
      if (!ptx::mbar_wait(&tmem_full[acc], acc_phase, p.wait_budget)) {
        record_error(p.err, kDevErrEpilogueTimeout, abort_flag);
        break;
      }
      if (aborted(abort_flag)) break;
      ptx::tc_fence_after();
      const bool ok = epilogue_work<KIND, kWarpCols / 32, 2>(
          p, w, pair, crank, &tma_y, epi, sw_s, bias_s, sxr, store_count,
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16),
          static_cast<uint32_t>(acc * kTN + half * kWarpCols), r_base, row_end, g, n0,
          half * (kWarpCols / 32), y_vec, acc_vec, quarter, ew, lane, abort_flag);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(leader_tmem_empty0 + static_cast<uint32_t>(acc * 8));
      if (!ok) break;
      epilogue_publish<2>(p, w, pair, crank, ew, lane, r_base < row_end);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) ptx::bulk_wait_group_all();  // stores done before shared memory is released
  }

  ptx::tc_fence_before();
  __syncwarp();
  ptx::cluster_sync();  // both CTAs done with TMEM, remote arrivals and loads
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D K-major operand map: `rows` rows of `k` elements, row stride `ld`
// elements, box = 128 bytes of K x box_rows rows, 128-byte swizzle, zero fill.
int make_operand_map(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                     int elem_bytes, int64_t rows, int64_t k, int64_t ld, int box_rows) {
  auto encode = get_encode_fn();
  if (encode == nullptr)
    return set_error(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * elem_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kRowBytes / elem_bytes),
                       static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " +
                                        std::to_string(static_cast<int>(r)) + ")");
  return LEMA_OK;
}

// Output map for the TMA-store epilogue: bf16 [rows, n] with row stride ldy,
// box = 32 columns (64 B) x 32 rows, 64-byte swizzle.
int make_y_map(CUtensorMap* map, void* y, int64_t rows, int64_t n, int64_t ldy) {
  auto encode = get_encode_fn();
  if (encode == nullptr)
    return set_error(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldy) * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled (y) failed (code " +
                                        std::to_string(static_cast<int>(r)) + ")");
  return LEMA_OK;
}

template <int KIND, int BN, int STAGES>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my,
           const GemmParams& p, int workers, cudaStream_t stream) {
  using L = SmemLayout<BN, STAGES, kEpiWarps1, BN>;
  auto kern = gemm_sm100_kernel<KIND, BN, STAGES>;
  static bool attr_done[64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(LEMA_ERR_CUDA, "bad device");
  if (!attr_done[dev]) {
    LEMA_CUDA_TRY(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(workers);
  cfg.blockDim = dim3(threads_for(kEpiWarps1));
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LEMA_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ma, mb, my, p));
  return LEMA_OK;
}

constexpr int kPairStages = 5;
using PairLayout = SmemLayout<128, kPairStages, kEpiWarpsPair, 256 / (kEpiWarpsPair / 4)>;

// Pairs (clusters of 2 CTAs, 1 CTA per SM) the device can keep resident.
template <int KIND>
int pair_slots() {
  using L = PairLayout;
  auto kern = gemm_sm100_pair_kernel<KIND, kPairStages>;
  static int cache[64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return 0;
  if (cache[dev] == 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
        cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (device_sm_count() / 2));
    cfg.blockDim = dim3(threads_for(kEpiWarpsPair));
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = device_sm_count() / 2;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

template <int KIND>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my,
                const GemmParams& p, int workers, cudaStream_t stream) {
  using L = PairLayout;
  auto kern = gemm_sm100_pair_kernel<KIND, kPairStages>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(2 * workers);
  cfg.blockDim = dim3(threads_for(kEpiWarpsPair));
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  LEMA_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ma, mb, my, p));
  return LEMA_OK;
}

int32_t* gemm_err_ptr() {
  int32_t* ptr = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_gemm_err) != cudaSuccess)
    return nullptr;
  return ptr;
}

struct Groups {
  int num = 0;
  int64_t row_start[kMaxGroups + 1];
};

// ---- stream-K: plan and per-stream workspace -------------------------------

thread_local bool t_no_split = false;

// Test hooks (lema_gemm_set_test_hooks): read at every launch.
std::atomic<int32_t> g_skip_publish{0};
std::atomic<long long> g_wait_budget{ptx::kWaitBudgetCycles};

struct SplitWorkspace {
  int32_t* slots = nullptr;
  int32_t* flags = nullptr;
  int32_t epoch = 0;  // the last epoch handed to a launch on this workspace
  bool failed = false;
};

std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, SplitWorkspace> g_ws;
constexpr size_t kMaxSplitWorkspaces = 8;  // (device, stream) pairs, 19 MB each on B200

// Partial slots for every CTA of a full grid (one per SM: 128 KB each) and
// their publish flags, allocated once per (device, stream) so that GEMMs on
// different streams never share them; GEMMs on one stream run in order. Each
// launch gets the workspace's next epoch, which its partials publish and its
// owners wait for, so flags left by an earlier launch (finished or aborted)
// never pass for this launch's. None while this thread holds a
// ScopedNoGemmWorkspace, or while the stream is being captured into a graph (a
// replay may run on another stream).
bool split_workspace(cudaStream_t stream, int32_t** slots, int32_t** flags, int32_t* epoch) {
  if (t_no_split) return false;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  if (cap != cudaStreamCaptureStatusNone) return false;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_ws_mu);
  if (g_ws.size() >= kMaxSplitWorkspaces && g_ws.find({dev, stream}) == g_ws.end())
    return false;  // bounded: GEMMs on further streams run whole tiles
  SplitWorkspace& w = g_ws[{dev, stream}];
  if (w.failed) return false;
  if (w.slots == nullptr) {
    const size_t n = static_cast<size_t>(device_sm_count());
    const size_t slot_bytes = n * kSlotElems * sizeof(int32_t);
    const size_t flag_bytes = n * kMaxEpiWarps * sizeof(int32_t);  // per slot and epilogue warp
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, slot_bytes + flag_bytes) != cudaSuccess) {
      (void)cudaGetLastError();
      w.failed = true;
      return false;
    }
    if (cudaMemset(static_cast<uint8_t*>(ptr) + slot_bytes, 0, flag_bytes) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      (void)cudaFree(ptr);
      w.failed = true;
      return false;
    }
    w.slots = static_cast<int32_t*>(ptr);
    w.flags = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ptr) + slot_bytes);
  }
  w.epoch = w.epoch == INT32_MAX ? 1 : w.epoch + 1;  // never 0, the flags' initial value
  *slots = w.slots;
  *flags = w.flags;
  *epoch = w.epoch;
  return true;
}

// Stream-K plan. T tiles of KB K-slices (128 bytes of K each) on W workers:
// whole tiles take ceil(T / W) waves, so when T is not a multiple of W the
// last wave leaves workers idle. Stream-K instead gives every worker the same
// number of K-slice units: the R = T mod W tiles of the part-empty wave are
// cut into contiguous unit ranges over all W workers (at most one worker per
// kMinUnits units), run first, and the other F * W tiles (F = floor(T / W))
// follow whole, F per worker, every worker on the same K-slice of its tile at
// the same time (so concurrently running tiles share their operands in L2).
// Each split tile costs its owner a fix-up (waiting for and adding the
// partials), hidden behind its next tile's MMAs because partials are every
// worker's first item; the plan is used for tiles of at least kMinSlices
// K-slices when its makespan, in K-slice times plus kFixupSlices, beats the
// waves. Measured on B200 (interleaved, 256 x 256 tiles): -9 % at int8
// K = 11008 (86 slices); +3 to +5 % at K = 4096 (32 slices), where the
// partials' exchange and the owners' fix-ups cost more than the part-empty
// wave, and where whole tiles also let the next launch's set-up start on the
// SMs the last wave leaves idle.
// LEMA_GEMM_SPLIT=0 turns stream-K off; =1 uses it whenever a tile count
// allows it, down to one unit per worker (tests). Returns the workers to
// launch.
constexpr int kMinUnits = 8;
constexpr int kMinSlices = 64;
constexpr int kFixupSlices = 4;

int plan_schedule(GemmParams& p, int workers) {
  p.sk_tiles = 0;
  p.sk_workers = 0;
  const int T = p.total_tiles;
  const int W = workers;
  const char* env = std::getenv("LEMA_GEMM_SPLIT");
  const bool off = env != nullptr && std::strcmp(env, "0") == 0;
  const bool forced = env != nullptr && std::strcmp(env, "1") == 0;
  const int whole = std::min(T, W);
  if (off || T % W == 0 || (!forced && p.num_kb < kMinSlices)) return whole;
  const int64_t KB = p.num_kb;
  const int full = T / W;
  const int sk_tiles = T % W;
  const int64_t units = static_cast<int64_t>(sk_tiles) * KB;
  const int64_t per = forced ? 1 : kMinUnits;
  const int S = static_cast<int>(std::min<int64_t>(W, units / per));
  if (S < 2) return whole;
  const int64_t dp_cost = static_cast<int64_t>(full + 1) * KB;
  const int64_t sk_cost = static_cast<int64_t>(full) * KB + (units + S - 1) / S + kFixupSlices;
  if (!forced && sk_cost >= dp_cost) return whole;
  p.sk_tiles = sk_tiles;
  p.sk_workers = S;
  return full >= 1 ? W : S;
}

// Column tiles per raster panel (decode_tile): LEMA_GEMM_RASTER=n overrides.
int raster_width(int n_tiles) {
  int r = 1;
  if (const char* env = std::getenv("LEMA_GEMM_RASTER")) r = std::atoi(env);
  return std::max(1, std::min(r, std::max(1, n_tiles)));
}

// Optional timing of the int8 GEMM launches (the bench's tensor roofline):
// a pre-created pool of CUDA event pairs recorded on the launching stream
// around each launch, so an instrumented step keeps the fused entry points
// and pays one event record on either side of each GEMM. Launches on a
// capturing stream, on another device or past the pool are not recorded
// (counted as dropped).
struct GemmTimer {
  std::mutex mu;
  bool on = false;
  int device = -1;
  std::vector<cudaEvent_t> events;  // 2 per record
  std::vector<double> ops;
  int64_t used = 0;
  int64_t dropped = 0;
};

GemmTimer& gemm_timer() {
  static GemmTimer t;
  return t;
}

// Reserves a record slot for a launch on `stream`; -1 when not timing it.
int64_t timer_begin(cudaStream_t stream, double ops) {
  GemmTimer& t = gemm_timer();
  std::lock_guard<std::mutex> lock(t.mu);
  if (!t.on) return -1;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    (void)cudaGetLastError();
    ++t.dropped;
    return -1;
  }
  if (cap != cudaStreamCaptureStatusNone || current_device() != t.device ||
      2 * (t.used + 1) > static_cast<int64_t>(t.events.size())) {
    ++t.dropped;
    return -1;
  }
  const int64_t i = t.used++;
  t.ops[i] = ops;
  if (cudaEventRecord(t.events[2 * i], stream) != cudaSuccess) (void)cudaGetLastError();
  return i;
}

void timer_end(int64_t i, cudaStream_t stream) {
  if (i < 0) return;
  GemmTimer& t = gemm_timer();
  std::lock_guard<std::mutex> lock(t.mu);
  if (cudaEventRecord(t.events[2 * i + 1], stream) != cudaSuccess) (void)cudaGetLastError();
}

enum TilePath { kPath1Sm128 = 0, kPath1Sm256 = 1, kPathPair = 2 };

// Tile path: LEMA_GEMM_TILE=1sm128|1sm256|pair forces one (tests, tuning);
// otherwise the pair kernel (256 x 256 per CTA pair) when its tiles fill the
// resident pairs, else 128 x 256 when those fill the SMs, else 128 x 128.
int choose_path(int kind, const Groups& groups, int64_t n) {
  const char* env = std::getenv("LEMA_GEMM_TILE");
  if (env != nullptr) {
    if (std::strcmp(env, "1sm128") == 0) return kPath1Sm128;
    if (std::strcmp(env, "1sm256") == 0) return kPath1Sm256;
    if (std::strcmp(env, "pair") == 0) return kPathPair;
  }
  auto m_tiles = [&](int tm) {
    int64_t t = 0;
    for (int g = 0; g < groups.num; ++g)
      t += (groups.row_start[g + 1] - groups.row_start[g] + tm - 1) / tm;
    return t;
  };
  const int sms = device_sm_count();
  const int slots = kind == kKindI8 ? pair_slots<kKindI8>() : pair_slots<kKindBF16>();
  if (slots > 0 && n > 128 && m_tiles(256) * ((n + 255) / 256) >= slots) return kPathPair;
  if (n > 128 && m_tiles(128) * ((n + 255) / 256) >= sms) return kPath1Sm256;
  return kPath1Sm128;
}

// Shared front end of the dense, grouped and bf16 GEMMs.
int run_gemm(int kind, const void* a, int64_t lda, const void* b, int64_t ldb,
             const Groups& groups, int64_t n, int64_t k, const float* sx, const float* sw,
             const void* bias, void* y, int64_t ldy, int32_t* acc, int64_t ldacc,
             cudaStream_t stream) {
  const int elem = (kind == kKindI8) ? 1 : 2;
  const int64_t rows = groups.row_start[groups.num];
  if (rows == 0 || n == 0) return LEMA_OK;
  if (a == nullptr || b == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null operand");
  if (y == nullptr && acc == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "no output (y and acc_dbg both null)");
  if (kind == kKindI8 && sx == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "null row scale pointer");
  if (rows > INT32_MAX || n > INT32_MAX || k > INT32_MAX ||
      n * static_cast<int64_t>(groups.num) > INT32_MAX)
    return set_error(LEMA_ERR_UNSUPPORTED, "dimension exceeds int32");
  if ((y != nullptr && ldy < n) || (acc != nullptr && ldacc < n))
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "output leading dimension < N");
  if (k == 0) return set_error(LEMA_ERR_UNSUPPORTED, "K == 0 must be handled by the caller");
  if (lda < k || ldb < k) return set_error(LEMA_ERR_INVALID_ARGUMENT, "operand ld < K");
  if (!aligned16(a) || !aligned16(b) || (lda * elem) % 16 != 0 || (ldb * elem) % 16 != 0)
    return set_error(LEMA_ERR_MISALIGNED,
                     "TMA operands need 16-byte aligned base pointers and row strides");

  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.num_kb = static_cast<int>((k * elem + kRowBytes - 1) / kRowBytes);
  p.n = static_cast<int32_t>(n);
  p.num_groups = groups.num;
  p.sx = sx;
  p.sw = sw;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.acc = acc;
  p.ldacc = ldacc;
  p.err = gemm_err_ptr();
  if (p.err == nullptr) return set_error(LEMA_ERR_CUDA, "cannot resolve device error word");

  const int path = choose_path(kind, groups, n);
  const int tm = path == kPathPair ? 256 : 128;
  const int tn = path == kPath1Sm128 ? 128 : 256;
  p.num_n_tiles = static_cast<int32_t>((n + tn - 1) / tn);
  int64_t tiles = 0;
  for (int g = 0; g < groups.num; ++g) {
    p.row_start[g] = static_cast<int32_t>(groups.row_start[g]);
    p.tile_start[g] = static_cast<int32_t>(tiles);
    const int64_t mt = (groups.row_start[g + 1] - groups.row_start[g] + tm - 1) / tm;
    tiles += mt * p.num_n_tiles;
  }
  p.row_start[groups.num] = static_cast<int32_t>(rows);
  p.tile_start[groups.num] = static_cast<int32_t>(tiles);
  if (tiles > INT32_MAX) return set_error(LEMA_ERR_UNSUPPORTED, "too many tiles");
  p.total_tiles = static_cast<int32_t>(tiles);
  if (tiles == 0) return LEMA_OK;

  // Workers: resident CTA pairs or SMs. Stream-K when it pays and a workspace
  // is available; otherwise every tile runs whole.
  const int max_workers = path == kPathPair
                              ? (kind == kKindI8 ? pair_slots<kKindI8>() : pair_slots<kKindBF16>())
                              : device_sm_count();
  if (max_workers <= 0) return set_error(LEMA_ERR_CUDA, "cannot size the GEMM grid");
  p.raster = raster_width(p.num_n_tiles);
  p.skip_publish = g_skip_publish.load();
  p.wait_budget = g_wait_budget.load();
  int workers = plan_schedule(p, max_workers);
  if (p.sk_workers > 0 && !split_workspace(stream, &p.ws, &p.ws_flags, &p.epoch)) {
    p.sk_tiles = 0;
    p.sk_workers = 0;
    workers = std::min(p.total_tiles, max_workers);
  }

  const CUtensorMapDataType dt =
      (kind == kKindI8) ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int b_box = path == kPath1Sm256 ? 256 : 128;
  CUtensorMap ma, mb;
  int rc = make_operand_map(&ma, a, dt, elem, rows, k, lda, kBM);
  if (rc) return rc;
  rc = make_operand_map(&mb, b, dt, elem, n * groups.num, k, ldb, b_box);
  if (rc) return rc;

  // y through TMA stores: 16-byte aligned rows, at least one full 32 x 32 box
  CUtensorMap my;
  std::memset(&my, 0, sizeof(my));
  if (y != nullptr && aligned16(y) && (ldy * 2) % 16 == 0 && n >= 32 && rows >= 32) {
    rc = make_y_map(&my, y, rows, n, ldy);
    if (rc) return rc;
    p.y_tma = 1;
  }
  p.total_rows = static_cast<int32_t>(rows);

  if (kind == kKindI8) {
    const int64_t rec = timer_begin(stream, 2.0 * static_cast<double>(rows) *
                                                static_cast<double>(n) * static_cast<double>(k));
    if (path == kPathPair)
      rc = launch_pair<kKindI8>(ma, mb, my, p, workers, stream);
    else
      rc = path == kPath1Sm256 ? launch<kKindI8, 256, 4>(ma, mb, my, p, workers, stream)
                               : launch<kKindI8, 128, 6>(ma, mb, my, p, workers, stream);
    timer_end(rec, stream);
    return rc;
  }
  if (path == kPathPair) return launch_pair<kKindBF16>(ma, mb, my, p, workers, stream);
  return path == kPath1Sm256 ? launch<kKindBF16, 256, 4>(ma, mb, my, p, workers, stream)
                             : launch<kKindBF16, 128, 6>(ma, mb, my, p, workers, stream);
}

// y = bias (or 0) broadcast over rows: the K == 0 case.
__global__ void fill_bias_kernel(__nv_bfloat16* y, int64_t ldy, int64_t m, int64_t n,
                                 const __nv_bfloat16* bias) {
  const int64_t total = m * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / n, c = i % n;
    y[r * ldy + c] = bias ? bias[c] : __float2bfloat16_rn(0.f);
  }
}

__global__ void fill_zero_i32_kernel(int32_t* a, int64_t lda, int64_t m, int64_t n) {
  const int64_t total = m * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    a[(i / n) * lda + (i % n)] = 0;
}

int k_zero_outputs(void* y, int64_t ldy, const void* bias, int32_t* acc, int64_t ldacc,
                   int64_t m, int64_t n, cudaStream_t s) {
  if (m == 0 || n == 0) return LEMA_OK;
  const int grid = static_cast<int>(std::min<int64_t>((m * n + 255) / 256, 4096));
  if (y)
    fill_bias_kernel<<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(y), ldy, m, n,
                                          static_cast<const __nv_bfloat16*>(bias));
  if (acc) fill_zero_i32_kernel<<<grid, 256, 0, s>>>(acc, ldacc, m, n);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

// Moves the error word into a host word (mapped pinned memory) when it is
// nonzero, and clears it: the host reads the word later without a sync.
__global__ void error_snapshot_kernel(int32_t* host_word) {
  const int32_t v = atomicExch(&g_gemm_err, 0);
  if (v != 0) *reinterpret_cast<volatile int32_t*>(host_word) = v;
}

}  // namespace

ScopedNoGemmWorkspace::ScopedNoGemmWorkspace() : prev(t_no_split) { t_no_split = true; }
ScopedNoGemmWorkspace::~ScopedNoGemmWorkspace() { t_no_split = prev; }

int32_t* gemm_error_word() { return gemm_err_ptr(); }

int gemm_read_device_error(int32_t* out) {
  int32_t v = 0, zero = 0;
  LEMA_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_gemm_err, sizeof(v)));
  LEMA_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_err, &zero, sizeof(zero)));
  *out = v;
  return LEMA_OK;
}

}  // namespace lema

using namespace lema;

extern "C" int lema_w8a8_gemm(const int8_t* xq, int64_t ldx, const float* sx, const int8_t* wq,
                              int64_t ldw, const float* sw, const void* bias_bf16, void* y_bf16,
                              int64_t ldy, int32_t* acc_dbg, int64_t ldacc, int64_t M, int64_t N,
                              int64_t K, void* stream) {
  clear_error();
  if (M < 0 || N < 0 || K < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  auto s = static_cast<cudaStream_t>(stream);
  if (K == 0) return k_zero_outputs(y_bf16, ldy, bias_bf16, acc_dbg, ldacc, M, N, s);
  Groups g;
  g.num = 1;
  g.row_start[0] = 0;
  g.row_start[1] = M;
  return run_gemm(kKindI8, xq, ldx, wq, ldw, g, N, K, sx, sw, bias_bf16, y_bf16, ldy, acc_dbg,
                  ldacc, s);
}

extern "C" int lema_bf16_gemm_tn(const void* a_bf16, int64_t lda, const void* b_bf16,
                                 int64_t ldb, void* y_bf16, int64_t ldy, int64_t M, int64_t N,
                                 int64_t K, void* stream) {
  clear_error();
  if (M < 0 || N < 0 || K < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  auto s = static_cast<cudaStream_t>(stream);
  if (K == 0) return k_zero_outputs(y_bf16, ldy, nullptr, nullptr, 0, M, N, s);
  Groups g;
  g.num = 1;
  g.row_start[0] = 0;
  g.row_start[1] = M;
  return run_gemm(kKindBF16, a_bf16, lda, b_bf16, ldb, g, N, K, nullptr, nullptr, nullptr,
                  y_bf16, ldy, nullptr, 0, s);
}

extern "C" int lema_grouped_w8a8_gemm(const int8_t* xq, int64_t ldx, const float* sx,
                                      const int8_t* wq, int64_t ldw, const float* sw,
                                      const void* bias_bf16, void* y_bf16, int64_t ldy,
                                      const int64_t* offsets_host, int32_t E, int64_t N,
                                      int64_t K, void* stream) {
  clear_error();
  if (offsets_host == nullptr || E <= 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "offsets must hold E+1 entries, E >= 1");
  if (E > kMaxGroups)
    return set_error(LEMA_ERR_UNSUPPORTED, "more than 64 experts per grouped launch");
  if (N < 0 || K < 0 || offsets_host[0] != 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad sizes or offsets[0] != 0");
  Groups g;
  g.num = E;
  for (int e = 0; e <= E; ++e) {
    g.row_start[e] = offsets_host[e];
    if (e > 0 && offsets_host[e] < offsets_host[e - 1])
      return set_error(LEMA_ERR_INVALID_ARGUMENT, "offsets must be non-decreasing");
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    // Every row gets its expert's bias.
    for (int e = 0; e < E; ++e) {
      const int64_t r0 = offsets_host[e], r1 = offsets_host[e + 1];
      if (r1 == r0) continue;
      const void* b = bias_bf16 ? static_cast<const __nv_bfloat16*>(bias_bf16) + e * N : nullptr;
      int rc = k_zero_outputs(static_cast<__nv_bfloat16*>(y_bf16) + r0 * ldy, ldy, b, nullptr, 0,
                              r1 - r0, N, s);
      if (rc) return rc;
    }
    return LEMA_OK;
  }
  return run_gemm(kKindI8, xq, ldx, wq, ldw, g, N, K, sx, sw, bias_bf16, y_bf16, ldy, nullptr, 0,
                  s);
}

extern "C" int lema_grouped_bf16_gemm_tn(const void* a_bf16, int64_t lda, const void* b_bf16,
                                         int64_t ldb, void* y_bf16, int64_t ldy,
                                         const int64_t* offsets_host, int32_t E, int64_t N,
                                         int64_t K, void* stream) {
  clear_error();
  if (offsets_host == nullptr || E <= 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "offsets must hold E+1 entries, E >= 1");
  if (E > kMaxGroups)
    return set_error(LEMA_ERR_UNSUPPORTED, "more than 64 groups per grouped launch");
  if (N < 0 || K < 0 || offsets_host[0] != 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad sizes or offsets[0] != 0");
  Groups g;
  g.num = E;
  for (int e = 0; e <= E; ++e) {
    g.row_start[e] = offsets_host[e];
    if (e > 0 && offsets_host[e] < offsets_host[e - 1])
      return set_error(LEMA_ERR_INVALID_ARGUMENT, "offsets must be non-decreasing");
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (K == 0)
    return k_zero_outputs(y_bf16, ldy, nullptr, nullptr, 0, offsets_host[E], N, s);
  return run_gemm(kKindBF16, a_bf16, lda, b_bf16, ldb, g, N, K, nullptr, nullptr, nullptr,
                  y_bf16, ldy, nullptr, 0, s);
}

extern "C" int lema_bf16_gemm_tn_f32(const void* a_bf16, int64_t lda, const void* b_bf16,
                                     int64_t ldb, float* y_f32, int64_t ldy, int64_t M, int64_t N,
                                     int64_t K, void* stream) {
  clear_error();
  if (M < 0 || N < 0 || K < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "negative size");
  if (y_f32 == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null output");
  auto s = static_cast<cudaStream_t>(stream);
  if (K == 0)
    return k_zero_outputs(nullptr, 0, nullptr, reinterpret_cast<int32_t*>(y_f32), ldy, M, N, s);
  Groups g;
  g.num = 1;
  g.row_start[0] = 0;
  g.row_start[1] = M;
  return run_gemm(kKindBF16, a_bf16, lda, b_bf16, ldb, g, N, K, nullptr, nullptr, nullptr,
                  nullptr, 0, reinterpret_cast<int32_t*>(y_f32), ldy, s);
}

extern "C" int lema_gemm_timer_start(int64_t max_records) {
  clear_error();
  if (max_records <= 0 || max_records > (int64_t{1} << 20))
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "max_records must be in [1, 2^20]");
  GemmTimer& t = gemm_timer();
  std::lock_guard<std::mutex> lock(t.mu);
  const int dev = current_device();
  if (dev != t.device) {
    for (cudaEvent_t e : t.events) (void)cudaEventDestroy(e);
    t.events.clear();
    t.device = dev;
  }
  while (static_cast<int64_t>(t.events.size()) < 2 * max_records) {
    cudaEvent_t e = nullptr;
    LEMA_CUDA_TRY(cudaEventCreate(&e));
    t.events.push_back(e);
  }
  t.ops.assign(static_cast<size_t>(max_records), 0.0);
  t.used = 0;
  t.dropped = 0;
  t.on = true;
  return LEMA_OK;
}

extern "C" int lema_gemm_timer_stop(double* total_ops, double* total_ms, int64_t* launches,
                                    int64_t* dropped) {
  clear_error();
  GemmTimer& t = gemm_timer();
  std::lock_guard<std::mutex> lock(t.mu);
  t.on = false;
  double ops = 0.0, ms = 0.0;
  for (int64_t i = 0; i < t.used; ++i) {
    LEMA_CUDA_TRY(cudaEventSynchronize(t.events[2 * i + 1]));
    float e = 0.f;
    LEMA_CUDA_TRY(cudaEventElapsedTime(&e, t.events[2 * i], t.events[2 * i + 1]));
    ms += e;
    ops += t.ops[i];
  }
  if (total_ops) *total_ops = ops;
  if (total_ms) *total_ms = ms;
  if (launches) *launches = t.used;
  if (dropped) *dropped = t.dropped;
  t.used = 0;
  return LEMA_OK;
}

extern "C" int lema_device_error_async(int32_t* host_word, void* stream) {
  clear_error();
  if (host_word == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null host_word");
  cudaPointerAttributes attr;
  LEMA_CUDA_TRY(cudaPointerGetAttributes(&attr, host_word));
  if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr)
    return set_error(LEMA_ERR_INVALID_ARGUMENT,
                     "host_word must be page-locked host memory mapped into the device "
                     "(cudaHostAlloc / pin_memory)");
  error_snapshot_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<int32_t*>(attr.devicePointer));
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_gemm_set_test_hooks(int32_t skip_publish, int64_t wait_budget_cycles) {
  clear_error();
  if (wait_budget_cycles < 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "wait_budget_cycles must be >= 0");
  g_skip_publish.store(skip_publish != 0 ? 1 : 0);
  g_wait_budget.store(wait_budget_cycles == 0 ? ptx::kWaitBudgetCycles
                                              : static_cast<long long>(wait_budget_cycles));
  return LEMA_OK;
}

extern "C" int lema_gemm_workspace_count(int64_t* count) {
  clear_error();
  if (count == nullptr) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null count");
  std::lock_guard<std::mutex> lock(g_ws_mu);
  int64_t n = 0;
  for (const auto& kv : g_ws) n += kv.second.slots != nullptr ? 1 : 0;
  *count = n;
  return LEMA_OK;
}
