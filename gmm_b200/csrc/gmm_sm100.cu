// gmm_sm100.cu -- persistent grouped-GEMM forward for B200 (sm_100a) and its C ABI.
//
// Replaces the reference's CUTLASS sm_90a grouped GEMM
// (reference csrc/hopper_gmm_forward.cu:67-138 kernel configuration,
//  :230-325 launcher, :372-486 host entry) with a hand-written kernel:
//
//   * one persistent CTA per SM walks a static (group, m-tile, n-tile) tile
//     list built from the host batch_sizes; zero-row experts own no tiles;
//   * warp 0 (one lane) streams A and B tiles with TMA into a 4-stage
//     shared-memory ring (128-byte swizzle);
//   * warp 1 (one lane) issues tcgen05.mma (M=128, N=256, K=16 for bf16/fp16;
//     M=128, N=128, K=8 with three TF32 products for fp32) into one of two
//     TMEM accumulators;
//   * warps 4-7 drain the other accumulator (tcgen05.ld), convert to the
//     output type and store rows that belong to the tile's expert -- rows past
//     an expert's segment are never written, which keeps output placement exact.
//
// Two more kernels share the tile table: CTA pairs with 256-row tiles
// (gmm_pair_kernel.cuh) when the non-empty experts average at least 384 rows,
// and swap-AB tiles (gmm_swap_kernel.cuh: output columns on the MMA's M,
// token rows on its N) for decode-shaped problems whose experts all have at
// most 64 rows (choose_tile_kind).
//
// A is addressed through one 2D tensor map over all T rows (a tile of expert
// g starts at row off_g + 128 m); B through one 3D tensor map whose outer
// coordinate is the expert.  No per-expert descriptors, no TMA multicast.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <memory>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "gmm_sm100.h"
#include "sm100_ptx.cuh"

namespace gmm_sm100 {

// Device-side error word: set by a CTA whose bounded wait ran out.
__device__ int g_device_error = 0;

constexpr int kInlineGroups = 1024;  // groups whose table travels in the kernel parameters
constexpr int kInlineTableInts = 3 * kInlineGroups + 2;
constexpr int kMaxPeers = 8;         // expert-parallel ranks a kernel can address
constexpr int kMaxDevExperts = 1024;  // experts a device-built table can hold
constexpr int kDevTableBytes = (3 * kMaxDevExperts + 64) * 4;  // row_off | tile_off | expert | meta | 8-byte scan scratch
// meta sits at int 3 * kMaxDevExperts + 2; the scan scratch (8 warps x 3
// 64-bit values) at int 3 * kMaxDevExperts + 6, an 8-byte boundary.
static_assert((3 * kMaxDevExperts + 6) % 2 == 0 && (3 * kMaxDevExperts + 6) * 4 + 24 * 8 <= kDevTableBytes,
              "device table area");
constexpr int kMBlock = 16;          // m-tiles per raster block (L2 reuse of B columns)
constexpr int kThreads = 256;        // 8 warps: TMA, MMA, TMEM alloc, idle, 4x epilogue
constexpr int kEpiStageBytes = 4 * 32 * 128;  // epilogue staging: 4 warps x 32 rows x 128 B

struct __align__(64) GmmParamsBase {
  CUtensorMap tmap_a;   // A (fp32: raw fp32 tiles, split into TF32 hi/lo in shared memory)
  CUtensorMap tmap_b;   // B
  CUtensorMap tmap_a2;  // A in 64-row boxes (half tiles of the CTA-pair kernel)
  void* d;
  const int32_t* ext_table;  // device table when num_groups > kInlineGroups
  long long ldd;
  int num_groups;
  int n_tiles;
  int k_blocks;
  int total_tiles;
  int dim_out;
  int remote;  // 1: output rows go to the ranks they came from (expert-parallel combine)
  int world;   // ranks addressed through d_peer (remote mode)
  int act;     // 1: SwiGLU -- B is [gate | up] (act_cols columns each); D = silu(gate) * up
  int act_cols;
  // Device-resident batch sizes (dev_bs != nullptr): every CTA builds the
  // group table in shared memory from dev_bs[0..dev_experts) (int32); rows
  // past rows_cap are never touched and a bad table is reported through the
  // device error word.
  const int32_t* dev_bs;
  int dev_experts;
  int rows_cap;
  int tile_rows;  // 128 or 256 (m-tile height the device table is built for)
  int vk_m;        // variable-K kernel: rows of each D[e] (= columns of A)
  int vk_m_tiles;  // variable-K kernel: 128-row tiles per D[e]
  int ep_rank_base;  // remote mode: segment j of a group comes from rank (ep_rank_base + j) % world
  // Bounded waits: limit of every pipeline wait (0 = kWaitTimeoutNs).  Test
  // hook of the timeout path: drop_kb1 = k + 1 > 0 makes the producer(s) of
  // the first tile of CTA (pair) 0 skip the loads of k-block k, so that the
  // MMA warp's wait for them runs out (gmm_sm100_forward_inject_timeout);
  // 0 (the zeroed default) drops nothing.
  unsigned long long wait_ns;
  int drop_kb1;
  void* d_peer[kMaxPeers];  // each rank's output buffer (remote mode)
  int inline_ints;          // ints of inline_table in use (0: the table is in ext_table or built on device)
};

// Kernel parameters: the fields above plus the inline table, in two sizes.  A
// launch copies the whole parameter block, and the full one (12 KB of table)
// measured ~1 us slower per launch than a 1.5 KB one, so the 128-row and
// swap-AB kernels are also instantiated with the small table, which every
// call with at most kSmallGroups groups (or a table outside the parameters)
// uses.
template <int kTableInts>
struct GmmParamsT : GmmParamsBase {
  // Table of the non-empty groups, laid out as
  //   row_off[G+1] | tile_off[G+1] | expert[G] [| src_off[G][W+1] | dst_row[G][W]]
  // row_off: first row of group g in A/D (row_off[G] = T);
  // tile_off: prefix sum of m-tiles (ceil(m_g / tile rows));
  // expert: index of the expert (B slice) of group g;
  // remote mode only -- src_off: where each source rank's rows start inside
  // group g; dst_row: the row on that source where they go back to.
  int32_t inline_table[kTableInts];
};
constexpr int kSmallGroups = 128;
constexpr int kSmallTableInts = 3 * kSmallGroups + 2;
using GmmParams = GmmParamsT<kInlineTableInts>;
using GmmParamsSmall = GmmParamsT<kSmallTableInts>;

enum Kind : int { kKindTf32x3 = 0, kKindBf16 = 1, kKindF16 = 2 };

template <int kKind, bool kBMnMajor>
struct Cfg {
  static constexpr bool kTf32 = (kKind == kKindTf32x3);
  static constexpr int kElem = kTf32 ? 4 : 2;
  static constexpr int BM = 128;
  static constexpr int BN = kTf32 ? 128 : 256;
  static constexpr int BK = 128 / kElem;  // one 128-byte swizzle row of K
  static constexpr int kStages = kTf32 ? 3 : 4;
  static constexpr int kUmmaK = 32 / kElem;  // K per tcgen05.mma: 16 (16-bit), 8 (tf32)
  static constexpr int kKSteps = BK / kUmmaK;
  static constexpr int kParts = kTf32 ? 2 : 1;  // hi/lo operand copies
  static constexpr int kABytes = BM * BK * kElem;
  static constexpr int kBBytes = BN * BK * kElem;
  static constexpr int kStageBytes = kParts * (kABytes + kBBytes);
  static constexpr int kLoadBytes = kABytes + kBBytes;  // bytes TMA brings in per stage
  static constexpr int kPanelCols = 128 / kElem;        // MN-major B: columns per 128-byte panel
  static constexpr int kTmemCols = 2 * BN;  // double-buffered fp32 accumulator
  static constexpr uint32_t kIdesc =
      make_idesc(kTf32 ? 2u : (kKind == kKindBf16 ? 1u : 0u), kBMnMajor, BM, BN);
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + kEpiStageBytes + kDevTableBytes + 1024;
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms need 1 KB alignment");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct TableView {
  const int32_t* row_off;
  const int32_t* tile_off;
  const int32_t* expert;
  const int32_t* src_off;  // remote mode
  const int32_t* dst_row;  // remote mode
};

__device__ __forceinline__ TableView make_table_view(const GmmParamsBase& p, const int32_t* tab,
                                                     int num_groups) {
  TableView tv;
  tv.row_off = tab;
  tv.tile_off = tab + num_groups + 1;
  tv.expert = tab + 2 * (num_groups + 1);
  tv.src_off = tv.expert + num_groups;
  tv.dst_row = tv.src_off + num_groups * (p.world + 1);
  return tv;
}

// Exclusive block scan (256 threads) of three per-thread values; returns the
// block totals.  64-bit, so that no sum of (possibly corrupt) device batch
// sizes can wrap around.  `scratch` holds 8 warps x 3 values.
__device__ __forceinline__ void block_scan3(long long (&v)[3], long long (&tot)[3], long long* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long incl[3] = {v[0], v[1], v[2]};
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const long long o = __shfl_up_sync(0xffffffffu, incl[j], d);
      if (lane >= d) incl[j] += o;
    }
  }
  if (lane == 31)
    for (int j = 0; j < 3; ++j) scratch[warp * 3 + j] = incl[j];
  __syncthreads();
  long long warp_off[3] = {0, 0, 0};
  for (int j = 0; j < 3; ++j) {
    tot[j] = 0;
    for (int w = 0; w < 8; ++w) {
      if (w < warp) warp_off[j] += scratch[w * 3 + j];
      tot[j] += scratch[w * 3 + j];
    }
  }
  for (int j = 0; j < 3; ++j) v[j] = incl[j] - v[j] + warp_off[j];
  __syncthreads();
}

// Build the group table from device batch sizes into shared memory (all 256
// threads).  Layout as the host table: row_off[G+1] | tile_off[G+1] |
// expert[G]; meta[0] = G, meta[1] = m-tiles, meta[2] = error status.  Row,
// group and m-tile sums are taken in 64 bits: a negative size, or a total
// above rows_cap (however large the sizes), leaves an empty table and an
// error status, so no row past rows_cap is ever addressed.  After that check
// every prefix fits in 32 bits (rows_cap < 2^31 - 256).
__device__ void build_device_table(const GmmParamsBase& p, int32_t* tab, int32_t* meta, long long* scratch) {
  const int E = p.dev_experts;
  const int BM = p.tile_rows;
  constexpr int kPer = kMaxDevExperts / kThreads;  // experts per thread (4)
  int bsv[kPer];
  long long loc[3] = {0, 0, 0};  // rows, non-empty experts, m-tiles of this thread's experts
  bool bad = false;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = threadIdx.x * kPer + i;
    const int m = e < E ? p.dev_bs[e] : 0;
    bad |= m < 0;
    bsv[i] = m > 0 ? m : 0;
    loc[0] += bsv[i];
    loc[1] += bsv[i] > 0;
    loc[2] += (static_cast<long long>(bsv[i]) + BM - 1) / BM;
  }
  long long tot[3];
  long long pre[3] = {loc[0], loc[1], loc[2]};
  block_scan3(pre, tot, scratch);
  const int bad_any = __syncthreads_or(bad);
  const int G = static_cast<int>(tot[1]);
  if (bad_any || tot[0] > p.rows_cap) {
    if (threadIdx.x == 0) {
      meta[0] = 0;
      meta[1] = 0;
      meta[2] = bad_any ? GMM_ERR_INVALID_ARGUMENT : GMM_ERR_BATCH_SUM;
      tab[0] = 0;
      tab[1] = 0;
    }
    __syncthreads();
    return;
  }
  int row = static_cast<int>(pre[0]), g = static_cast<int>(pre[1]), mt = static_cast<int>(pre[2]);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    if (bsv[i] > 0) {
      tab[g] = row;
      tab[G + 1 + g] = mt;
      tab[2 * (G + 1) + g] = threadIdx.x * kPer + i;
      ++g;
      mt += (bsv[i] + BM - 1) / BM;
    }
    row += bsv[i];
  }
  if (threadIdx.x == 0) {
    tab[G] = static_cast<int>(tot[0]);
    tab[2 * G + 1] = static_cast<int>(tot[2]);
    meta[0] = G;
    meta[1] = static_cast<int>(tot[2]);
    meta[2] = 0;
  }
  __syncthreads();
}

// Where output row `row` (a row of A, inside group g) is stored: D itself, or
// in remote mode the output buffer of the rank the row came from.
template <typename T>
__device__ __forceinline__ T* out_row(const GmmParamsBase& p, const TableView& tv, int g, int row) {
  if (!p.remote) return reinterpret_cast<T*>(p.d) + static_cast<long long>(row) * p.ldd;
  const int grow = row - tv.row_off[g];
  const int32_t* so = tv.src_off + g * (p.world + 1);
  int j = 0;  // segment of the row inside its group
  while (j + 1 < p.world && grow >= so[j + 1]) ++j;
  const int32_t* dr = tv.dst_row + g * p.world;
  int s = p.ep_rank_base + j;
  if (s >= p.world) s -= p.world;
  return reinterpret_cast<T*>(p.d_peer[s]) + static_cast<long long>(dr[j] + grow - so[j]) * p.ldd;
}

struct Tile {
  int row0;    // first row of the tile in A / D
  int rows;    // rows of the tile that belong to its expert (1..128)
  int n0;      // first output column
  int expert;  // B slice
};

template <int BM, int BN>
__device__ __forceinline__ Tile decode_tile(const TableView& t, int n_tiles, int tile, int& g) {
  // Groups are visited in increasing order by every CTA, so a forward scan
  // from the previous group finds the owner in amortised O(1).
  while (tile >= t.tile_off[g + 1] * n_tiles) ++g;
  const int mt = t.tile_off[g + 1] - t.tile_off[g];
  const int local = tile - t.tile_off[g] * n_tiles;
  // Raster: blocks of up to kMBlock m-tiles; inside a block m varies fastest so
  // the CTAs working on one B column panel run at the same time (L2 reuse).
  const int blk = local / (kMBlock * n_tiles);
  const int r = local - blk * kMBlock * n_tiles;
  const int h = min(kMBlock, mt - blk * kMBlock);
  const int m = blk * kMBlock + r % h;
  const int n = r / h;
  Tile out;
  out.row0 = t.row_off[g] + m * BM;
  out.rows = min(BM, t.row_off[g + 1] - out.row0);
  out.n0 = n * BN;
  out.expert = t.expert[g];
  return out;
}

// Bounded wait used while draining after an abort: ignores the abort flag.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitTimeoutNs) return;
  }
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);

template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Drains one 32-row slab of an accumulator -- TMEM lanes [32q, 32q + 32) of
// columns [taddr, taddr + BN) -- into its output rows.  Each thread converts its
// own row; the rows then pass through `stage` (32 rows x 128 B, 16-byte chunks
// XOR-swizzled by row, conflict-free both ways) so that every store
// instruction writes four whole 128-byte row segments (8 lanes per row): full
// L2 lines locally, and large NVLink writes when the row lives on a peer.
// Drains one 32-row slab of an accumulator -- TMEM lanes [32q, 32q + 32) of
// columns [taddr, taddr + BN) -- into the rows rp[] (8 per lane: rows
// i*4 + lane/8; null = not stored).  Each thread converts its own row; the rows
// then pass through `stage` (32 rows x 128 B, 16-byte chunks XOR-swizzled by
// row, conflict-free both ways) so that every store instruction writes four
// whole 128-byte row segments (8 lanes per row): full L2 lines locally, and
// large NVLink writes when the row lives on a peer.  zero = store zeros
// without reading TMEM (a tile whose contraction is empty).
template <typename OutT, int BN>
__device__ __forceinline__ void drain_rows(OutT* const (&rp)[8], int n0, int dim_out, uint32_t taddr,
                                           uint32_t stage, int lane, bool zero = false) {
  constexpr int kColsPerSeg = 128 / static_cast<int>(sizeof(OutT));  // 64 (16-bit) or 32 (fp32)
  constexpr int kElemsPer16 = 16 / static_cast<int>(sizeof(OutT));
  const int ch = lane & 7;
  const uint32_t my_row = stage + lane * 128;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += kColsPerSeg) {
    const int col = n0 + c0;
    if (col >= dim_out) break;  // warp-uniform
#pragma unroll
    for (int h = 0; h < kColsPerSeg / 32; ++h) {
      uint32_t v[32];
      if (!zero) {
        tmem_ld_32x32b_x32(taddr + c0 + h * 32, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      if constexpr (sizeof(OutT) == 2) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 pk;
          pk.x = pack2<OutT>(__uint_as_float(v[8 * q + 0]), __uint_as_float(v[8 * q + 1]));
          pk.y = pack2<OutT>(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3]));
          pk.z = pack2<OutT>(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5]));
          pk.w = pack2<OutT>(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7]));
          st_shared_v4(my_row + (((h * 4 + q) ^ (lane & 7)) << 4), pk);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          st_shared_v4(my_row + ((q ^ (lane & 7)) << 4),
                       make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
      }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = i * 4 + (lane >> 3);
      const uint4 val = ld_shared_v4(stage + rr * 128 + ((ch ^ (rr & 7)) << 4));
      if (rp[i] && col + ch * kElemsPer16 < dim_out)
        *reinterpret_cast<uint4*>(rp[i] + col + ch * kElemsPer16) = val;
    }
    __syncwarp();
  }
}

// drain_rows for a slab of grouped-GEMM rows: destinations from out_row().
template <typename OutT, int BN>
__device__ __forceinline__ void drain_slab(const GmmParamsBase& p, const TableView& tv, int g,
                                           int slab_row0, int slab_rows, int n0, uint32_t taddr,
                                           uint32_t stage, int lane) {
  OutT* rp[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = i * 4 + (lane >> 3);
    rp[i] = rr < slab_rows ? out_row<OutT>(p, tv, g, slab_row0 + rr) : nullptr;
  }
  drain_rows<OutT, BN>(rp, n0, p.dim_out, taddr, stage, lane);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + __expf(-g)) * u; }

// SwiGLU variant of drain_slab: TMEM columns [0, 128) hold the tile's gate
// projections and [128, 256) the matching up projections; writes
// silu(gate) * up (fp32) rounded to the output type, 128 columns per tile.
template <typename OutT>
__device__ __forceinline__ void drain_slab_swiglu(const GmmParamsBase& p, const TableView& tv, int g,
                                                  int slab_row0, int slab_rows, int n0, uint32_t taddr,
                                                  uint32_t stage, int lane) {
  static_assert(sizeof(OutT) == 2, "SwiGLU epilogue is 16-bit");
  OutT* rp[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = i * 4 + (lane >> 3);
    rp[i] = rr < slab_rows ? out_row<OutT>(p, tv, g, slab_row0 + rr) : nullptr;
  }
  const int ch = lane & 7;
  const uint32_t my_row = stage + lane * 128;
#pragma unroll 1
  for (int c0 = 0; c0 < 128; c0 += 64) {
    const int col = n0 + c0;
    if (col >= p.dim_out) break;  // warp-uniform
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t gv[32], uv[32];
      tmem_ld_32x32b_x32(taddr + c0 + h * 32, gv);
      tmem_ld_32x32b_x32(taddr + 128 + c0 + h * 32, uv);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          a[j] = silu_mul(__uint_as_float(gv[8 * q + j]), __uint_as_float(uv[8 * q + j]));
        uint4 pk;
        pk.x = pack2<OutT>(a[0], a[1]);
        pk.y = pack2<OutT>(a[2], a[3]);
        pk.z = pack2<OutT>(a[4], a[5]);
        pk.w = pack2<OutT>(a[6], a[7]);
        st_shared_v4(my_row + (((h * 4 + q) ^ (lane & 7)) << 4), pk);
      }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = i * 4 + (lane >> 3);
      const uint4 val = ld_shared_v4(stage + rr * 128 + ((ch ^ (rr & 7)) << 4));
      if (rp[i] && col + ch * 8 < p.dim_out) *reinterpret_cast<uint4*>(rp[i] + col + ch * 8) = val;
    }
    __syncwarp();
  }
}

// Splits x into a TF32-exact high part (low 13 mantissa bits cleared) and the
// fp32 remainder, so that three TF32 products hi*hi + hi*lo + lo*hi recover
// close to fp32 accuracy.  Non-finite values pass through in hi with lo = 0.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  if (isfinite(x)) {
    hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    lo = x - hi;
  } else {
    hi = x;
    lo = 0.0f;
  }
}

template <int kKind, bool kBMnMajor, typename P = GmmParams>
__global__ void __launch_bounds__(kThreads, 1) gmm_persistent_kernel(const __grid_constant__ P p) {
  using C = Cfg<kKind, kBMnMajor>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full_bar = bars;                       // TMA -> MMA
  uint64_t* empty_bar = bars + C::kStages;         // MMA -> TMA
  uint64_t* tfull_bar = bars + 2 * C::kStages;     // MMA -> epilogue (2 accumulators)
  uint64_t* tempty_bar = bars + 2 * C::kStages + 2;  // epilogue -> MMA
  uint64_t* drain_bar = bars + 2 * C::kStages + 4;
  uint64_t* conv_bar = bars + 2 * C::kStages + 5;  // fp32: hi/lo split done -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * C::kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* epi_stage = smem + C::kStages * C::kStageBytes + C::kBarBytes;
  static_assert((3 * C::kStages + 6) * 8 <= C::kBarBytes, "barrier area");

  // fp32: warps 2-3 split every landed stage into TF32 hi/lo.  A CTA that owns
  // a single tile (a small, latency-bound problem) also lends its four
  // epilogue warps to the split, which they finish before their one
  // accumulator can be ready: six warps instead of two per stage.
  const int conv_warps =
      (C::kTf32 && p.dev_bs == nullptr && blockIdx.x + gridDim.x >= p.total_tiles) ? 6 : 2;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(full_bar + s), 1);
      mbar_init(smem_u32(empty_bar + s), 1);
      mbar_init(smem_u32(conv_bar + s), conv_warps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(tfull_bar + a), 1);
      mbar_init(smem_u32(tempty_bar + a), 4);
    }
    mbar_init(smem_u32(drain_bar), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    prefetch_tmap(&p.tmap_b);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = p.n_tiles;
  const int k_blocks = p.k_blocks;
  const unsigned long long wait_ns = p.wait_ns ? p.wait_ns : kWaitTimeoutNs;
  int num_groups = p.num_groups, total_tiles = p.total_tiles;
  const int32_t* tab = p.ext_table ? p.ext_table : p.inline_table;
  if (p.dev_bs) {
    int32_t* dtab = reinterpret_cast<int32_t*>(epi_stage + kEpiStageBytes);
    int32_t* meta = dtab + 3 * kMaxDevExperts + 2;
    build_device_table(p, dtab, meta, reinterpret_cast<long long*>(meta + 4));
    num_groups = meta[0];
    total_tiles = meta[1] * n_tiles;
    if (threadIdx.x == 0 && meta[2] != 0) atomicCAS(&g_device_error, 0, meta[2]);
    tab = dtab;
  }
  const TableView tv = make_table_view(p, tab, num_groups);

  // ------------------------------------------------------------ fp32 split (converter)
  // Each landed fp32 stage is split in shared memory: x -> hi (low 13
  // mantissa bits cleared, exact in TF32) in place, x - hi -> the stage's lo
  // copy at the same offset.  The split is element-wise, so the swizzled
  // layout is preserved; the writes are fenced into the async proxy before
  // the MMA warp (which waits on conv_bar for all conv_warps) hands them to
  // the tensor cores.  Run by warps 2 .. 1 + conv_warps, thread ct of
  // 32 * conv_warps taking every such 16-byte chunk of the stage.
  auto split_stages = [&]() {
    const int ct = threadIdx.x - 64;
    const int nthr = 32 * conv_warps;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait(smem_u32(full_bar + stage), phase, abort_flag, wait_ns)) {
          ok = false;
          break;
        }
        const uint32_t base = smem_u32(smem + stage * C::kStageBytes);
        constexpr int kChunksA = C::kABytes / 16, kChunks = (C::kABytes + C::kBBytes) / 16;
#pragma unroll 4
        for (int i = ct; i < kChunks; i += nthr) {
          // A: x at [0, kABytes), lo at [kABytes, 2 kABytes); B: x at 2 kABytes, lo kBBytes further
          const uint32_t off = i < kChunksA ? i * 16 : 2 * C::kABytes + (i - kChunksA) * 16;
          const uint32_t lo_off = off + (i < kChunksA ? C::kABytes : C::kBBytes);
          const uint4 v = ld_shared_v4(base + off);
          float h0, h1, h2, h3, l0, l1, l2, l3;
          split_tf32(__uint_as_float(v.x), h0, l0);
          split_tf32(__uint_as_float(v.y), h1, l1);
          split_tf32(__uint_as_float(v.z), h2, l2);
          split_tf32(__uint_as_float(v.w), h3, l3);
          st_shared_v4(base + off, make_uint4(__float_as_uint(h0), __float_as_uint(h1), __float_as_uint(h2),
                                              __float_as_uint(h3)));
          st_shared_v4(base + lo_off, make_uint4(__float_as_uint(l0), __float_as_uint(l1), __float_as_uint(l2),
                                                 __float_as_uint(l3)));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(conv_bar + stage));
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[C::kStages];
      for (int s = 0; s < C::kStages; ++s) issued[s] = 0;
      bool ok = true;
      int g = 0;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        const Tile t = decode_tile<C::BM, C::BN>(tv, n_tiles, tile, g);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(empty_bar + stage), phase ^ 1, abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          if (kb + 1 == p.drop_kb1 && tile == 0) {  // timeout test hook: this stage never fills
            if (++stage == C::kStages) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          const uint32_t fb = smem_u32(full_bar + stage);
          mbar_arrive_expect_tx(fb, C::kLoadBytes);
          uint8_t* sa = smem + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kParts * C::kABytes;
          const int k0 = kb * C::BK;
          tma_load_2d(smem_u32(sa), &p.tmap_a, fb, k0, t.row0);
          if (C::kTf32) {  // raw fp32 tiles; the converter warps split them in place
            if (kBMnMajor) {
#pragma unroll
              for (int c = 0; c < C::BN / C::kPanelCols; ++c)
                tma_load_3d(smem_u32(sb + c * (C::BK * 128)), &p.tmap_b, fb, t.n0 + C::kPanelCols * c, k0,
                            t.expert);
            } else {
              tma_load_3d(smem_u32(sb), &p.tmap_b, fb, k0, t.n0, t.expert);
            }
          } else if (kBMnMajor) {
            // B[e] is [K, N] (N contiguous): BN/64 panels of [BK rows][64 cols];
            // SwiGLU tiles take two gate panels and the two matching up panels.
#pragma unroll
            for (int c = 0; c < C::BN / 64; ++c) {
              const int col = !p.act ? t.n0 + 64 * c
                                     : (c < 2 ? (t.n0 >> 1) + 64 * c : p.act_cols + (t.n0 >> 1) + 64 * (c - 2));
              tma_load_3d(smem_u32(sb + c * (C::BK * 128)), &p.tmap_b, fb, col, k0, t.expert);
            }
          } else if (p.act) {  // K-major [gate rows | up rows], 128 each (box of 128 rows)
            tma_load_3d(smem_u32(sb), &p.tmap_b, fb, k0, t.n0 >> 1, t.expert);
            tma_load_3d(smem_u32(sb + 128 * 128), &p.tmap_b, fb, k0, p.act_cols + (t.n0 >> 1), t.expert);
          } else {
            tma_load_3d(smem_u32(sb), &p.tmap_b, fb, k0, t.n0, t.expert);
          }
          issued[stage]++;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let every copy already in flight land before the CTA can exit.
        for (int s = 0; s < C::kStages; ++s)
          if (issued[s] > 0) mbar_wait_drain(smem_u32(full_bar + s), (issued[s] - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(tempty_bar + acc), acc_phase ^ 1, abort_flag, wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32((C::kTf32 ? conv_bar : full_bar) + stage), phase, abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
          const uint32_t sb = sa + C::kParts * C::kABytes;
#pragma unroll
          for (int ks = 0; ks < C::kKSteps; ++ks) {
            const uint32_t acc_flag = (kb | ks) != 0 ? 1u : 0u;
            const uint64_t adesc = make_sw128_desc(sa + ks * 32, 16, 1024);
            uint64_t bdesc;
            if (kBMnMajor && C::kTf32)  // MN-major tf32: 32-byte-atom swizzle
              bdesc = make_sw128_atom32_desc(sb + ks * C::kUmmaK * 128, C::BK * 128, 512);
            else if (kBMnMajor)
              bdesc = make_sw128_desc(sb + ks * C::kUmmaK * 128, C::BK * 128, 1024);
            else
              bdesc = make_sw128_desc(sb + ks * 32, 16, 1024);
            if (C::kTf32) {
              const uint64_t adesc_lo = make_sw128_desc(sa + C::kABytes + ks * 32, 16, 1024);
              const uint64_t bdesc_lo =
                  kBMnMajor ? make_sw128_atom32_desc(sb + C::kBBytes + ks * C::kUmmaK * 128, C::BK * 128, 512)
                            : make_sw128_desc(sb + C::kBBytes + ks * 32, 16, 1024);
              mma_tf32_ss(d_tmem, adesc, bdesc, C::kIdesc, acc_flag);    // hi * hi
              mma_tf32_ss(d_tmem, adesc, bdesc_lo, C::kIdesc, 1u);      // hi * lo
              mma_tf32_ss(d_tmem, adesc_lo, bdesc, C::kIdesc, 1u);      // lo * hi
            } else {
              mma_f16_ss(d_tmem, adesc, bdesc, C::kIdesc, acc_flag);
            }
          }
          mma_commit(smem_u32(empty_bar + stage));  // frees the stage once these MMAs retire
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(smem_u32(tfull_bar + acc));  // accumulator ready for the epilogue
      }
      // Retire every MMA this thread issued before TMEM can be released.
      mma_commit(smem_u32(drain_bar));
      mbar_wait_drain(smem_u32(drain_bar), 0);
    }
  } else if (C::kTf32 && (warp == 2 || warp == 3)) {
    split_stages();
  } else if (warp >= 4) {
    // Single-tile fp32 CTA: help split the stages first (the one accumulator
    // cannot be ready before the last stage is split).
    if (C::kTf32 && conv_warps == 6) split_stages();
    // ------------------------------------------------------------ epilogue
    using OutT = typename std::conditional<C::kTf32, float,
        typename std::conditional<kKind == kKindBf16, __nv_bfloat16, __half>::type>::type;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t stage = smem_u32(epi_stage) + quarter * (32 * 128);
    int g = 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(tfull_bar + acc), acc_phase, abort_flag, wait_ns)) break;
      tc_fence_after();
      const Tile t = decode_tile<C::BM, C::BN>(tv, n_tiles, tile, g);
      if (quarter * 32 < t.rows) {  // warp-uniform: some row of this quarter is live
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::BN;
        if constexpr (!C::kTf32) {
          if (p.act) {
            drain_slab_swiglu<OutT>(p, tv, g, t.row0 + quarter * 32, min(32, t.rows - quarter * 32),
                                    t.n0 >> 1, taddr, stage, lane);
          } else {
            drain_slab<OutT, C::BN>(p, tv, g, t.row0 + quarter * 32, min(32, t.rows - quarter * 32),
                                    t.n0, taddr, stage, lane);
          }
        } else {
          drain_slab<OutT, C::BN>(p, tv, g, t.row0 + quarter * 32, min(32, t.rows - quarter * 32), t.n0,
                                  taddr, stage, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(tempty_bar + acc));
    }
    if (p.remote) __threadfence_system();  // peer stores performed before the kernel ends
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(&g_device_error, 0, GMM_ERR_DEVICE_TIMEOUT);
}

// ------------------------------------------------------------ expert-parallel dispatch
constexpr int kMaxGatherChunks = 2048;

struct GatherParams {
  const char* src[kMaxPeers];  // each rank's token rows (peer-accessible)
  char* x;                     // this rank's expert-major receive buffer
  long long row_bytes;
  int n_chunks;
  int total_rows;
  int chunk_dst[kMaxGatherChunks + 1];  // first row of each chunk in x (prefix sums)
  int chunk_rank[kMaxGatherChunks];     // source rank of the chunk
  int chunk_row[kMaxGatherChunks];      // first row of the chunk in the source
};

// One warp per row: pull each row of x from the rank it lives on over
// NVLink (plain peer loads, 16 bytes per lane, 4 in flight per lane).
__global__ void __launch_bounds__(256) ep_gather_kernel(const __grid_constant__ GatherParams p) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < p.total_rows; row += warps) {
    int lo = 0, hi = p.n_chunks - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.chunk_dst[mid] <= row) lo = mid; else hi = mid - 1;
    }
    const uint4* src = reinterpret_cast<const uint4*>(
        p.src[p.chunk_rank[lo]] + static_cast<long long>(p.chunk_row[lo] + row - p.chunk_dst[lo]) * p.row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(p.x + static_cast<long long>(row) * p.row_bytes);
    const int n16 = static_cast<int>(p.row_bytes >> 4);
    int i = lane;
    for (; i + 96 < n16; i += 128) {
      const uint4 v0 = src[i], v1 = src[i + 32], v2 = src[i + 64], v3 = src[i + 96];
      dst[i] = v0;
      dst[i + 32] = v1;
      dst[i + 64] = v2;
      dst[i + 96] = v3;
    }
    for (; i < n16; i += 32) dst[i] = src[i];
  }
}

// ------------------------------------------------------------ expert-parallel barrier
struct BarrierParams {
  int* flags[kMaxPeers];  // each rank's flag slots (peer-accessible), flags[s][r] = last epoch rank r posted to s
  int world;
  int rank;
  int epoch;
  unsigned long long timeout_ns;
};

// Cross-rank barrier over peer memory, one thread per rank: thread s posts
// this rank's epoch into rank s's slot for us (release, system scope: every
// write this rank made earlier in the stream, its peer stores included, is
// visible to s before the flag), then waits until rank s has posted the same
// epoch here (acquire).  The wait is bounded: past timeout_ns it records
// GMM_ERR_DEVICE_TIMEOUT in the device error word and returns.
__global__ void __launch_bounds__(32) ep_barrier_kernel(const __grid_constant__ BarrierParams p) {
  const int s = threadIdx.x;
  if (s >= p.world) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p.flags[s] + p.rank), "r"(p.epoch) : "memory");
  const int* mine = p.flags[p.rank] + s;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (v - p.epoch >= 0) break;  // epochs only grow; the difference is wrap-safe
    if (global_timer_ns() - t0 > p.timeout_ns) {
      atomicCAS(&g_device_error, 0, GMM_ERR_DEVICE_TIMEOUT);
      break;
    }
    __nanosleep(64);
  }
}

#include "gmm_pair_kernel.cuh"
#include "gmm_vark_kernel.cuh"
#include "gmm_swap_kernel.cuh"

}  // namespace gmm_sm100

// =====================================================================  host side
namespace {

using namespace gmm_sm100;

thread_local std::string t_last_error;

// NVTX range around the host half of an entry point (plan building, tensor
// maps, launch): shows in Nsight Systems / Compute timelines next to the
// kernels it enqueues; without an attached tool it costs a few nanoseconds.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(GMM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::atomic<int> state{0};  // 0 unknown, 1 ok, 2 wrong arch
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  // Bit per kernel variant whose shared-memory attribute is set: 0 fp32;
  // 1-4 128-row bf16/fp16 x NT/NN; 5-8 CTA pair; 9-10 variable-K bf16/fp16;
  // 11-14 swap-AB bf16/fp16 x NT/NN.
  std::atomic<unsigned> smem_attr_set{0};
  int pair_clusters[16] = {};               // resident CTA pairs per pair-kernel variant
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(int dev, DeviceInfo** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(GMM_ERR_INVALID_ARGUMENT, "device index out of range");
  DeviceInfo& d = g_dev[dev];
  if (d.state.load(std::memory_order_acquire) == 0) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (d.state.load() == 0) {
      cudaError_t e;
      if ((e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
          (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
          (e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return cuda_fail(e, "cudaDeviceGetAttribute");
      d.state.store((d.cc_major == 10 && d.cc_minor == 0) ? 1 : 2, std::memory_order_release);
    }
  }
  *out = &d;
  if (d.state.load() != 1)
    return fail(GMM_ERR_ARCH, "gmm_sm100 requires a compute capability 10.0 (B200) GPU, got " +
                                  std::to_string(d.cc_major) + "." + std::to_string(d.cc_minor));
  return GMM_OK;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Plan {
  int num_groups = 0;
  int n_tiles = 0, k_blocks = 0, total_tiles = 0;
  std::vector<int32_t> table;
  size_t table_bytes = 0;    // device table bytes (0 when inline)
};

int elem_size(int dtype) { return dtype == GMM_DTYPE_F32 ? 4 : 2; }

int make_plan(const int64_t* bs, int64_t E, int64_t T, int64_t K, int64_t N, int dtype, Plan& pl,
              int64_t tile_rows = 128) {
  if (E < 0 || T < 0 || K < 0 || N < 0) return fail(GMM_ERR_INVALID_ARGUMENT, "negative size");
  if (E > 0 && !bs) return fail(GMM_ERR_INVALID_ARGUMENT, "batch_sizes is null");
  if (dtype != GMM_DTYPE_F32 && dtype != GMM_DTYPE_BF16 && dtype != GMM_DTYPE_F16)
    return fail(GMM_ERR_DTYPE, "Unsupported dtype: only FP32 / BF16 / FP16 are supported");
  const int64_t BM = tile_rows;
  const int64_t BN = dtype == GMM_DTYPE_F32 ? 128 : 256;
  const int64_t BK = dtype == GMM_DTYPE_F32 ? 32 : 64;
  int64_t sum = 0, groups = 0, mtiles = 0;
  for (int64_t e = 0; e < E; ++e) {
    if (bs[e] < 0) return fail(GMM_ERR_INVALID_ARGUMENT, "batch_sizes[" + std::to_string(e) + "] is negative");
    sum += bs[e];
    if (bs[e] > 0) {
      ++groups;
      mtiles += (bs[e] + BM - 1) / BM;
    }
  }
  if (sum != T)
    return fail(GMM_ERR_BATCH_SUM, "Sum of batch_sizes (" + std::to_string(sum) +
                                       ") must equal A.size(0) (" + std::to_string(T) + ")");
  if (T > INT32_MAX - 256 || K > INT32_MAX || N > INT32_MAX || E > INT32_MAX)
    return fail(GMM_ERR_TOO_LARGE, "a dimension exceeds the int32 coordinate range");
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t total = mtiles * n_tiles;
  if (total > INT32_MAX) return fail(GMM_ERR_TOO_LARGE, "too many output tiles");
  pl.num_groups = static_cast<int>(groups);
  pl.n_tiles = static_cast<int>(n_tiles);
  pl.k_blocks = static_cast<int>((K + BK - 1) / BK);
  pl.total_tiles = static_cast<int>(total);
  pl.table.assign(3 * groups + 2, 0);
  int32_t* row_off = pl.table.data();
  int32_t* tile_off = row_off + groups + 1;
  int32_t* expert = tile_off + groups + 1;
  int64_t row = 0, tiles = 0, g = 0;
  for (int64_t e = 0; e < E; ++e) {
    if (bs[e] > 0) {
      row_off[g] = static_cast<int32_t>(row);
      tile_off[g] = static_cast<int32_t>(tiles);
      expert[g] = static_cast<int32_t>(e);
      ++g;
      tiles += (bs[e] + BM - 1) / BM;
    }
    row += bs[e];
  }
  row_off[groups] = static_cast<int32_t>(row);
  tile_off[groups] = static_cast<int32_t>(tiles);
  pl.table_bytes = groups > kInlineGroups ? round_up(pl.table.size() * sizeof(int32_t), 256) : 0;
  return GMM_OK;
}

int encode(CUtensorMap* m, CUtensorMapDataType type, int rank, const void* ptr,
           const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
           CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_tiled();
  if (!fn) return fail(GMM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, type, rank, const_cast<void*>(ptr), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return GMM_OK;
}

// Launch one instantiation of a kernel with its shared-memory attribute set
// once per device (bit `bit` of smem_attr_set).
template <typename P>
int launch_with(void (*kern)(P), const P& prm, int grid, int smem, cudaStream_t stream, DeviceInfo* di, int bit,
                const char* what) {
  if (!(di->smem_attr_set.load() & (1u << bit))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    di->smem_attr_set.fetch_or(1u << bit);
  }
  kern<<<grid, kThreads, smem, stream>>>(prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return GMM_OK;
}

// The small-table copy of `prm`, when its inline table (if any) fits.
bool small_params(const GmmParams& prm, GmmParamsSmall& sp) {
  if (prm.inline_ints > kSmallTableInts) return false;
  static_cast<GmmParamsBase&>(sp) = static_cast<const GmmParamsBase&>(prm);
  std::memcpy(sp.inline_table, prm.inline_table, static_cast<size_t>(prm.inline_ints) * sizeof(int32_t));
  return true;
}

// A launch whose table travels in the parameters must say how much of it is
// in use; anything else would hand the kernel a cut-off table.
int check_table(const GmmParams& prm) {
  if (prm.num_groups > 0 && prm.ext_table == nullptr && prm.dev_bs == nullptr &&
      prm.inline_ints < 3 * prm.num_groups + 2)
    return fail(GMM_ERR_INVALID_ARGUMENT, "internal: inline tile table size not set");
  return GMM_OK;
}

// Small-table instantiations use bit + 16 of smem_attr_set (bits 0-15 are
// taken by the full-table variants and the pair and variable-K kernels).
template <int kKind, bool kMn>
int launch_variant(const GmmParams& prm, int grid, cudaStream_t stream, DeviceInfo* di, int bit) {
  using C = Cfg<kKind, kMn>;
  if (int rc = check_table(prm)) return rc;
  GmmParamsSmall sp;
  if (small_params(prm, sp))
    return launch_with(gmm_persistent_kernel<kKind, kMn, GmmParamsSmall>, sp, grid, C::kSmemBytes, stream, di,
                       bit + 16, "gmm kernel launch");
  return launch_with(gmm_persistent_kernel<kKind, kMn>, prm, grid, C::kSmemBytes, stream, di, bit,
                     "gmm kernel launch");
}

// Launch the CTA-pair kernel: clusters of 2 CTAs, as many pairs as can be
// resident at once (capped by the tile count).
template <int kKind, bool kMn>
int launch_pair(const GmmParams& prm, int total_tiles, cudaStream_t stream, DeviceInfo* di, int bit) {
  using C = PairCfg<kKind, kMn>;
  auto kern = gmm_pair_kernel<kKind, kMn>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!(di->smem_attr_set.load() & (1u << bit))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair)");
    cfg.gridDim = dim3(2 * std::max(1, di->sm_count / 2), 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters <= 0) clusters = di->sm_count / 2;
    di->pair_clusters[bit] = clusters;
    di->smem_attr_set.fetch_or(1u << bit);
  }
  const int pairs = std::max(1, std::min(total_tiles, di->pair_clusters[bit]));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm);
  if (e != cudaSuccess) return cuda_fail(e, "gmm pair kernel launch");
  return GMM_OK;
}

template <int kKind, bool kMn>
int launch_swap(const GmmParams& prm, int grid, cudaStream_t stream, DeviceInfo* di, int bit) {
  using C = SwapCfg<kKind, kMn>;
  if (int rc = check_table(prm)) return rc;
  GmmParamsSmall sp;
  if (small_params(prm, sp))
    return launch_with(gmm_swap_kernel<kKind, kMn, GmmParamsSmall>, sp, grid, C::kSmemBytes, stream, di, bit + 16,
                       "gmm swap kernel launch");
  return launch_with(gmm_swap_kernel<kKind, kMn>, prm, grid, C::kSmemBytes, stream, di, bit,
                     "gmm swap kernel launch");
}

// Tile kind of a problem.  fp32: 128-row tiles.  16-bit: CTA-pair 256-row
// tiles when the non-empty experts average at least 384 rows; swap-AB tiles
// when no expert has more than 64 rows (decode-shaped routing, where a
// 128-row tile would be at least half padding) and neither the SwiGLU nor the
// expert-parallel epilogue is needed; else single-CTA 128-row tiles.
// A process-wide override (gmm_sm100_set_tile_kind; initially from
// GMM_SM100_TILE=128 / 256 / swap, read once) forces one of them (swap falls
// back to 128 for the SwiGLU and expert-parallel epilogues, which it does not
// have).
enum TileKind { kTile128 = 0, kTilePair = 1, kTileSwap = 2 };

std::atomic<int> g_tile_force{-1};  // a gmm_tile_kind; -1 = not initialised yet
std::once_flag g_tile_force_once;

int tile_force() {
  std::call_once(g_tile_force_once, [] {
    const char* s = std::getenv("GMM_SM100_TILE");
    int k = GMM_TILE_AUTO;
    if (s && std::strcmp(s, "128") == 0) k = GMM_TILE_128;
    else if (s && std::strcmp(s, "256") == 0) k = GMM_TILE_PAIR;
    else if (s && std::strcmp(s, "swap") == 0) k = GMM_TILE_SWAP;
    int expect = -1;
    g_tile_force.compare_exchange_strong(expect, k);  // a setter call that came first wins
  });
  return g_tile_force.load(std::memory_order_relaxed);
}

TileKind choose_tile_kind(const int64_t* bs, int64_t E, int64_t T, int dtype, int act, bool remote) {
  if (dtype == GMM_DTYPE_F32) return kTile128;
  const bool swap_ok = !act && !remote;
  const int force = tile_force();
  if (force == GMM_TILE_128) return kTile128;
  if (force == GMM_TILE_PAIR) return kTilePair;
  if (force == GMM_TILE_SWAP) return swap_ok ? kTileSwap : kTile128;
  int64_t groups = 0, max_m = 0;
  for (int64_t e = 0; e < E; ++e) {
    groups += bs[e] > 0;
    max_m = std::max(max_m, bs[e]);
  }
  if (groups > 0 && T >= 384 * groups) return kTilePair;
  return (swap_ok && max_m <= 64) ? kTileSwap : kTile128;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Expert-parallel routing of a local grouped GEMM: rows of local expert e
// arrive from source ranks s = 0..world-1 in order (counts[e*world + s] rows
// each) and their results go back to row dst_rows[e*world + s] of rank s's
// output buffer out_peers[s].
struct EpRoute {
  int world;
  void* const* out_peers;
  const int64_t* counts;    // [E_local][world], segment order
  const int64_t* dst_rows;  // [E_local][world], segment order
  int rank_base;            // segment j comes from rank (rank_base + j) % world
};

// Append src_off[G][W+1] | dst_row[G][W] for the non-empty groups and decide
// whether the table still fits in the kernel parameters.
bool append_ep_table(Plan& pl, const int64_t* local_bs, int64_t E, const EpRoute& ep) {
  const int W = ep.world;
  std::vector<int32_t> src, dst;
  for (int64_t e = 0; e < E; ++e) {
    if (local_bs[e] <= 0) continue;
    int64_t acc = 0;
    for (int s = 0; s < W; ++s) {
      src.push_back(static_cast<int32_t>(acc));
      acc += ep.counts[e * W + s];
      if (ep.dst_rows[e * W + s] < 0 || ep.dst_rows[e * W + s] > INT32_MAX) return false;
      dst.push_back(static_cast<int32_t>(ep.dst_rows[e * W + s]));
    }
    src.push_back(static_cast<int32_t>(acc));
  }
  pl.table.insert(pl.table.end(), src.begin(), src.end());
  pl.table.insert(pl.table.end(), dst.begin(), dst.end());
  pl.table_bytes = pl.table.size() > static_cast<size_t>(kInlineTableInts)
                       ? round_up(pl.table.size() * sizeof(int32_t), 256)
                       : 0;
  return true;
}

// Tensor maps and the launch of the chosen kernel variant.  `grid_tiles`
// caps the grid (the tile count when the host knows it).
int setup_and_launch(GmmParams& prm, const void* A, const void* B, int64_t T, int64_t K, int64_t N, int64_t E,
                     int dtype, int trans_b, int64_t tile_rows, int act, int grid_tiles, DeviceInfo* di,
                     cudaStream_t stream, bool swap = false) {
  int rc = GMM_OK;
  const cuuint64_t uT = T, uK = K, uN = N, uE = E;
  if (dtype == GMM_DTYPE_F32) {  // raw fp32 operands; the kernel splits them into TF32 hi/lo in shared memory
    const cuuint64_t adims[2] = {uK, uT}, astr[1] = {uK * 4};
    const cuuint32_t abox[2] = {32, 128};
    if ((rc = encode(&prm.tmap_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, A, adims, astr, abox))) return rc;
    if (trans_b) {  // B[e] is [N, K], K contiguous
      const cuuint64_t bdims[3] = {uK, uN, uE}, bstr[2] = {uK * 4, uN * uK * 4};
      const cuuint32_t bbox[3] = {32, 128, 1};
      if ((rc = encode(&prm.tmap_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, B, bdims, bstr, bbox))) return rc;
    } else {  // B[e] is [K, N], N contiguous: [32 k][32 cols] panels, 32-byte-atom swizzle (MN-major tf32)
      const cuuint64_t bdims[3] = {uN, uK, uE}, bstr[2] = {uN * 4, uK * uN * 4};
      const cuuint32_t bbox[3] = {32, 32, 1};
      if ((rc = encode(&prm.tmap_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, B, bdims, bstr, bbox,
                       CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)))
        return rc;
    }
  } else {
    const CUtensorMapDataType tt =
        dtype == GMM_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint64_t adims[2] = {uK, uT}, astr[1] = {uK * 2};
    const cuuint32_t abox[2] = {64, 128};
    if ((rc = encode(&prm.tmap_a, tt, 2, A, adims, astr, abox))) return rc;
    if (tile_rows == 256) {  // half tiles of the CTA-pair kernel: 64 A rows per CTA
      const cuuint32_t abox_half[2] = {64, 64};
      if ((rc = encode(&prm.tmap_a2, tt, 2, A, adims, astr, abox_half))) return rc;
    }
    if (trans_b) {  // B[e] is [N, K], K contiguous; a CTA of a pair holds half the tile's columns
      const cuuint64_t bdims[3] = {uK, uN, uE}, bstr[2] = {uK * 2, uN * uK * 2};
      const cuuint32_t bbox[3] = {64, (tile_rows == 256 || act) ? 128u : 256u, 1};
      if ((rc = encode(&prm.tmap_b, tt, 3, B, bdims, bstr, bbox))) return rc;
    } else {  // B[e] is [K, N], N contiguous
      const cuuint64_t bdims[3] = {uN, uK, uE}, bstr[2] = {uN * 2, uK * uN * 2};
      const cuuint32_t bbox[3] = {64, 64, 1};
      if ((rc = encode(&prm.tmap_b, tt, 3, B, bdims, bstr, bbox))) return rc;
    }
  }

  const int grid = std::max(1, std::min(grid_tiles, di->sm_count));
  if (dtype == GMM_DTYPE_F32)
    return trans_b ? launch_variant<kKindTf32x3, false>(prm, grid, stream, di, 0)
                   : launch_variant<kKindTf32x3, true>(prm, grid, stream, di, 15);
  if (swap) {
    if (dtype == GMM_DTYPE_BF16)
      return trans_b ? launch_swap<kKindBf16, false>(prm, grid, stream, di, 11)
                     : launch_swap<kKindBf16, true>(prm, grid, stream, di, 12);
    return trans_b ? launch_swap<kKindF16, false>(prm, grid, stream, di, 13)
                   : launch_swap<kKindF16, true>(prm, grid, stream, di, 14);
  }
  if (tile_rows == 256) {
    if (dtype == GMM_DTYPE_BF16)
      return trans_b ? launch_pair<kKindBf16, false>(prm, grid_tiles, stream, di, 5)
                     : launch_pair<kKindBf16, true>(prm, grid_tiles, stream, di, 6);
    return trans_b ? launch_pair<kKindF16, false>(prm, grid_tiles, stream, di, 7)
                   : launch_pair<kKindF16, true>(prm, grid_tiles, stream, di, 8);
  }
  if (dtype == GMM_DTYPE_BF16)
    return trans_b ? launch_variant<kKindBf16, false>(prm, grid, stream, di, 1)
                   : launch_variant<kKindBf16, true>(prm, grid, stream, di, 2);
  return trans_b ? launch_variant<kKindF16, false>(prm, grid, stream, di, 3)
                 : launch_variant<kKindF16, true>(prm, grid, stream, di, 4);
}

// The host half of a forward call: the tile table and the kernel choice,
// from the host batch sizes alone (no CUDA call).
struct PlanObj {
  Plan pl;
  TileKind kind = kTile128;
  int64_t tile_rows = 128;
  int64_t E = 0, T = 0, K = 0, N = 0;
  int dtype = 0, trans_b = 0;
};

int plan_impl(const int64_t* batch_sizes, int64_t num_experts, int64_t num_tokens, int64_t dim,
              int64_t dim_out, int dtype, int trans_b, int act, bool remote, PlanObj& po) {
  NvtxRange range("gmm_sm100 plan");
  int rc = make_plan(batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, po.pl);
  if (rc != GMM_OK) return rc;
  po.kind = choose_tile_kind(batch_sizes, num_experts, num_tokens, dtype, act, remote);
  po.tile_rows = po.kind == kTilePair ? 256 : 128;
  if (po.tile_rows != 128 &&
      (rc = make_plan(batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, po.pl, po.tile_rows)) != GMM_OK)
    return rc;
  po.E = num_experts;
  po.T = num_tokens;
  po.K = dim;
  po.N = dim_out;
  po.dtype = dtype;
  po.trans_b = trans_b;
  return GMM_OK;
}

// Test hook of the bounded-wait path (gmm_sm100_forward_inject_timeout).
struct InjectTimeout {
  int drop_k_block;
  unsigned long long wait_ns;
};

// The device half: argument checks that need the pointers, tensor maps, launch.
// `pl` is the plan's table (with the expert-parallel segments appended in EP mode).
int launch_impl(const PlanObj& po, const Plan& pl, const void* A, const void* B, void* D, void* workspace,
                size_t workspace_bytes, void* stream_ptr, const EpRoute* ep, int act,
                const InjectTimeout* inject = nullptr) {
  NvtxRange range("gmm_sm100 launch");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int rc = GMM_OK;
  const TileKind kind = po.kind;
  const int64_t tile_rows = po.tile_rows;
  const int64_t T = po.T, K = po.K, N = po.N, E = po.E;
  const int dtype = po.dtype, trans_b = po.trans_b;
  if (T == 0 || N == 0) return GMM_OK;  // nothing to write
  const int es = elem_size(dtype);
  // SwiGLU: B has 2*I output columns ([gate | up]); D has I = N / 2 columns.
  const int64_t N_out = act ? N / 2 : N;
  if (act) {
    if (dtype == GMM_DTYPE_F32) return fail(GMM_ERR_DTYPE, "the fused SwiGLU path takes bf16 / fp16");
    if (N % 16 != 0)
      return fail(GMM_ERR_ALIGNMENT, "SwiGLU needs the gate/up width (dim_out / 2) to be a multiple of 8");
  }
  if (ep) {
    if (ep->world < 1 || ep->world > kMaxPeers || !ep->out_peers)
      return fail(GMM_ERR_INVALID_ARGUMENT, "expert-parallel world must be 1.." + std::to_string(kMaxPeers));
    for (int s = 0; s < ep->world; ++s)
      if (!ep->out_peers[s] || !aligned16(ep->out_peers[s]))
        return fail(GMM_ERR_ALIGNMENT, "every rank's output buffer must be non-null and 16-byte aligned");
    if (K == 0) return fail(GMM_ERR_INVALID_ARGUMENT, "expert-parallel forward needs dim > 0");
  } else {
    if (!D) return fail(GMM_ERR_INVALID_ARGUMENT, "D is null");
    if (!aligned16(D)) return fail(GMM_ERR_ALIGNMENT, "D must be 16-byte aligned");
  }
  if ((N * es) % 16 != 0)
    return fail(GMM_ERR_ALIGNMENT, "dim_out * element size must be a multiple of 16 bytes, got dim_out=" +
                                       std::to_string(N));
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceInfo* di = nullptr;
  if ((rc = device_info(dev, &di)) != GMM_OK) return rc;
  if (K == 0) {  // empty contraction: D = 0 (SwiGLU: silu(0) * 0 = 0)
    ce = cudaMemsetAsync(D, 0, static_cast<size_t>(T) * N_out * es, stream);
    return ce == cudaSuccess ? GMM_OK : cuda_fail(ce, "cudaMemsetAsync");
  }
  if (!A || !B) return fail(GMM_ERR_INVALID_ARGUMENT, "A or B is null");
  if (!aligned16(A) || !aligned16(B)) return fail(GMM_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
  if ((K * es) % 16 != 0)
    return fail(GMM_ERR_ALIGNMENT, "dim * element size must be a multiple of 16 bytes, got dim=" +
                                       std::to_string(K));
  const size_t need = pl.table_bytes;
  if (need > 0 && (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u)))
    return fail(GMM_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes (256-byte aligned), got " +
                                       std::to_string(workspace_bytes));

  static_assert(sizeof(GmmParams) <= 32764, "kernel parameter limit");
  GmmParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.d = D;
  prm.ldd = N_out;
  prm.num_groups = pl.num_groups;
  prm.n_tiles = pl.n_tiles;
  prm.k_blocks = pl.k_blocks;
  prm.total_tiles = pl.total_tiles;
  prm.dim_out = static_cast<int>(N_out);
  prm.act = act;
  prm.act_cols = act ? static_cast<int>(N_out) : 0;
  prm.tile_rows = static_cast<int>(tile_rows);
  if (inject) {
    prm.drop_kb1 = inject->drop_k_block + 1;
    prm.wait_ns = inject->wait_ns;
  }
  if (ep) {
    prm.remote = 1;
    prm.world = ep->world;
    prm.ep_rank_base = ((ep->rank_base % ep->world) + ep->world) % ep->world;
    for (int s = 0; s < ep->world; ++s) prm.d_peer[s] = ep->out_peers[s];
  }
  if (pl.table_bytes == 0) {
    std::memcpy(prm.inline_table, pl.table.data(), pl.table.size() * sizeof(int32_t));
    prm.inline_ints = static_cast<int>(pl.table.size());
    prm.ext_table = nullptr;
  } else {
    ce = cudaMemcpyAsync(workspace, pl.table.data(), pl.table.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                         stream);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaMemcpyAsync(table)");
    prm.ext_table = static_cast<const int32_t*>(workspace);
  }

  return setup_and_launch(prm, A, B, T, K, N, E, dtype, trans_b, tile_rows, act, pl.total_tiles, di, stream,
                          kind == kTileSwap);
}

int forward_impl(const void* A, const void* B, const int64_t* batch_sizes, int64_t num_experts,
                 int64_t num_tokens, int64_t dim, int64_t dim_out, int dtype, int trans_b, void* D,
                 void* workspace, size_t workspace_bytes, void* stream_ptr, const EpRoute* ep,
                 int act = 0) {
  PlanObj po;
  int rc = plan_impl(batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, trans_b, act, ep != nullptr, po);
  if (rc != GMM_OK) return rc;
  if (ep && num_tokens > 0 && dim_out > 0 && ep->world >= 1 && ep->world <= kMaxPeers &&
      !append_ep_table(po.pl, batch_sizes, num_experts, *ep))
    return fail(GMM_ERR_TOO_LARGE, "EP table too large");
  return launch_impl(po, po.pl, A, B, D, workspace, workspace_bytes, stream_ptr, ep, act);
}

}  // namespace

struct gmm_sm100_plan_s {
  PlanObj po;
};

extern "C" {

const char* gmm_sm100_errstr(int status) {
  switch (status) {
    case GMM_OK: return "ok";
    case GMM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case GMM_ERR_BATCH_SUM: return "sum of batch_sizes does not match the number of rows";
    case GMM_ERR_DTYPE: return "unsupported dtype";
    case GMM_ERR_ALIGNMENT: return "misaligned pointer or row pitch";
    case GMM_ERR_ARCH: return "unsupported GPU architecture (needs sm_100)";
    case GMM_ERR_CUDA: return "CUDA error";
    case GMM_ERR_WORKSPACE: return "workspace too small";
    case GMM_ERR_TOO_LARGE: return "problem too large";
    case GMM_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

const char* gmm_sm100_last_error(void) { return t_last_error.c_str(); }

int gmm_sm100_set_tile_kind(int kind) {
  if (kind < GMM_TILE_AUTO || kind > GMM_TILE_SWAP)
    return fail(GMM_ERR_INVALID_ARGUMENT, "tile kind must be one of gmm_tile_kind");
  const int prev = tile_force();
  g_tile_force.store(kind, std::memory_order_relaxed);
  return prev;
}

int gmm_sm100_check_device(int device) {
  DeviceInfo* di = nullptr;
  return device_info(device, &di);
}

size_t gmm_sm100_workspace_size(const int64_t* batch_sizes, int64_t num_experts, int64_t num_tokens,
                                int64_t dim, int64_t dim_out, int dtype, int trans_b) {
  (void)trans_b;
  Plan pl;
  if (make_plan(batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, pl) != GMM_OK) return 0;
  return pl.table_bytes;
}

int gmm_sm100_forward(const void* A, const void* B, const int64_t* batch_sizes, int64_t num_experts,
                      int64_t num_tokens, int64_t dim, int64_t dim_out, int dtype, int trans_b,
                      void* D, void* workspace, size_t workspace_bytes, void* stream_ptr) {
  return forward_impl(A, B, batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, trans_b, D,
                      workspace, workspace_bytes, stream_ptr, nullptr);
}

int gmm_sm100_plan(const int64_t* batch_sizes, int64_t num_experts, int64_t num_tokens, int64_t dim,
                   int64_t dim_out, int dtype, int trans_b, gmm_sm100_plan_t** plan_out) {
  if (!plan_out) return fail(GMM_ERR_INVALID_ARGUMENT, "plan_out is null");
  *plan_out = nullptr;
  try {
    std::unique_ptr<gmm_sm100_plan_s> h(new gmm_sm100_plan_s);
    const int rc = plan_impl(batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, trans_b, 0, false, h->po);
    if (rc != GMM_OK) return rc;
    *plan_out = h.release();
    return GMM_OK;
  } catch (const std::exception& e) {
    return fail(GMM_ERR_TOO_LARGE, std::string("host allocation failed: ") + e.what());
  }
}

size_t gmm_sm100_plan_workspace_size(const gmm_sm100_plan_t* plan) {
  return plan ? plan->po.pl.table_bytes : 0;
}

int gmm_sm100_launch(const gmm_sm100_plan_t* plan, const void* A, const void* B, void* D, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!plan) return fail(GMM_ERR_INVALID_ARGUMENT, "plan is null");
  return launch_impl(plan->po, plan->po.pl, A, B, D, workspace, workspace_bytes, stream, nullptr, 0);
}

void gmm_sm100_plan_free(gmm_sm100_plan_t* plan) { delete plan; }

size_t gmm_sm100_ep_workspace_size(const int64_t* counts, int64_t num_local_experts, int world,
                                   int64_t num_rows, int64_t dim, int64_t dim_out, int dtype) {
  if (!counts || num_local_experts < 0 || world < 1 || world > kMaxPeers) return 0;
  std::vector<int64_t> local_bs(static_cast<size_t>(num_local_experts), 0);
  std::vector<int64_t> zeros(static_cast<size_t>(num_local_experts * world), 0);
  for (int64_t e = 0; e < num_local_experts; ++e)
    for (int s = 0; s < world; ++s) local_bs[e] += counts[e * world + s];
  Plan pl;
  if (make_plan(local_bs.data(), num_local_experts, num_rows, dim, dim_out, dtype, pl) != GMM_OK) return 0;
  EpRoute route{world, nullptr, counts, zeros.data(), 0};
  if (!append_ep_table(pl, local_bs.data(), num_local_experts, route)) return 0;
  return pl.table_bytes;
}

int gmm_sm100_forward_ep(const void* X, const void* B, const int64_t* counts, const int64_t* dst_rows,
                         int64_t num_local_experts, int world, int rank_base, void* const* out_peers,
                         int64_t num_rows, int64_t dim, int64_t dim_out, int dtype, int trans_b,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!counts || !dst_rows || num_local_experts < 0 || world < 1 || world > kMaxPeers)
    return fail(GMM_ERR_INVALID_ARGUMENT, "bad expert-parallel routing arguments");
  std::vector<int64_t> local_bs(static_cast<size_t>(num_local_experts), 0);
  for (int64_t e = 0; e < num_local_experts; ++e)
    for (int s = 0; s < world; ++s) {
      if (counts[e * world + s] < 0) return fail(GMM_ERR_INVALID_ARGUMENT, "negative row count");
      local_bs[e] += counts[e * world + s];
    }
  EpRoute route{world, out_peers, counts, dst_rows, rank_base};
  return forward_impl(X, B, local_bs.data(), num_local_experts, num_rows, dim, dim_out, dtype, trans_b,
                      nullptr, workspace, workspace_bytes, stream, &route);
}

int gmm_sm100_ep_gather(void* X, const void* const* src_peers, const int64_t* counts,
                        const int64_t* src_rows, int64_t num_local_experts, int world, int rank_base,
                        int64_t row_bytes, void* stream_ptr) {
  NvtxRange range("gmm_sm100 ep_gather");
  if (!counts || !src_rows || !src_peers || world < 1 || world > kMaxPeers || num_local_experts < 0)
    return fail(GMM_ERR_INVALID_ARGUMENT, "bad gather arguments");
  if (row_bytes <= 0 || row_bytes % 16 != 0)
    return fail(GMM_ERR_ALIGNMENT, "row bytes must be a positive multiple of 16");
  static_assert(sizeof(GatherParams) <= 32764, "kernel parameter limit");
  GatherParams prm;
  std::memset(&prm, 0, sizeof(prm));
  int64_t rows = 0;
  int n = 0;
  const int base = ((rank_base % world) + world) % world;
  for (int64_t e = 0; e < num_local_experts; ++e)
    for (int j = 0; j < world; ++j) {
      const int64_t m = counts[e * world + j];
      if (m < 0 || src_rows[e * world + j] < 0) return fail(GMM_ERR_INVALID_ARGUMENT, "negative count or row");
      if (m == 0) continue;
      if (src_rows[e * world + j] > INT32_MAX - m)  // the kernel indexes source rows in 32 bits
        return fail(GMM_ERR_TOO_LARGE, "source rows beyond the 32-bit row range");
      if (n >= kMaxGatherChunks) return fail(GMM_ERR_TOO_LARGE, "too many (expert, rank) chunks");
      prm.chunk_dst[n] = static_cast<int>(rows);
      prm.chunk_rank[n] = (base + j) % world;
      prm.chunk_row[n] = static_cast<int>(src_rows[e * world + j]);
      ++n;
      rows += m;
    }
  if (rows == 0) return GMM_OK;
  if (rows > INT32_MAX) return fail(GMM_ERR_TOO_LARGE, "too many rows");
  if (!X || !aligned16(X)) return fail(GMM_ERR_ALIGNMENT, "X must be non-null and 16-byte aligned");
  for (int s = 0; s < world; ++s) {
    prm.src[s] = static_cast<const char*>(src_peers[s]);
    if (prm.src[s] && !aligned16(prm.src[s])) return fail(GMM_ERR_ALIGNMENT, "source rows must be 16-byte aligned");
  }
  for (int c = 0; c < n; ++c)
    if (!prm.src[prm.chunk_rank[c]]) return fail(GMM_ERR_INVALID_ARGUMENT, "null source pointer");
  prm.chunk_dst[n] = static_cast<int>(rows);
  prm.x = static_cast<char*>(X);
  prm.row_bytes = row_bytes;
  prm.n_chunks = n;
  prm.total_rows = static_cast<int>(rows);
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceInfo* di = nullptr;
  int rc = device_info(dev, &di);
  if (rc != GMM_OK) return rc;
  const int blocks = static_cast<int>(std::min<int64_t>((rows + 7) / 8, 4LL * di->sm_count));
  ep_gather_kernel<<<std::max(blocks, 1), 256, 0, static_cast<cudaStream_t>(stream_ptr)>>>(prm);
  ce = cudaGetLastError();
  return ce == cudaSuccess ? GMM_OK : cuda_fail(ce, "ep gather launch");
}

int gmm_sm100_ep_barrier(int* const* flag_peers, int world, int rank, int epoch, double timeout_s,
                         void* stream_ptr) {
  NvtxRange range("gmm_sm100 ep_barrier");
  if (!flag_peers || world < 1 || world > kMaxPeers || rank < 0 || rank >= world || !(timeout_s > 0.0))
    return fail(GMM_ERR_INVALID_ARGUMENT, "bad barrier arguments");
  BarrierParams prm;
  std::memset(&prm, 0, sizeof(prm));
  for (int s = 0; s < world; ++s) {
    if (!flag_peers[s] || (reinterpret_cast<uintptr_t>(flag_peers[s]) & 3u))
      return fail(GMM_ERR_ALIGNMENT, "every rank's flag slots must be non-null and 4-byte aligned");
    prm.flags[s] = flag_peers[s];
  }
  prm.world = world;
  prm.rank = rank;
  prm.epoch = epoch;
  prm.timeout_ns = static_cast<unsigned long long>(std::min(timeout_s, 3600.0) * 1e9);
  ep_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream_ptr)>>>(prm);
  const cudaError_t ce = cudaGetLastError();
  return ce == cudaSuccess ? GMM_OK : cuda_fail(ce, "ep barrier launch");
}

int gmm_sm100_forward_swiglu(const void* A, const void* B, const int64_t* batch_sizes, int64_t num_experts,
                             int64_t num_tokens, int64_t dim, int64_t dim_out, int dtype, int trans_b,
                             void* D, void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(A, B, batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, trans_b, D,
                      workspace, workspace_bytes, stream, nullptr, 1);
}

size_t gmm_sm100_dev_workspace_size(int64_t num_experts, int64_t rows_cap, int64_t dim, int64_t dim_out,
                                    int dtype) {
  (void)num_experts, (void)rows_cap, (void)dim, (void)dim_out, (void)dtype;
  return 0;  // the kernels build their tables in shared memory and split fp32 in shared memory
}

int gmm_sm100_forward_dev(const void* A, const void* B, const int32_t* batch_sizes_dev, int64_t num_experts,
                          int64_t rows_cap, int64_t dim, int64_t dim_out, int dtype, int trans_b, int swiglu,
                          void* D, void* workspace, size_t workspace_bytes, void* stream_ptr) {
  NvtxRange range("gmm_sm100 forward_dev");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (num_experts < 1 || num_experts > kMaxDevExperts || rows_cap < 0 || dim < 0 || dim_out < 0)
    return fail(GMM_ERR_INVALID_ARGUMENT, "device batch sizes need 1 <= num_experts <= 1024");
  if (dtype != GMM_DTYPE_F32 && dtype != GMM_DTYPE_BF16 && dtype != GMM_DTYPE_F16)
    return fail(GMM_ERR_DTYPE, "Unsupported dtype: only FP32 / BF16 / FP16 are supported");
  if (swiglu && (dtype == GMM_DTYPE_F32 || dim_out % 16 != 0))
    return fail(GMM_ERR_INVALID_ARGUMENT, "SwiGLU takes bf16 / fp16 and dim_out a multiple of 16");
  if (rows_cap > INT32_MAX - 256 || dim > INT32_MAX || dim_out > INT32_MAX)
    return fail(GMM_ERR_TOO_LARGE, "a dimension exceeds the int32 coordinate range");
  const int64_t T = rows_cap, K = dim, N = dim_out, E = num_experts;
  if (T == 0 || N == 0) return GMM_OK;
  const int es = elem_size(dtype);
  const int64_t N_out = swiglu ? N / 2 : N;
  if (!D || !aligned16(D)) return fail(GMM_ERR_ALIGNMENT, "D must be non-null and 16-byte aligned");
  if (!batch_sizes_dev || (reinterpret_cast<uintptr_t>(batch_sizes_dev) & 3u))
    return fail(GMM_ERR_ALIGNMENT, "batch_sizes must be a 4-byte aligned device pointer");
  if ((N * es) % 16 != 0) return fail(GMM_ERR_ALIGNMENT, "dim_out * element size must be a multiple of 16 bytes");
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceInfo* di = nullptr;
  int rc = device_info(dev, &di);
  if (rc != GMM_OK) return rc;
  if (K == 0) {
    ce = cudaMemsetAsync(D, 0, static_cast<size_t>(T) * N_out * es, stream);
    return ce == cudaSuccess ? GMM_OK : cuda_fail(ce, "cudaMemsetAsync");
  }
  if (!A || !B || !aligned16(A) || !aligned16(B))
    return fail(GMM_ERR_ALIGNMENT, "A and B must be non-null and 16-byte aligned");
  if ((K * es) % 16 != 0) return fail(GMM_ERR_ALIGNMENT, "dim * element size must be a multiple of 16 bytes");
  (void)workspace, (void)workspace_bytes;  // none needed (gmm_sm100_dev_workspace_size is 0)
  // Tile kind from the capacity alone (the sizes are only known on the device):
  // CTA pairs when the capacity averages at least 384 rows per expert,
  // swap-AB tiles when it averages at most 16 (decode), else 128-row tiles.
  int64_t tile_rows = 128;
  bool swap = false;
  if (dtype != GMM_DTYPE_F32) {
    const int force = tile_force();
    if (force == GMM_TILE_PAIR) tile_rows = 256;
    else if (force == GMM_TILE_SWAP) swap = !swiglu;
    else if (force != GMM_TILE_128) {
      if (T >= 384 * E) tile_rows = 256;
      else swap = !swiglu && T <= 16 * E;
    }
  }
  const int64_t BN = dtype == GMM_DTYPE_F32 ? 128 : 256;
  const int64_t BK = dtype == GMM_DTYPE_F32 ? 32 : 64;
  GmmParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.d = D;
  prm.ldd = N_out;
  prm.n_tiles = static_cast<int>((N + BN - 1) / BN);
  prm.k_blocks = static_cast<int>((K + BK - 1) / BK);
  prm.dim_out = static_cast<int>(N_out);
  prm.act = swiglu ? 1 : 0;
  prm.act_cols = swiglu ? static_cast<int>(N_out) : 0;
  prm.dev_bs = batch_sizes_dev;
  prm.dev_experts = static_cast<int>(E);
  prm.rows_cap = static_cast<int>(T);
  prm.tile_rows = static_cast<int>(tile_rows);
  return setup_and_launch(prm, A, B, T, K, N, E, dtype, trans_b, tile_rows, prm.act, INT32_MAX, di, stream, swap);
}

int gmm_sm100_forward_vark(const void* A, const void* B, const int64_t* batch_sizes, int64_t num_experts,
                           int64_t num_tokens, int64_t dim_a, int64_t dim_b, int dtype, void* D,
                           void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int64_t E = num_experts, T = num_tokens, M = dim_a, N = dim_b;
  if (E < 0 || T < 0 || M < 0 || N < 0) return fail(GMM_ERR_INVALID_ARGUMENT, "negative size");
  if (E > 0 && !batch_sizes) return fail(GMM_ERR_INVALID_ARGUMENT, "batch_sizes is null");
  if (dtype != GMM_DTYPE_BF16 && dtype != GMM_DTYPE_F16)
    return fail(GMM_ERR_DTYPE, "the variable-K grouped GEMM takes bf16 / fp16");
  if (E + 1 > kInlineTableInts) return fail(GMM_ERR_TOO_LARGE, "too many experts for the variable-K kernel");
  int64_t sum = 0;
  for (int64_t e = 0; e < E; ++e) {
    if (batch_sizes[e] < 0) return fail(GMM_ERR_INVALID_ARGUMENT, "batch_sizes[" + std::to_string(e) + "] is negative");
    sum += batch_sizes[e];
  }
  if (sum != T)
    return fail(GMM_ERR_BATCH_SUM, "Sum of batch_sizes (" + std::to_string(sum) + ") must equal A.size(0) (" +
                                       std::to_string(T) + ")");
  if (E == 0 || M == 0 || N == 0) return GMM_OK;
  if (T > INT32_MAX - 256 || M > INT32_MAX || N > INT32_MAX) return fail(GMM_ERR_TOO_LARGE, "too large");
  if ((M * 2) % 16 != 0 || (N * 2) % 16 != 0)
    return fail(GMM_ERR_ALIGNMENT, "A and B row pitches must be multiples of 16 bytes");
  if (!D || !aligned16(D)) return fail(GMM_ERR_ALIGNMENT, "D must be non-null and 16-byte aligned");
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceInfo* di = nullptr;
  int rc = device_info(dev, &di);
  if (rc != GMM_OK) return rc;
  if (T == 0) {  // every expert is empty: D = 0
    ce = cudaMemsetAsync(D, 0, static_cast<size_t>(E) * M * N * 2, stream);
    return ce == cudaSuccess ? GMM_OK : cuda_fail(ce, "cudaMemsetAsync");
  }
  if (!A || !B || !aligned16(A) || !aligned16(B))
    return fail(GMM_ERR_ALIGNMENT, "A and B must be non-null and 16-byte aligned");
  const int64_t m_tiles = (M + 127) / 128, n_tiles = (N + 255) / 256;
  const int64_t total = E * m_tiles * n_tiles;
  if (total > INT32_MAX) return fail(GMM_ERR_TOO_LARGE, "too many output tiles");
  GmmParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.d = D;
  prm.ldd = N;
  prm.dim_out = static_cast<int>(N);
  prm.n_tiles = static_cast<int>(n_tiles);
  prm.vk_m = static_cast<int>(M);
  prm.vk_m_tiles = static_cast<int>(m_tiles);
  prm.total_tiles = static_cast<int>(total);
  prm.num_groups = static_cast<int>(E);
  int64_t row = 0;
  for (int64_t e = 0; e < E; ++e) {
    prm.inline_table[e] = static_cast<int32_t>(row);
    row += batch_sizes[e];
  }
  prm.inline_table[E] = static_cast<int32_t>(row);
  const CUtensorMapDataType tt =
      dtype == GMM_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t adims[2] = {static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(T)};
  const cuuint64_t astr[1] = {static_cast<cuuint64_t>(M) * 2};
  const cuuint64_t bdims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(T)};
  const cuuint64_t bstr[1] = {static_cast<cuuint64_t>(N) * 2};
  const cuuint32_t box[2] = {64, 64};
  if ((rc = encode(&prm.tmap_a, tt, 2, A, adims, astr, box)) || (rc = encode(&prm.tmap_b, tt, 2, B, bdims, bstr, box)))
    return rc;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(total, di->sm_count)));
  const int bit = dtype == GMM_DTYPE_BF16 ? 9 : 10;
  auto launch = [&](auto kern, int smem) -> int {
    if (!(di->smem_attr_set.load() & (1u << bit))) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(vark)");
      di->smem_attr_set.fetch_or(1u << bit);
    }
    kern<<<grid, kThreads, smem, stream>>>(prm);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GMM_OK : cuda_fail(e, "variable-K kernel launch");
  };
  return dtype == GMM_DTYPE_BF16 ? launch(gmm_vark_kernel<kKindBf16>, VarKCfg<kKindBf16>::kSmemBytes)
                                 : launch(gmm_vark_kernel<kKindF16>, VarKCfg<kKindF16>::kSmemBytes);
}

int gmm_sm100_forward_inject_timeout(const void* A, const void* B, const int64_t* batch_sizes,
                                     int64_t num_experts, int64_t num_tokens, int64_t dim, int64_t dim_out,
                                     int dtype, int trans_b, void* D, int drop_k_block, double wait_s,
                                     void* stream) {
  if (dtype != GMM_DTYPE_BF16 && dtype != GMM_DTYPE_F16)
    return fail(GMM_ERR_DTYPE, "the timeout test hook runs the 16-bit kernels");
  if (!(wait_s > 0.0 && wait_s <= 2.0) || drop_k_block < 0)
    return fail(GMM_ERR_INVALID_ARGUMENT, "wait_s must be in (0, 2] and drop_k_block >= 0");
  PlanObj po;
  int rc = plan_impl(batch_sizes, num_experts, num_tokens, dim, dim_out, dtype, trans_b, 0, false, po);
  if (rc != GMM_OK) return rc;
  if (po.kind == kTileSwap)
    return fail(GMM_ERR_INVALID_ARGUMENT, "the timeout test hook runs the 128-row and CTA-pair kernels");
  if (po.pl.table_bytes != 0 || drop_k_block >= po.pl.k_blocks || po.pl.total_tiles == 0)
    return fail(GMM_ERR_INVALID_ARGUMENT, "the timeout test hook needs a small problem with that k-block");
  const InjectTimeout inj{drop_k_block, static_cast<unsigned long long>(wait_s * 1e9)};
  return launch_impl(po, po.pl, A, B, D, nullptr, 0, stream, nullptr, 0, &inj);
}

int gmm_sm100_device_error(int* status_out, int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(g_device_error)");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(g_device_error)");
  }
  if (status_out) *status_out = v;
  return GMM_OK;
}

}  // extern "C"

// ============================================================ allocation-free fp32 entry
// The scratch of gmm_sm100_forward_f32_noalloc: a fixed device array in this
// library, so that callers which cannot allocate device memory can still use
// the fp32 (3xTF32) path.  Host code must not use the symbol's name as a
// pointer; the device address comes from cudaGetSymbolAddress, once per device.
namespace gmm_sm100 {
static __device__ __align__(256) unsigned char g_noalloc_scratch[GMM_SM100_NOALLOC_SCRATCH_BYTES];
}  // namespace gmm_sm100

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on device `dev` (which must be current),
// looked up once per device ordinal: the address in that device's primary
// context, which is where the runtime API (and so every launch here) runs.
int noalloc_scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, gmm_sm100::g_noalloc_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return GMM_OK;
}

}  // namespace

extern "C" int gmm_sm100_forward_f32_noalloc(const float* A, const float* B,
                                             const int64_t* batch_sizes, int64_t num_experts,
                                             int64_t num_tokens, int64_t dim, int64_t dim_out,
                                             int trans_b, float* D, void* stream_ptr) {
  NvtxRange range("gmm_sm100 forward_f32_noalloc");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  Plan pl;
  int rc = make_plan(batch_sizes, num_experts, num_tokens, dim, dim_out, GMM_DTYPE_F32, pl);
  if (rc != GMM_OK) return rc;
  const int64_t T = num_tokens, K = dim, N = dim_out, E = num_experts;
  if (T == 0 || N == 0) return GMM_OK;
  if (!D) return fail(GMM_ERR_INVALID_ARGUMENT, "D is null");
  if (!aligned16(D)) return fail(GMM_ERR_ALIGNMENT, "D must be 16-byte aligned");
  if ((N * 4) % 16 != 0)
    return fail(GMM_ERR_ALIGNMENT, "dim_out must be a multiple of 4 for fp32, got " + std::to_string(N));
  // The only scratch of the fp32 path is the tile table of more than 1024
  // non-empty experts (the TF32 split happens in shared memory).
  const size_t need = pl.table_bytes;
  if (need > GMM_SM100_NOALLOC_SCRATCH_BYTES)
    return fail(GMM_ERR_TOO_LARGE, "gmm_sm100_forward_f32_noalloc needs " + std::to_string(need) +
                                       " bytes of scratch; its fixed scratch holds " +
                                       std::to_string(GMM_SM100_NOALLOC_SCRATCH_BYTES) +
                                       " bytes (use gmm_sm100_forward with a workspace)");
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DeviceInfo* di = nullptr;
  if ((rc = device_info(dev, &di)) != GMM_OK) return rc;
  if (K == 0) {
    ce = cudaMemsetAsync(D, 0, static_cast<size_t>(T) * N * 4, stream);
    return ce == cudaSuccess ? GMM_OK : cuda_fail(ce, "cudaMemsetAsync");
  }
  if (!A || !B) return fail(GMM_ERR_INVALID_ARGUMENT, "A or B is null");
  if (!aligned16(A) || !aligned16(B)) return fail(GMM_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
  if ((K * 4) % 16 != 0)
    return fail(GMM_ERR_ALIGNMENT, "dim must be a multiple of 4 for fp32, got " + std::to_string(K));

  GmmParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.d = D;
  prm.ldd = N;
  prm.num_groups = pl.num_groups;
  prm.n_tiles = pl.n_tiles;
  prm.k_blocks = pl.k_blocks;
  prm.total_tiles = pl.total_tiles;
  prm.dim_out = static_cast<int>(N);
  prm.tile_rows = 128;
  if (pl.table_bytes == 0) {
    std::memcpy(prm.inline_table, pl.table.data(), pl.table.size() * sizeof(int32_t));
    prm.inline_ints = static_cast<int>(pl.table.size());
  } else {
    // The table is written in full (stream-ordered) before the kernel reads it.
    void* scratch = nullptr;
    if ((rc = noalloc_scratch_address(dev, &scratch)) != GMM_OK) return rc;
    ce = cudaMemcpyAsync(scratch, pl.table.data(), pl.table.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                         stream);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaMemcpyAsync(table)");
    prm.ext_table = static_cast<const int32_t*>(scratch);
  }
  return setup_and_launch(prm, A, B, T, K, N, E, GMM_DTYPE_F32, trans_b, 128, 0, pl.total_tiles, di, stream);
}
