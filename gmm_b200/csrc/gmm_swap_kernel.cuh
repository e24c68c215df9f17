// gmm_swap_kernel.cuh -- swap-AB grouped-GEMM tiles for small and ragged
// experts: decode-shaped routing (reference configuration E=128 with 1..16
// rows each) and fine-grained expert loads where most experts own fewer rows
// than a 128-row tile (E=256, Zipf-skewed).
//
// The MMA's M dimension runs over output COLUMNS -- rows of B^T -- and its N
// dimension over the expert's token rows:
//     D[rows, c0:c0+128]^T = B[e][:, c0:c0+128]^T (128 x K)  @  A[rows]^T (K x n)
// A tile is 256 output columns (two such MMAs sharing the rows operand) by
// one row block of an expert.  The expert's rows are cut into ceil(m / 128)
// balanced blocks whose height is rounded up to 16 and becomes the MMA's N
// (16..128), so an 8-row expert costs 128x16 products per K step instead of
// 128x128, and a 200-row expert two 112-row blocks instead of 256 rows.
//
//   * B^T operand (MMA A): NT B ([E, N, K], K contiguous) is read K-major,
//     one [256 rows][64] box per k-block; NN B ([E, K, N], N contiguous) is
//     read MN-major as four [64 k][64 cols] panels (descriptor LBO = panel
//     stride) -- the same boxes as the 128-row kernel's B tile, neither layout
//     transposed in memory.
//   * A rows operand (MMA B): one K-major [128 rows][64] box from the block's
//     first row (rows past the block are loaded but not multiplied: the
//     MMA's N covers the block only).  One box issues fewer TMA requests than
//     16-row pieces, which measured faster on the fine-grained loads.
//   * Accumulators: two TMEM buffers of 2 x 128 columns (fp32, 128 lanes).
//     Lane l of half h is output column c0 + 128 h + l; column j is row j.
//   * Epilogue: warp q (of 4) owns lanes [32q, 32q + 32): each thread holds one
//     output column; 16 rows at a time pass through shared memory
//     ([16 rows][32 columns] per warp) and leave as 16-byte row pieces.
//
// Same warp roles, bounded waits and teardown as the main kernel; supports
// the host tile table and the device-built table (device batch sizes).
// 16-bit operands, local output only (no SwiGLU or expert-parallel epilogue).
#pragma once

template <int kKind, bool kBMnMajor>
struct SwapCfg {
  static_assert(kKind == kKindBf16 || kKind == kKindF16, "swap-AB tiles are 16-bit");
  static constexpr int BM = 128;          // output columns per MMA (MMA M)
  static constexpr int kCols = 256;       // output columns per tile: two MMAs share the rows operand
  static constexpr int kHalves = kCols / BM;
  static constexpr int kMaxRows = 128;    // token rows per tile (MMA N: 16..128, multiple of 16)
  static constexpr int BK = 64;           // one 128-byte swizzle row of K
  static constexpr int kStages = 4;
  static constexpr int kAccs = 2;
  static constexpr int kBtBytes = kCols * BK * 2;     // 32 KB
  static constexpr int kRowBytes = kMaxRows * BK * 2;  // 16 KB: one [128 rows][64] box of A
  static constexpr int kStageBytes = kBtBytes + kRowBytes;  // 48 KB
  static constexpr int kAccCols = kHalves * kMaxRows;  // 256 TMEM columns per tile
  static constexpr int kTmemCols = kAccs * kAccCols;   // 512
  static constexpr int kBarBytes = 256;
  static constexpr int kEpiBytes = 4 * 16 * 32 * 2;  // per epilogue warp: 16 rows x 32 columns
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + kDevTableBytes + kEpiBytes + 1024;
  __device__ static constexpr uint32_t idesc(int n) {
    return make_idesc(kKind == kKindBf16 ? 1u : 0u, false, BM, n) | (kBMnMajor ? (1u << 15) : 0u);
  }
  static_assert(2 * kStages + 2 * kAccs + 1 <= kBarBytes / 8 - 1, "barrier area");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Tile decode for swap-AB tiles.  The table counts ceil(m / 128) row blocks per
// expert (the same m-tiles as the 128-row kernel); the blocks of an expert
// are balanced -- height ceil(m / blocks) rounded up to 16 -- so an expert of
// m rows costs at most 15 padded rows per block instead of up to 127.  Every
// block is non-empty: with b = ceil(m / 128) blocks of height h <= 128,
// (b - 1) * h < m.
template <int BN>
__device__ __forceinline__ Tile decode_swap_tile(const TableView& t, int n_tiles, int tile, int& g) {
  while (tile >= t.tile_off[g + 1] * n_tiles) ++g;
  const int mt = t.tile_off[g + 1] - t.tile_off[g];
  const int local = tile - t.tile_off[g] * n_tiles;
  const int blk = local / (kMBlock * n_tiles);
  const int r = local - blk * kMBlock * n_tiles;
  const int hgt = min(kMBlock, mt - blk * kMBlock);
  const int m = blk * kMBlock + r % hgt;
  const int n = r / hgt;
  const int rows_g = t.row_off[g + 1] - t.row_off[g];
  const int bh = ((rows_g + mt - 1) / mt + 15) & ~15;
  Tile out;
  out.row0 = t.row_off[g] + m * bh;
  out.rows = min(bh, t.row_off[g + 1] - out.row0);
  out.n0 = n * BN;
  out.expert = t.expert[g];
  return out;
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }

template <int kKind, bool kBMnMajor, typename P = GmmParams>
__global__ void __launch_bounds__(kThreads, 1) gmm_swap_kernel(const __grid_constant__ P p) {
  using C = SwapCfg<kKind, kBMnMajor>;
  constexpr int kCols = C::kCols;
  using OutT = typename std::conditional<kKind == kKindBf16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + C::kStages;
  uint64_t* tfull_bar = bars + 2 * C::kStages;
  uint64_t* tempty_bar = tfull_bar + C::kAccs;
  uint64_t* drain_bar = tempty_bar + C::kAccs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* dev_area = smem + C::kStages * C::kStageBytes + C::kBarBytes;
  uint8_t* epi_area = dev_area + kDevTableBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(full_bar + s), 1);
      mbar_init(smem_u32(empty_bar + s), 1);
    }
    for (int a = 0; a < C::kAccs; ++a) {
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

  const int n_tiles = p.n_tiles, k_blocks = p.k_blocks;
  int num_groups = p.num_groups, total_tiles = p.total_tiles;
  const int32_t* tab = p.ext_table ? p.ext_table : p.inline_table;
  if (p.dev_bs) {
    int32_t* dtab = reinterpret_cast<int32_t*>(dev_area);
    int32_t* meta = dtab + 3 * kMaxDevExperts + 2;
    build_device_table(p, dtab, meta, reinterpret_cast<long long*>(meta + 4));
    num_groups = meta[0];
    total_tiles = meta[1] * n_tiles;
    if (threadIdx.x == 0 && meta[2] != 0) atomicCAS(&g_device_error, 0, meta[2]);
    tab = dtab;
  }
  const TableView tv = make_table_view(p, tab, num_groups);

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
        const Tile t = decode_swap_tile<kCols>(tv, n_tiles, tile, g);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(empty_bar + stage), phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full_bar + stage);
          mbar_arrive_expect_tx(fb, C::kStageBytes);
          uint8_t* sbt = smem + stage * C::kStageBytes;
          uint8_t* srow = sbt + C::kBtBytes;
          const int k0 = kb * C::BK;
          if (kBMnMajor) {  // kCols / 64 panels of [64 k][64 cols]
#pragma unroll
            for (int c = 0; c < kCols / 64; ++c)
              tma_load_3d(smem_u32(sbt + c * (C::BK * 128)), &p.tmap_b, fb, t.n0 + 64 * c, k0, t.expert);
          } else {  // one [kCols rows][64] box
            tma_load_3d(smem_u32(sbt), &p.tmap_b, fb, k0, t.n0, t.expert);
          }
          // one box from the block's first row; the MMA reads its first n rows
          tma_load_2d(smem_u32(srow), &p.tmap_a, fb, k0, t.row0);
          issued[stage]++;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
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
      int local = 0, g = 0;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++local) {
        const int acc = local % C::kAccs;
        const uint32_t acc_phase = (local / C::kAccs) & 1;
        if (!mbar_wait(smem_u32(tempty_bar + acc), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const Tile t = decode_swap_tile<kCols>(tv, n_tiles, tile, g);
        const uint32_t idesc = C::idesc(max(1, (t.rows + 15) >> 4) * 16);
        const uint32_t d_tmem = tmem_base + acc * C::kAccCols;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(full_bar + stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sbt = smem_u32(smem + stage * C::kStageBytes);
          const uint32_t srow = sbt + C::kBtBytes;
#pragma unroll
          for (int ks = 0; ks < C::BK / 16; ++ks) {
            const uint64_t bdesc = make_sw128_desc(srow + ks * 32, 16, 1024);
#pragma unroll
            for (int h = 0; h < C::kHalves; ++h) {  // 128 output columns each: 16 KB of B^T
              const uint32_t sh = sbt + h * (C::BM * 128);
              const uint64_t adesc = kBMnMajor ? make_sw128_desc(sh + ks * 16 * 128, C::BK * 128, 1024)
                                               : make_sw128_desc(sh + ks * 32, 16, 1024);
              mma_f16_ss(d_tmem + h * C::kMaxRows, adesc, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
            }
          }
          mma_commit(smem_u32(empty_bar + stage));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(smem_u32(tfull_bar + acc));
      }
      mma_commit(smem_u32(drain_bar));
      mbar_wait_drain(smem_u32(drain_bar), 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    OutT* stg = reinterpret_cast<OutT*>(epi_area) + quarter * (16 * 32);
    int local = 0, g = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++local) {
      const int acc = local % C::kAccs;
      const uint32_t acc_phase = (local / C::kAccs) & 1;
      if (!mbar_wait(smem_u32(tfull_bar + acc), acc_phase, abort_flag)) break;
      tc_fence_after();
      const Tile t = decode_swap_tile<kCols>(tv, n_tiles, tile, g);
#pragma unroll 1
      for (int h = 0; h < C::kHalves; ++h) {
        const int col0 = t.n0 + h * C::BM + quarter * 32;  // this warp's first column
        if (col0 >= p.dim_out) break;                       // warp-uniform
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::kAccCols +
                               h * C::kMaxRows;
#pragma unroll 1
        for (int r0 = 0; r0 < t.rows; r0 += 16) {
          // 16 rows of this thread's column -> [16 rows][32 columns] in shared
          // memory -> 16-byte row pieces (four per 64-byte row of the warp).
          uint32_t v[16];
          tmem_ld_32x32b_x16(taddr + r0, v);
          tmem_wait_ld();
#pragma unroll
          for (int r = 0; r < 16; ++r) stg[r * 32 + lane] = to_out<OutT>(__uint_as_float(v[r]));
          __syncwarp();
          const int nr = min(16, t.rows - r0);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int c = lane + 32 * i;
            const int rr = c >> 2, part = c & 3;
            const uint4 val = *reinterpret_cast<const uint4*>(stg + rr * 32 + part * 8);
            if (rr < nr && col0 + part * 8 < p.dim_out) {
              OutT* rp = reinterpret_cast<OutT*>(p.d) + static_cast<long long>(t.row0 + r0 + rr) * p.ldd;
              *reinterpret_cast<uint4*>(rp + col0 + part * 8) = val;
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(tempty_bar + acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(&g_device_error, 0, GMM_ERR_DEVICE_TIMEOUT);
}
