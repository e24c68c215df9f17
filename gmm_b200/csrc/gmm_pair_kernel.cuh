// gmm_pair_kernel.cuh -- the CTA-pair (cta_group::2) variant of the persistent
// grouped-GEMM kernel, for groups with many rows (prefill-sized experts).
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x 256 output tile:
//   * CTA r (r = 0 leader, 1 peer) TMA-loads A rows [row0 + 128 r, +128) and
//     the B column half [n0 + 128 r, +128) into its own shared memory, in a
//     6-stage ring of 32 KB per CTA (16 KB A + 16 KB B, 128-byte swizzle);
//     both CTAs' loads complete on the leader's stage barrier, for which the
//     leader alone posts the expected byte count.  No load is multicast.
//   * one thread of the leader issues tcgen05.mma.cta_group::2 M=256 N=256
//     K=16, reading both CTAs' shared memory; each CTA's TMEM receives its own
//     128 rows x 256 columns (fp32), double-buffered (512 columns).
//   * the leader's tcgen05.commit (multicast to both CTAs) frees a stage in
//     both rings and tells both epilogues that an accumulator is ready; the
//     four epilogue warps of each CTA drain their rows and arrive on the
//     leader's accumulator-empty barrier (count 8) through the cluster window.
// Per CTA this moves 32 KB of operands per 64-deep k-block for the same MMA
// work the single-CTA 128x256 tile needs 48 KB for.
//
// Half tiles: the last m-tile of an expert whose remaining rows fit in 128
// runs as a 128 x 256 pair MMA (M = 128, cta_group::2): each CTA loads 64 A
// rows (a 64-row TMA box, tmap_a2) and its usual 128 B columns, and half the
// tensor work of a 256-row tile is spent on padding rows no more.  The
// accumulator of such an MMA sits in TMEM as the "2x2" data-path layout: in
// each CTA, row m (0..63) of output columns [0, 128) is TMEM lane m and of
// columns [128, 256) lane 64 + m, both at accumulator columns [0, 128) -- so
// epilogue warp q drains rows 32 (q & 1) .. +31 of column half q >> 1.  The
// SwiGLU epilogue pairs gate and up columns inside one thread's row, which
// this layout splits across lanes, so SwiGLU launches keep 256-row tiles.
#pragma once

template <int kKind, bool kBMnMajor>
struct PairCfg {
  static_assert(kKind == kKindBf16 || kKind == kKindF16, "pair tiles are 16-bit only");
  static constexpr int kElem = 2;
  static constexpr int BM = 256;      // rows per pair tile
  static constexpr int BM_CTA = 128;  // rows per CTA
  static constexpr int BN = 256;      // output columns per tile
  static constexpr int BN_CTA = 128;  // B columns held by each CTA
  static constexpr int BK = 64;
  static constexpr int kStages = 6;
  static constexpr int kUmmaK = 16;
  static constexpr int kKSteps = BK / kUmmaK;
  static constexpr int kABytes = BM_CTA * BK * kElem;  // 16 KB
  static constexpr int kBBytes = BN_CTA * BK * kElem;  // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr uint32_t kIdesc = make_idesc(kKind == kKindBf16 ? 1u : 0u, kBMnMajor, BM, BN);
  static constexpr uint32_t kIdescHalf = make_idesc(kKind == kKindBf16 ? 1u : 0u, kBMnMajor, BM / 2, BN);
  static constexpr int kHalfABytes = kABytes / 2;  // 64 A rows per CTA in a half tile
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + kEpiStageBytes + kDevTableBytes + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Spin for `ns` nanoseconds (abort path only: lets in-flight copies land).
__device__ __forceinline__ void spin_ns(unsigned long long ns) {
  const unsigned long long t0 = global_timer_ns();
  while (global_timer_ns() - t0 < ns) {
  }
}

template <int kKind, bool kBMnMajor>
__global__ void __launch_bounds__(kThreads, 1) gmm_pair_kernel(const __grid_constant__ GmmParams p) {
  using C = PairCfg<kKind, kBMnMajor>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_cta_rank();  // 0 = leader, 1 = peer
  const bool leader = (cta == 0);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full_bar = bars;                           // both CTAs' TMA -> leader MMA (leader's)
  uint64_t* empty_bar = bars + C::kStages;             // leader MMA -> each producer
  uint64_t* tfull_bar = bars + 2 * C::kStages;         // leader MMA -> each epilogue
  uint64_t* tempty_bar = bars + 2 * C::kStages + 2;    // 8 epilogue warps -> leader MMA
  uint64_t* drain_bar = bars + 2 * C::kStages + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* epi_stage = smem + C::kStages * C::kStageBytes + C::kBarBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(full_bar + s), 1);
      mbar_init(smem_u32(empty_bar + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(tfull_bar + a), 1);
      mbar_init(smem_u32(tempty_bar + a), 8);
    }
    mbar_init(smem_u32(drain_bar), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    prefetch_tmap(&p.tmap_a2);
    prefetch_tmap(&p.tmap_b);
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish_pair();
  }
  // Barriers initialised and TMEM allocated in both CTAs before any remote use.
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = p.n_tiles;
  const int k_blocks = p.k_blocks;
  const unsigned long long wait_ns = p.wait_ns ? p.wait_ns : kWaitTimeoutNs;
  const bool halves = !p.act;  // half tiles for expert tails of <= 128 rows
  int num_groups = p.num_groups, total_tiles = p.total_tiles;
  const int32_t* tab = p.ext_table ? p.ext_table : p.inline_table;
  if (p.dev_bs) {  // both CTAs of a pair build the same table
    int32_t* dtab = reinterpret_cast<int32_t*>(epi_stage + kEpiStageBytes);
    int32_t* meta = dtab + 3 * kMaxDevExperts + 2;
    build_device_table(p, dtab, meta, reinterpret_cast<long long*>(meta + 4));
    num_groups = meta[0];
    total_tiles = meta[1] * n_tiles;
    if (threadIdx.x == 0 && leader && meta[2] != 0) atomicCAS(&g_device_error, 0, meta[2]);
    tab = dtab;
  }
  const TableView tv = make_table_view(p, tab, num_groups);
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  bool aborted_here = false;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int g = 0;
      for (int tile = pair; ok && tile < total_tiles; tile += num_pairs) {
        const Tile t = decode_tile<C::BM, C::BN>(tv, n_tiles, tile, g);
        const bool half = halves && t.rows <= C::BM_CTA;
        const int arow = t.row0 + (half ? C::BM_CTA / 2 : C::BM_CTA) * static_cast<int>(cta);
        // SwiGLU: the leader holds the tile's 128 gate columns, the peer the matching up columns.
        const int bcol = !p.act ? t.n0 + C::BN_CTA * static_cast<int>(cta)
                                : (t.n0 >> 1) + (cta ? p.act_cols : 0);
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
          const uint32_t fb_local = smem_u32(full_bar + stage);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * (half ? C::kHalfABytes + C::kBBytes : C::kStageBytes));
          const uint32_t fb = map_shared_to_rank(fb_local, 0);
          uint8_t* sa = smem + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          const int k0 = kb * C::BK;
          tma_load_2d_pair(smem_u32(sa), half ? &p.tmap_a2 : &p.tmap_a, fb, k0, arow);
          if (kBMnMajor) {
#pragma unroll
            for (int c = 0; c < C::BN_CTA / 64; ++c)
              tma_load_3d_pair(smem_u32(sb + c * (C::BK * 128)), &p.tmap_b, fb, bcol + 64 * c, k0,
                               t.expert);
          } else {
            tma_load_3d_pair(smem_u32(sb), &p.tmap_b, fb, k0, bcol, t.expert);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) aborted_here = true;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      int g = 0;
      for (int tile = pair; ok && tile < total_tiles; tile += num_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const Tile t = decode_tile<C::BM, C::BN>(tv, n_tiles, tile, g);
        const uint32_t idesc = (halves && t.rows <= C::BM_CTA) ? C::kIdescHalf : C::kIdesc;
        if (!mbar_wait(smem_u32(tempty_bar + acc), acc_phase ^ 1, abort_flag, wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(full_bar + stage), phase, abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
#pragma unroll
          for (int ks = 0; ks < C::kKSteps; ++ks) {
            const uint64_t adesc = make_sw128_desc(sa + ks * 32, 16, 1024);
            const uint64_t bdesc = kBMnMajor
                                       ? make_sw128_desc(sb + ks * C::kUmmaK * 128, C::BK * 128, 1024)
                                       : make_sw128_desc(sb + ks * 32, 16, 1024);
            mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          mma_commit_pair_mc(smem_u32(empty_bar + stage), 0x3);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair_mc(smem_u32(tfull_bar + acc), 0x3);
      }
      mma_commit_pair(smem_u32(drain_bar));
      mbar_wait_drain(smem_u32(drain_bar), 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    using OutT = typename std::conditional<kKind == kKindBf16, __nv_bfloat16, __half>::type;
    const int quarter = warp & 3;
    const uint32_t stage = smem_u32(epi_stage) + quarter * (32 * 128);
    const uint32_t tempty_leader0 = map_shared_to_rank(smem_u32(tempty_bar), 0);
    int g = 0;
    int local = 0;
    for (int tile = pair; tile < total_tiles; tile += num_pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(tfull_bar + acc), acc_phase, abort_flag, wait_ns)) break;
      tc_fence_after();
      const Tile t = decode_tile<C::BM, C::BN>(tv, n_tiles, tile, g);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::BN;
      if (halves && t.rows <= C::BM_CTA) {
        // half tile: this CTA holds rows [64 cta, 64 cta + 64) of the tile;
        // warp q drains rows 32 (q & 1) .. +31 of output columns 128 (q >> 1) .. +127
        const int rows_cta = t.rows - (C::BM_CTA / 2) * static_cast<int>(cta);
        const int rb = (quarter & 1) * 32;
        if (rb < rows_cta)  // warp-uniform
          drain_slab<OutT, C::BN / 2>(p, tv, g, t.row0 + (C::BM_CTA / 2) * static_cast<int>(cta) + rb,
                                      min(32, rows_cta - rb), t.n0 + (quarter >> 1) * (C::BN / 2), taddr,
                                      stage, lane);
      } else {
        const int rows_cta = t.rows - C::BM_CTA * static_cast<int>(cta);
        const int row0 = t.row0 + C::BM_CTA * static_cast<int>(cta);
        if (quarter * 32 < rows_cta) {  // warp-uniform
          if (p.act)
            drain_slab_swiglu<OutT>(p, tv, g, row0 + quarter * 32, min(32, rows_cta - quarter * 32),
                                    t.n0 >> 1, taddr, stage, lane);
          else
            drain_slab<OutT, C::BN>(p, tv, g, row0 + quarter * 32, min(32, rows_cta - quarter * 32), t.n0,
                                    taddr, stage, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
    }
    if (p.remote) __threadfence_system();  // peer stores performed before the kernel ends
  }

  // --------------------------------------------------------------- teardown
  if (aborted_here || *abort_flag) spin_ns(2000000);  // in-flight copies land before exit
  tc_fence_before();
  __syncwarp();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its shared memory
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(&g_device_error, 0, GMM_ERR_DEVICE_TIMEOUT);
  __syncwarp();
  cluster_sync_all();
}
