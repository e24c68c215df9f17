// gmm_vark_kernel.cuh -- variable-K grouped GEMM for the MoE backward pass:
// for every expert e with rows [off_e, off_e + m_e) of A [T, M] and B [T, N],
//     D[e] = A[rows_e]^T @ B[rows_e]          ([M, N], fp32 accumulation)
// (the weight gradient dW_e = x_e^T dy_e).  This is the kernel family the
// reference removed from its forward-only extract (reference
// csrc/hopper_gmm_forward.cu:16-21, `CutlassGroupedGemmVariableK`).
//
// Same warp roles and TMEM double buffering as the forward kernel.  Output
// tiles are 128 (rows of D[e], i.e. columns of A) x 256 (columns of B); the
// contraction runs over the expert's rows in 64-row blocks.  Both operands
// are read MN-major straight from A and B (64-column panels of [64 rows][64]),
// so no transpose is ever materialised.  The last block of an expert may pull
// in rows of the next expert: the MMA warp zeroes those rows in shared memory
// (then fences the async proxy) before the tensor cores read them.  An expert
// with no rows gets a zero D[e].
#pragma once

template <int kKind>
struct VarKCfg {
  static_assert(kKind == kKindBf16 || kKind == kKindF16, "variable-K tiles are 16-bit");
  static constexpr int BM = 128, BN = 256, BK = 64, kStages = 4;
  static constexpr int kPanelBytes = BK * 128;             // [64 rows][64 elements] = 8 KB
  static constexpr int kABytes = (BM / 64) * kPanelBytes;  // 16 KB
  static constexpr int kBBytes = (BN / 64) * kPanelBytes;  // 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = 256;
  // A and B both MN-major (bit 15 = A major, bit 16 = B major).
  static constexpr uint32_t kIdesc =
      make_idesc(kKind == kKindBf16 ? 1u : 0u, true, BM, BN) | (1u << 15);
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + kEpiStageBytes + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int kKind>
__global__ void __launch_bounds__(kThreads, 1) gmm_vark_kernel(const __grid_constant__ GmmParams p) {
  using C = VarKCfg<kKind>;
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
  uint64_t* tempty_bar = bars + 2 * C::kStages + 2;
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

  const int32_t* row_off = p.inline_table;  // [E + 1]
  const int m_tiles = p.vk_m_tiles, n_tiles = p.n_tiles;
  const int per_expert = m_tiles * n_tiles;
  const int M = p.vk_m, N = p.dim_out;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x) {
        const int e = tile / per_expert, r = tile - e * per_expert;
        const int m0 = (r % m_tiles) * C::BM, n0 = (r / m_tiles) * C::BN;
        const int off = row_off[e], kbs = (row_off[e + 1] - off + C::BK - 1) / C::BK;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!mbar_wait(smem_u32(empty_bar + stage), phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full_bar + stage);
          mbar_arrive_expect_tx(fb, C::kStageBytes);
          uint8_t* sa = smem + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          const int k0 = off + kb * C::BK;
#pragma unroll
          for (int c = 0; c < C::BM / 64; ++c)
            tma_load_2d(smem_u32(sa + c * C::kPanelBytes), &p.tmap_a, fb, m0 + 64 * c, k0);
#pragma unroll
          for (int c = 0; c < C::BN / 64; ++c)
            tma_load_2d(smem_u32(sb + c * C::kPanelBytes), &p.tmap_b, fb, n0 + 64 * c, k0);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp)
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int local = 0;
    for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x, ++local) {
      const int e = tile / per_expert;
      const int off = row_off[e], me = row_off[e + 1] - off;
      const int kbs = (me + C::BK - 1) / C::BK;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // every lane waits (the zeroing below needs the landed data); all break together
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(tempty_bar + acc), acc_phase ^ 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * C::BN;
      for (int kb = 0; kb < kbs; ++kb) {
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(full_bar + stage), phase, abort_flag))) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
        const int valid = me - kb * C::BK;
        if (valid < C::BK) {
          // rows [valid, 64) of every panel belong to the next expert: zero them
          const int chunks = (C::BK - valid) * 8;  // 16-byte chunks per panel
          constexpr int kPanels = (C::BM + C::BN) / 64;
          for (int i = lane; i < kPanels * chunks; i += 32) {
            const int panel = i / chunks, c = i - panel * chunks;
            st_shared_v4(sa + panel * C::kPanelBytes + valid * 128 + c * 16, make_uint4(0, 0, 0, 0));
          }
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) {
          tc_fence_after();
          const uint32_t sb = sa + C::kABytes;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t adesc = make_sw128_desc(sa + ks * 16 * 128, C::kPanelBytes, 1024);
            const uint64_t bdesc = make_sw128_desc(sb + ks * 16 * 128, C::kPanelBytes, 1024);
            mma_f16_ss(d_tmem, adesc, bdesc, C::kIdesc, (kb | ks) != 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(empty_bar + stage));
        }
        __syncwarp();
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) mma_commit(smem_u32(tfull_bar + acc));  // also for an empty expert
      __syncwarp();
    }
    if (lane == 0) {
      mma_commit(smem_u32(drain_bar));
      mbar_wait_drain(smem_u32(drain_bar), 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const uint32_t stage = smem_u32(epi_stage) + quarter * (32 * 128);
    int local = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(tfull_bar + acc), acc_phase, abort_flag)) break;
      tc_fence_after();
      const int e = tile / per_expert, r = tile - e * per_expert;
      const int m0 = (r % m_tiles) * C::BM, n0 = (r / m_tiles) * C::BN;
      const bool empty = row_off[e + 1] == row_off[e];
      const int slab0 = m0 + quarter * 32;
      if (slab0 < M) {  // warp-uniform
        OutT* rp[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = slab0 + i * 4 + (lane >> 3);
          rp[i] = m < M ? reinterpret_cast<OutT*>(p.d) + (static_cast<long long>(e) * M + m) * p.ldd
                        : nullptr;
        }
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::BN;
        drain_rows<OutT, C::BN>(rp, n0, N, taddr, stage, lane, empty);
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
