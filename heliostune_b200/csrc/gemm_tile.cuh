// tcgen05 tile GEMM, C[M,N] = A[M,K] * B[K,N] in FP16 with an FP32 TMEM accumulator.
//
// One kernel serves the reference's "tile" family (kernel.py:21-118, one CTA per output tile)
// and its "persistent" family (hopper_kernel.py:148-290, a grid of one CTA per SM striding over
// the tiles); the launcher picks the grid. Both walk tiles in the reference's grouped raster
// (group_m tile rows per group).
//
// CTA of 192 threads, warp-specialised:
//   warp 0      TMA producer: A tiles [UM rows x 64 k] (K-major) and B tiles [BK k x 64 n]
//               (N-major) into a ring of shared-memory stages, 128-byte swizzled.
//   warp 1      TMEM owner and UMMA issuer: tcgen05.mma (M = UM, N = BN, K = 16) into one of two
//               TMEM accumulators, tcgen05.commit frees each stage and publishes each tile.
//   warps 2..5  epilogue: tcgen05.ld of their 32-lane TMEM quarter, FP32 -> FP16, swizzled
//               staging in shared memory, TMA store of 64-column sub-tiles (edges clipped).
// Two accumulators let the epilogue of one tile overlap the main loop of the next.
#pragma once

#include "ptx.cuh"

namespace hst {

constexpr int kTileThreads = 192;
constexpr int kMaxStages = 12;
constexpr int kEpilogueStageBytes = 4096;  // 32 rows x 128 bytes

struct TileArgs {
  int m, n, k;
  int tiles_m, tiles_n, num_tiles;
  int k_blocks;
  int group_m;
  int stages;
  int* status;
};

template <int UM, int MA, int BN, int BK>
struct TileShape {
  static_assert(UM == 64 || UM == 128, "UMMA M must be 64 or 128");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64, 128 or 256");
  static_assert(BK % 64 == 0 && BK <= 128, "BK must be 64 or 128");
  static constexpr int kAtomsK = BK / 64;           // 128-byte swizzle atoms of A along K
  static constexpr int kAtomsN = BN / 64;           // 128-byte swizzle atoms of B along N
  static constexpr int kABoxBytes = UM * 128;       // one TMA box of A: UM rows x 64 k
  static constexpr int kBBoxBytes = BK * 128;       // one TMA box of B: BK rows x 64 n
  static constexpr int kABytes = MA * kAtomsK * kABoxBytes;
  static constexpr int kBBytes = kAtomsN * kBBoxBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccCols = MA * BN;          // TMEM columns of one accumulator
  static constexpr int kAccBufs = (2 * kAccCols <= 512) ? 2 : 1;
  static constexpr int kTmemCols = (kAccBufs * kAccCols <= 32)    ? 32
                                   : (kAccBufs * kAccCols <= 64)  ? 64
                                   : (kAccBufs * kAccCols <= 128) ? 128
                                   : (kAccBufs * kAccCols <= 256) ? 256
                                                                  : 512;
  static constexpr int kEpilogueBytes = 4 * 2 * kEpilogueStageBytes;
  static constexpr int kBarrierBytes = 256 + 16 * kMaxStages;
  static constexpr uint32_t kIdesc = umma_idesc_f16(UM, BN, false, true);
  // Rows of one epilogue warp's quarter of a UMMA atom.
  static constexpr int kRowsPerWarp = UM / 4;

  static constexpr int smem_bytes(int stages) {
    return 1024 /* alignment slack */ + stages * kStageBytes + kEpilogueBytes + kBarrierBytes;
  }
};

template <int UM, int MA, int BN, int BK>
__global__ void __launch_bounds__(kTileThreads, 1)
    tile_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const TileArgs args) {
  using S = TileShape<UM, MA, BN, BK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = args.stages;
  uint8_t* ring = smem;
  uint8_t* epi = ring + stages * S::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi + S::kEpilogueBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* tmem_full = bars + 2 * kMaxStages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_done = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_c);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t policy = l2_policy_evict_normal();
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x) {
      int pm, pn;
      grouped_tile(tile, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
      const int m0 = pm * UM * MA;
      const int n0 = pn * BN;
      for (int kb = 0; kb < args.k_blocks; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          raise_abort(args.status, abort_flag, kStatusProducerTimeout);
          ok = false;
          break;
        }
        uint8_t* st = ring + stage * S::kStageBytes;
        mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
        const int k0 = kb * BK;
#pragma unroll
        for (int ma = 0; ma < MA; ++ma) {
#pragma unroll
          for (int ka = 0; ka < S::kAtomsK; ++ka) {
            tma_load_2d(st + (ma * S::kAtomsK + ka) * S::kABoxBytes, &map_a, &full[stage],
                        k0 + 64 * ka, m0 + ma * UM, policy);
          }
        }
#pragma unroll
        for (int na = 0; na < S::kAtomsN; ++na) {
          tma_load_2d(st + S::kABytes + na * S::kBBoxBytes, &map_b, &full[stage], n0 + 64 * na,
                      k0, policy);
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      // Let every copy this thread started land before the CTA's shared memory is released.
      for (int s = 0; s < stages; ++s) {
        if (issued_mask & (1u << s)) {
          if (!mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, 200000000ull)) {
            atomicOr(args.status, kStatusDrainTimeout);
          }
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- UMMA issuer ----------------
    // Stage 0's operand descriptors at K step 0; any other operand adds its byte offset / 16 to
    // the start-address field (bits 0-13; shared memory stays below 256 KB).
    const uint64_t a_desc0 = smem_desc(smem_addr(ring), 16, 1024);
    const uint64_t b_desc0 = smem_desc(smem_addr(ring) + S::kABytes, S::kBBoxBytes, 1024);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x) {
      if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusMmaTimeout);
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t d_base = tmem_base + acc * S::kAccCols;
      for (int kb = 0; kb < args.k_blocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          raise_abort(args.status, abort_flag, kStatusMmaTimeout);
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint64_t stage_off = static_cast<uint64_t>(stage * (S::kStageBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const int ka = kk >> 2;
          const int kin = kk & 3;
          const uint64_t bdesc = b_desc0 + stage_off + ((kk * 2048) >> 4);
#pragma unroll
          for (int ma = 0; ma < MA; ++ma) {
            const uint64_t adesc =
                a_desc0 + stage_off + (((ma * S::kAtomsK + ka) * S::kABoxBytes + kin * 32) >> 4);
            umma_f16(d_base + ma * BN, adesc, bdesc, S::kIdesc, (kb | kk) != 0);
          }
        }
        umma_commit(&empty[stage]);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      umma_commit(&tmem_full[acc]);
      if (++acc == S::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Every UMMA this thread issued must retire before TMEM is released.
    umma_commit(mma_done);
    if (!mbar_wait(mma_done, 0, nullptr, 200000000ull)) {
      atomicOr(args.status, kStatusDrainTimeout);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    uint8_t* staging = epi + (warp - 2) * 2 * kEpilogueStageBytes;
    int buf = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
      int pm, pn;
      grouped_tile(tile, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
      const int m0 = pm * UM * MA;
      const int n0 = pn * BN;
      // The warp leaves together: tcgen05.ld below needs all 32 lanes.
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&tmem_full[acc], acc_phase, abort_flag));
      if (!ready) {
        if (lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
        break;
      }
      tc_fence_after_sync();
#pragma unroll 1
      for (int ma = 0; ma < MA; ++ma) {
        const int row0 = m0 + ma * UM + quarter * S::kRowsPerWarp;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 acc * S::kAccCols + ma * BN + c * 64;
          uint32_t lo[32], hi[32];
          tmem_ld_32x32b_x32(taddr, lo);
          tmem_ld_32x32b_x32(taddr + 32, hi);
          tmem_ld_wait();
          uint8_t* dst = staging + buf * kEpilogueStageBytes;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          if (static_cast<int>(lane) < S::kRowsPerWarp) {
            const uint32_t row_addr = smem_addr(dst) + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t* src = (j < 4) ? &lo[j * 8] : &hi[(j - 4) * 8];
              const uint32_t w0 = pack_half2(__uint_as_float(src[0]), __uint_as_float(src[1]));
              const uint32_t w1 = pack_half2(__uint_as_float(src[2]), __uint_as_float(src[3]));
              const uint32_t w2 = pack_half2(__uint_as_float(src[4]), __uint_as_float(src[5]));
              const uint32_t w3 = pack_half2(__uint_as_float(src[6]), __uint_as_float(src[7]));
              st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), w0, w1, w2, w3);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_c, dst, n0 + c * 64, row0);
            bulk_commit_group();
          }
          buf ^= 1;
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&tmem_empty[acc]);
      if (++acc == S::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace hst
