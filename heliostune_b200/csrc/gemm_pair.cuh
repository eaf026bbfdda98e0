// CTA-pair tcgen05 GEMM: C[M,N] = A[M,K] * B[K,N], 256 x BN output tiles per pair of SMs.
//
// B200 "pair" family (no reference counterpart; the reference's largest tiles are the
// 128x256 / 256x128 frozen candidates of action_configs.py:91-96). A cluster of two CTAs on the
// two SMs of a TPC computes one 256 x BN tile with tcgen05.mma.cta_group::2 (UMMA M = 256):
//   * CTA r loads its own 128 rows of A and its own BN/2 columns of B for every K block, so
//     each SM pulls half the B bytes a single-SM 128 x BN tile would;
//   * both CTAs' TMA loads complete on the leader CTA's (rank 0) stage barrier;
//   * one thread of the leader issues the UMMAs; they read A and B from both CTAs' shared
//     memory and accumulate rows 128r..128r+127 in CTA r's TMEM;
//   * the leader's tcgen05.commit releases each stage in both CTAs (one commit per CTA) and
//     publishes each finished accumulator to both CTAs' epilogues;
//   * each CTA drains its own 128 rows x BN columns exactly like the single-SM kernel, and its
//     epilogue warps report a free accumulator on the leader's barrier.
// The kernel is persistent: cluster p walks tiles p, p + #pairs, ... in the grouped raster, with
// two TMEM accumulators so a tile's epilogue overlaps the next tile's main loop.
//
// SPLIT = true (split-K for tile counts far below the SM count): the cluster grows to (2, S):
// S pairs compute the same 256 x BN tile over S contiguous K ranges. CTA (r, s) owns columns
// [s*BN/S, (s+1)*BN/S) of its 128 rows. Once every CTA's main loop is done (cluster barrier, so
// all rings are drained), each CTA pushes every column slice of its FP32 partial from TMEM
// straight into the owning CTA's shared memory (remote stores, slot = source split, 16-byte
// chunks swizzled by row); after a second barrier each owner sums its S slots in split order
// from local shared memory and stores FP16 C. One tile per cluster; no workspace, no atomics,
// bitwise reproducible.
// No TMA load here feeds more than one CTA's shared memory.
#pragma once

#include "gemm_tile.cuh"
#include "ptx.cuh"

namespace hst {

template <int BN, int BK>
struct PairShape {
  static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
  static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
  static constexpr int kHalfN = BN / 2;
  static constexpr int kAtomsK = BK / 64;
  static constexpr int kAtomsN = kHalfN / 64;
  static constexpr int kABoxBytes = 128 * 128;  // 128 rows x 64 k
  static constexpr int kBBoxBytes = BK * 128;   // BK rows x 64 n
  static constexpr int kABytes = kAtomsK * kABoxBytes;
  static constexpr int kBBytes = kAtomsN * kBBoxBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;  // per CTA
  static constexpr int kAccCols = BN;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  static constexpr int kEpilogueBytes = 4 * 2 * kEpilogueStageBytes;
  static constexpr int kBarrierBytes = 256 + 16 * kMaxStages;
  static constexpr uint32_t kIdesc = umma_idesc_f16(256, BN, false, true);
  static constexpr int smem_bytes(int stages) {
    return 1024 + stages * kStageBytes + kEpilogueBytes + kBarrierBytes;
  }
};

// Column-parallel fan-out of the persistent pair kernel: every finished 64-column sub-tile of
// this rank's C slice is also written, with coalesced 16-byte stores, into the same columns of
// the other ranks' C (peer pointers over NVLink). The local copy goes through the TMA store.
constexpr int kMaxPeers = 8;
struct PairFanoutArgs {
  uint64_t peers[kMaxPeers];  // other ranks' C base + this rank's column offset (elements)
  int count;                  // number of peers (0 = no fan-out)
  int64_t ldc;                // row stride of every rank's full C, elements
};

struct PairSplitArgs {
  int splits;        // cluster extent along y (1 = persistent mode)
  int kb_per_split;  // K blocks of one split
  __half* c;         // C for the split-mode epilogue (row stride ldc)
  int64_t ldc;
};

template <int BN, int BK, bool SPLIT>
__global__ void __launch_bounds__(kTileThreads, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const TileArgs args,
                     const PairSplitArgs split_args, const __grid_constant__ PairFanoutArgs fanout) {
  using S = PairShape<BN, BK>;
  static_assert(!SPLIT || BN * 128 * 4 <= 6 * 32768, "the FP32 partial reuses the ring");
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
  const uint32_t crank = cluster_ctarank();
  const uint32_t rank = crank & 1u;           // row half of the pair tile
  const uint32_t leader = crank & ~1u;        // cluster rank of this pair's leader CTA
  const int pair = SPLIT ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(cluster_id_x());
  const int pairs = SPLIT ? args.num_tiles : static_cast<int>(nclusters_x());
  const int split = SPLIT ? static_cast<int>(blockIdx.y) : 0;
  const int kb_begin = SPLIT ? split * split_args.kb_per_split : 0;
  const int kb_end = SPLIT ? min(kb_begin + split_args.kb_per_split, args.k_blocks) : args.k_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);  // four epilogue warps in each CTA (leader's copy is used)
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  bool split_ready = false;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    const uint64_t policy = l2_policy_evict_normal();
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed_mask = 0, armed_parity = 0;
    bool ok = true;
    for (int tile = pair; tile < args.num_tiles && ok; tile += pairs) {
      int pm, pn;
      grouped_tile(tile, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
      const int m0 = pm * 256 + static_cast<int>(rank) * 128;
      const int n0 = pn * BN + static_cast<int>(rank) * S::kHalfN;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          raise_abort(args.status, abort_flag, kStatusProducerTimeout);
          ok = false;
          break;
        }
        uint8_t* st = ring + stage * S::kStageBytes;
        const uint32_t leader_full = map_to_rank(smem_addr(&full[stage]), leader);
        if (rank == 0) {
          mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
          armed_mask |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        }
        const int k0 = kb * BK;
#pragma unroll
        for (int ka = 0; ka < S::kAtomsK; ++ka) {
          tma_load_2d_pair(st + ka * S::kABoxBytes, &map_a, leader_full, k0 + 64 * ka, m0, policy);
        }
#pragma unroll
        for (int na = 0; na < S::kAtomsN; ++na) {
          tma_load_2d_pair(st + S::kABytes + na * S::kBBoxBytes, &map_b, leader_full,
                           n0 + 64 * na, k0, policy);
        }
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && rank == 0) {
      for (int s = 0; s < stages; ++s) {
        if ((armed_mask & (1u << s)) &&
            !mbar_wait(&full[s], (armed_parity >> s) & 1u, nullptr, 200000000ull)) {
          atomicOr(args.status, kStatusDrainTimeout);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- UMMA issuer (leader only) ----------------
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = pair; tile < args.num_tiles && ok; tile += pairs) {
      if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusMmaTimeout);
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t d_base = tmem_base + acc * S::kAccCols;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          raise_abort(args.status, abort_flag, kStatusMmaTimeout);
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t a_base = smem_addr(ring + stage * S::kStageBytes);
        const uint32_t b_base = a_base + S::kABytes;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t adesc =
              smem_desc(a_base + (kk >> 2) * S::kABoxBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bdesc = smem_desc(b_base + kk * 2048, S::kBBoxBytes, 1024);
          umma_f16_pair(d_base, adesc, bdesc, S::kIdesc, (kb != kb_begin || kk != 0) ? 1u : 0u);
        }
        const uint32_t own_empty = smem_addr(&empty[stage]);
        umma_commit_pair(own_empty);
        umma_commit_pair(map_to_rank(own_empty, crank | 1u));
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      const uint32_t own_full = smem_addr(&tmem_full[acc]);
      umma_commit_pair(own_full);
      umma_commit_pair(map_to_rank(own_full, crank | 1u));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    umma_commit_pair(smem_addr(mma_done));
    if (!mbar_wait(mma_done, 0, nullptr, 200000000ull)) atomicOr(args.status, kStatusDrainTimeout);
  } else if (SPLIT && warp >= 2) {
    // ---------------- split mode: wait for the accumulator; the push follows below ----------
    split_ready = __all_sync(0xffffffffu, mbar_wait(&tmem_full[0], 0, abort_flag));
    if (!split_ready && lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
  } else if (!SPLIT && warp >= 2) {
    // ---------------- epilogue (both CTAs, own 128 rows) ----------------
    const int quarter = warp & 3;
    uint8_t* staging = epi + (warp - 2) * 2 * kEpilogueStageBytes;
    int buf = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < args.num_tiles; tile += pairs) {
      int pm, pn;
      grouped_tile(tile, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
      const int row0 = pm * 256 + static_cast<int>(rank) * 128 + quarter * 32;
      const int n0 = pn * BN;
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&tmem_full[acc], acc_phase, abort_flag));
      if (!ready) {
        if (lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
        break;
      }
      tc_fence_after_sync();
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               acc * S::kAccCols + c * 64;
        uint32_t lo[32], hi[32];
        tmem_ld_32x32b_x32(taddr, lo);
        tmem_ld_32x32b_x32(taddr + 32, hi);
        tmem_ld_wait();
        uint8_t* dst = staging + buf * kEpilogueStageBytes;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
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
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_c, dst, n0 + c * 64, row0);
          bulk_commit_group();
        }
        if (fanout.count > 0) {
          // Each lane moves 8 of the sub-tile's 256 16-byte chunks; one shared-memory read per
          // chunk feeds every peer. Rows and columns past the slice are skipped.
          const uint32_t src = smem_addr(dst);
#pragma unroll 1
          for (int i = static_cast<int>(lane); i < 256; i += 32) {
            const int r = i >> 3, ch = i & 7;
            const int m = row0 + r, n = n0 + c * 64 + ch * 8;
            if (m >= args.m || n >= args.n) continue;
            const float4 v = ld_shared_f32x4(src + r * 128 + ((ch ^ (r & 7)) << 4));
            const bool full8 = n + 8 <= args.n;
            for (int q = 0; q < fanout.count; ++q) {
              __half* out = reinterpret_cast<__half*>(fanout.peers[q]) + static_cast<int64_t>(m) * fanout.ldc + n;
              if (full8) {
                *reinterpret_cast<float4*>(out) = v;
              } else {
                const __half* h = reinterpret_cast<const __half*>(&v);
                for (int j = 0; j < 8 && n + j < args.n; ++j) out[j] = h[j];
              }
            }
          }
        }
        buf ^= 1;
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) {
          mbar_arrive(&tmem_empty[acc]);
        } else {
          mbar_arrive_cluster(map_to_rank(smem_addr(&tmem_empty[acc]), leader));
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    if (fanout.count > 0) __threadfence_system();  // peer stores are visible before exit
    __syncwarp();
  }

  if constexpr (SPLIT) {
    const int splits = split_args.splits;
    const int cols = BN / splits;              // columns each CTA owns
    const int slot_bytes = 128 * cols * 4;     // one source split's slice, FP32
    const int row_bytes = cols * 4;
    const uint32_t base = smem_addr(ring);
    cluster_sync();  // every main loop is done: all rings are free to receive
    if (warp >= 2 && split_ready) {
      // ---- push: TMEM -> owner CTA's shared memory, slot = this CTA's split ----
      tc_fence_after_sync();
      const int quarter = warp & 3;
      const uint32_t row = static_cast<uint32_t>(quarter * 32) + lane;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c, v);
        tmem_ld_wait();
        const int owner = c / cols;            // 32-column chunks never straddle two owners
        const int local = c - owner * cols;    // first column inside the owner's slice
        const uint32_t dst = map_to_rank(
            base + split * slot_bytes + row * row_bytes, rank + 2u * static_cast<uint32_t>(owner));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t chunk = static_cast<uint32_t>(local / 4 + j);
          st_dsmem_v4(dst + ((chunk ^ (row & 7u)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                      v[4 * j + 3]);
        }
      }
    }
    cluster_sync();  // every slice has arrived
    // ---- reduce locally in split order and store FP16 C ----
    const int chunks = cols / 4;
    int pm, pn;
    grouped_tile(pair, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
    const int row_base = pm * 256 + static_cast<int>(rank) * 128;
    const int col_base = pn * BN + split * cols;
    const bool vec = (split_args.ldc % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(split_args.c) & 7) == 0);
    for (int i = threadIdx.x; i < 128 * chunks; i += blockDim.x) {
      const uint32_t row = static_cast<uint32_t>(i / chunks);
      const uint32_t chunk = static_cast<uint32_t>(i % chunks);
      const uint32_t offset = row * row_bytes + ((chunk ^ (row & 7u)) << 4);
      float4 acc = ld_shared_f32x4(base + offset);
      for (int s2 = 1; s2 < splits; ++s2) {
        const float4 v = ld_shared_f32x4(base + s2 * slot_bytes + offset);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int m = row_base + static_cast<int>(row);
      const int n = col_base + static_cast<int>(chunk) * 4;
      if (m < args.m) {
        __half* dst = split_args.c + static_cast<int64_t>(m) * split_args.ldc + n;
        if (vec && n + 3 < args.n) {
          __half2 lo = __floats2half2_rn(acc.x, acc.y);
          __half2 hi = __floats2half2_rn(acc.z, acc.w);
          uint2 packed;
          packed.x = *reinterpret_cast<uint32_t*>(&lo);
          packed.y = *reinterpret_cast<uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(dst) = packed;
        } else {
          const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
          for (int j = 0; j < 4 && n + j < args.n; ++j) dst[j] = __float2half_rn(vals[j]);
        }
      }
    }
  }

  tc_fence_before_sync();
  cluster_sync();  // the leader's UMMAs read the peer's shared memory until here
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, S::kTmemCols);
  }
}

}  // namespace hst
