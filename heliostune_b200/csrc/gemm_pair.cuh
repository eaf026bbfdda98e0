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
//   * the leader's tcgen05.commit releases each stage in both CTAs (one commit, multicast onto
//     both CTAs' barriers) and publishes each finished accumulator to both CTAs' epilogues;
//   * each CTA drains its own 128 rows x BN columns exactly like the single-SM kernel, and its
//     epilogue warps report a free accumulator on the leader's barrier.
// The kernel is persistent: cluster p walks tiles p, p + #pairs, ... in the grouped raster, with
// two TMEM accumulators so a tile's epilogue overlaps the next tile's main loop.
//
// SPLIT = true (split-K for tile counts far below the SM count): the cluster grows to (2, S):
// S pairs compute the same 256 x BN tile over S contiguous K ranges. CTA (r, s) owns columns
// [s*BN/S, (s+1)*BN/S) of its 128 rows. Once every CTA's main loop is done (cluster barrier, so
// all rings are drained), each CTA stages the column slices it does not own from TMEM into its
// own shared memory, 64 columns at a time, and sends each piece with one asynchronous bulk copy
// into the owner's receive slot while it stages the next (completed in bytes on the owner's
// mbarrier of that piece). The owner then adds, piece by piece as they arrive and in split
// order, its own columns read straight from TMEM and the S - 1 received pieces, and stores FP16
// C through the usual staged TMA-store epilogue. One tile per cluster; no workspace, no atomics,
// bitwise reproducible.
//
// Stream-K (persistent mode with PairStreamKArgs::sk_tiles > 0), for tile counts that leave the
// last wave of pairs part-empty: the first sk_tiles tiles are cut along K into one contiguous
// range of (tile, K block) iterations per pair, so every pair does the same number of K
// blocks; the remaining tiles follow round-robin as whole tiles. A piece that does not start at
// the tile's first K block is published as an FP32 partial tile in global memory (one slot per
// pair, 16-byte chunks laid out so a warp's 32 rows are one 512-byte run) with a release flag
// per epilogue warp. The piece holding the tile's first K blocks belongs to the highest-numbered
// pair among the tile's pieces and is the last of that pair's stream-K work; its epilogue waits
// for the flags, adds the partials in K order onto its accumulator and stores FP16 C. Finishers
// only ever wait on lower-numbered pairs, which never wait on them. Bitwise reproducible.
// No TMA load here feeds more than one CTA's shared memory.
#pragma once

#include "gemm_tile.cuh"
#include "ptx.cuh"

namespace hst {

// BN = 512 ("wide"): two N = 256 UMMAs per K step into the two halves of TMEM, which then holds
// one 128 x 512 FP32 accumulator per CTA instead of two 128 x 256 ones. Each SM moves 48 KB per
// 64-deep K block for 2 x 128 x 256 x 64 multiply-adds -- a quarter fewer L2-to-SM bytes per
// FLOP than the 256-wide tile -- at the price of the double-buffered accumulator: the epilogue
// frees the first half as soon as it has drained it, and the UMMA issuer runs the next tile's
// first-half UMMAs on the stages it holds until the second half is free too.
template <int BN, int BK>
struct PairShape {
  static_assert(BN == 128 || BN == 256 || BN == 512, "pair tiles are 256 x 128, 256 or 512");
  static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
  static_assert(BN != 512 || BK == 64, "the 512-wide tile uses BK 64");
  static constexpr bool kWide = BN == 512;
  static constexpr int kHalfN = BN / 2;         // B columns each CTA loads per tile
  static constexpr int kAtomsK = BK / 64;
  static constexpr int kAtomsN = kHalfN / 64;
  static constexpr int kABoxBytes = 128 * 128;  // 128 rows x 64 k
  static constexpr int kBBoxBytes = BK * 128;   // BK rows x 64 n
  static constexpr int kABytes = kAtomsK * kABoxBytes;
  static constexpr int kBBytes = kAtomsN * kBBoxBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;  // per CTA
  static constexpr int kUmmaN = kWide ? 256 : BN;          // N of one UMMA
  static constexpr int kAccCols = kWide ? 0 : BN;          // column offset of accumulator 1
  static constexpr int kTmemCols = BN == 128 ? 256 : 512;  // two accumulators, or one wide one
  static constexpr int kEpilogueBytes = 4 * 2 * kEpilogueStageBytes;
  static constexpr int kBarrierBytes = 256 + 16 * kMaxStages;
  static constexpr uint32_t kIdesc = umma_idesc_f16(256, kUmmaN, false, true);
  static constexpr int smem_bytes(int stages) {
    return 1024 + stages * kStageBytes + kEpilogueBytes + kBarrierBytes;
  }
  // Tile column of this CTA's B atom `na`: the 256-wide UMMAs each take 128 columns per CTA.
  __host__ __device__ static constexpr int b_col(int rank, int na) {
    return kWide ? (na / 2) * 256 + rank * 128 + (na % 2) * 64 : rank * kHalfN + na * 64;
  }
};

// Column-parallel fan-out of the persistent pair kernel: every finished 64-column sub-tile of
// this rank's C slice is also written into the same columns of the other ranks' C over NVLink,
// in one of two forms. The local copy goes through the TMA store.
//   * stores (count > 0): the epilogue warp reads the staged sub-tile back once per lane and
//     writes it to every peer with coalesced 16-byte stores (peer pointers);
//   * bulk (bulk_count > 0): the warp's elected lane issues one more TMA tensor store of the
//     staged sub-tile per peer (each peer's C slice as a tensor map), in the same bulk group as
//     the local one, so the copy engine of the SM moves it while the warp drains on.
constexpr int kMaxPeers = 8;
struct PairFanoutArgs {
  CUtensorMap peer_maps[kMaxPeers];  // bulk form: peer q's C slice [m, cols], 64 x 32 boxes
  uint64_t peers[kMaxPeers];         // stores form: peer C base + this rank's column offset
  int count;                         // stores form: number of peers (0 = none)
  int bulk_count;                    // bulk form: number of peer maps (0 = none)
  int64_t ldc;                       // row stride of every rank's full C, elements
};

struct PairSplitArgs {
  int splits;        // cluster extent along y (1 = persistent mode)
  int kb_per_split;  // K blocks of one split
  __half* c;         // C for the split-mode epilogue (row stride ldc)
  int64_t ldc;
};

struct PairStreamKArgs {
  int sk_tiles;               // tiles [0, sk_tiles) are shared out along K (0 = whole tiles only)
  float* partials;            // [pairs][2 CTAs][BN / 4 chunks][128 rows][4] FP32, one tile per pair
  unsigned long long* flags;  // [pairs][2 CTAs][4 epilogue warps] publication words
  unsigned long long token;   // the value that publishes a partial in this launch
};

// The work of one pair in order, as segments (tile, [kb0, kb1)): first its share of the
// stream-K iterations (tile-major, K-block-minor over tiles [0, sk_tiles); pair p takes share
// pairs - 1 - p), then whole tiles sk_tiles + p, sk_tiles + p + pairs, ...
struct PairWork {
  int64_t total;  // stream-K iterations of all pairs
  int64_t it, hi;
  int pairs, next_tile, num_tiles, k_blocks;

  __device__ static int64_t share_begin(int64_t total, int pairs, int pair) {
    return total * (pairs - 1 - pair) / pairs;
  }
  __device__ static int64_t share_end(int64_t total, int pairs, int pair) {
    return total * (pairs - pair) / pairs;
  }
  __device__ PairWork(const TileArgs& a, int sk_tiles, int pair, int pairs_)
      : total(int64_t(sk_tiles) * a.k_blocks),
        pairs(pairs_),
        next_tile(sk_tiles + pair),
        num_tiles(a.num_tiles),
        k_blocks(a.k_blocks) {
    it = share_begin(total, pairs, pair);
    hi = share_end(total, pairs, pair);
  }
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (it < hi) {
      tile = static_cast<int>(it / k_blocks);
      kb0 = static_cast<int>(it - int64_t(tile) * k_blocks);
      const int64_t left = hi - it;
      kb1 = left < int64_t(k_blocks - kb0) ? kb0 + static_cast<int>(left) : k_blocks;
      it += kb1 - kb0;
      return true;
    }
    if (next_tile < num_tiles) {
      tile = next_tile;
      kb0 = 0;
      kb1 = k_blocks;
      next_tile += pairs;
      return true;
    }
    return false;
  }
};

template <int BN, int BK, bool SPLIT>
__global__ void __launch_bounds__(kTileThreads, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const TileArgs args,
                     const PairSplitArgs split_args, const __grid_constant__ PairFanoutArgs fanout,
                     const PairStreamKArgs sk) {
  using S = PairShape<BN, BK>;

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
  uint64_t* recv_bar = mma_done + 1;  // split mode: one per 64-column piece this CTA owns
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 2);
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
  const int sk_tiles = SPLIT ? 0 : sk.sk_tiles;
  // One segment of this pair's work: split mode has one tile and this split's K blocks.
  auto next_segment = [&](PairWork& work, int& tile, int& kb0, int& kb1) {
    if (!work.next(tile, kb0, kb1)) return false;
    if (SPLIT) {
      kb0 = kb_begin;
      kb1 = kb_end;
    }
    return true;
  };

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
    if (SPLIT) {
      // Armed before anyone can send: a piece's phase completes once all S - 1 copies are here.
      for (int q = 0; q < BN / split_args.splits / 64; ++q) {
        mbar_init(&recv_bar[q], 1);
        mbar_arrive_expect_tx(&recv_bar[q], (split_args.splits - 1) * 128 * 64 * 4);
      }
    }
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
    PairWork work(args, sk_tiles, pair, pairs);
    int tile, kb0, kb1;
    while (ok && next_segment(work, tile, kb0, kb1)) {
      int pm, pn;
      grouped_tile(tile, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
      const int m0 = pm * 256 + static_cast<int>(rank) * 128;
      const int n0 = pn * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
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
                           n0 + S::b_col(static_cast<int>(rank), na), k0, policy);
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
    PairWork work(args, sk_tiles, pair, pairs);
    int tile, kb0, kb1;
    // Stage 0's A and B descriptors at K step 0. Any other operand's descriptor adds its byte
    // offset / 16 to the start-address field (bits 0-13; shared memory stays below 256 KB).
    const uint64_t a_desc0 = smem_desc(smem_addr(ring), 16, 1024);
    const uint64_t b_desc0 = smem_desc(smem_addr(ring) + S::kABytes, S::kBBoxBytes, 1024);
    // UMMAs of one K block of stage `st` into accumulator columns [col, col + kUmmaN); B atoms
    // from `b_atom` on. `first`: the segment's first K block (overwrite instead of accumulate).
    auto issue = [&](int st, uint32_t col, int b_atom, bool first) {
      const uint64_t a_st = a_desc0 + static_cast<uint64_t>(st * (S::kStageBytes >> 4));
      const uint64_t b_st = b_desc0 + static_cast<uint64_t>(st * (S::kStageBytes >> 4) +
                                                            b_atom * (S::kBBoxBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t adesc = a_st + (((kk >> 2) * S::kABoxBytes + (kk & 3) * 32) >> 4);
        const uint64_t bdesc = b_st + ((kk * 2048) >> 4);
        umma_f16_pair(tmem_base + col, adesc, bdesc, S::kIdesc, (!first || kk != 0) ? 1u : 0u);
      }
    };
    // Both CTAs of the pair (cluster ranks crank and crank + 1; the leader's rank is even).
    const uint16_t pair_mask = static_cast<uint16_t>(3u << crank);
    auto release_stage = [&](int st) { umma_commit_pair_multicast(smem_addr(&empty[st]), pair_mask); };
    while (ok && next_segment(work, tile, kb0, kb1)) {
      if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusMmaTimeout);
        ok = false;
        break;
      }
      tc_fence_after_sync();
      // Wide tile: the second accumulator half may still be draining. Its UMMAs wait, on the
      // stages this thread holds, until the epilogue frees it or every stage is held.
      bool second = !S::kWide;
      int held = 0, held_stage = stage;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          raise_abort(args.status, abort_flag, kStatusMmaTimeout);
          ok = false;
          break;
        }
        tc_fence_after_sync();
        issue(stage, static_cast<uint32_t>(acc * S::kAccCols), 0, kb == kb0);
        if constexpr (S::kWide) {
          if (second) {
            issue(stage, 256u, 2, kb == kb0);
            release_stage(stage);
          } else {
            ++held;
            if (held == stages || mbar_test_wait(&tmem_empty[1], acc_phase ^ 1u)) {
              if (!mbar_wait(&tmem_empty[1], acc_phase ^ 1u, abort_flag)) {
                raise_abort(args.status, abort_flag, kStatusMmaTimeout);
                ok = false;
                break;
              }
              tc_fence_after_sync();
              second = true;
              for (int j = 0; j < held; ++j) {
                const int st = (held_stage + j) % stages;
                issue(st, 256u, 2, j == 0);
                release_stage(st);
              }
              held = 0;
            }
          }
        } else {
          release_stage(stage);
        }
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok && !second) {
        // A segment shorter than the ring: the held K blocks' second halves.
        if (!mbar_wait(&tmem_empty[1], acc_phase ^ 1u, abort_flag)) {
          raise_abort(args.status, abort_flag, kStatusMmaTimeout);
          ok = false;
        } else {
          tc_fence_after_sync();
          for (int j = 0; j < held; ++j) {
            const int st = (held_stage + j) % stages;
            issue(st, 256u, 2, j == 0);
            release_stage(st);
          }
        }
      }
      if (!ok) break;
      umma_commit_pair_multicast(smem_addr(&tmem_full[acc]), pair_mask);
      if (S::kWide) {
        acc_phase ^= 1u;
      } else if (++acc == 2) {
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
    const int row = quarter * 32 + static_cast<int>(lane);  // row of this CTA's 128
    uint8_t* staging = epi + (warp - 2) * 2 * kEpilogueStageBytes;
    int buf = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    constexpr int kChunks = BN / 4;  // 16-byte chunks of one partial-tile row
    // Partial-tile slot of pair q for this CTA, and its publication word for this warp.
    auto slot_of_pair = [&](int q) {
      return sk.partials + (static_cast<size_t>(q) * 2 + rank) * (kChunks * 128 * 4);
    };
    auto flag_of_pair = [&](int q) { return sk.flags + (static_cast<size_t>(q) * 2 + rank) * 4 + quarter; };
    // Reports accumulator `which` (or, for the wide tile, accumulator half `which`) drained, on
    // the leader's barrier.
    auto release_acc = [&](int which) {
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) {
          mbar_arrive_relaxed(&tmem_empty[which]);
        } else {
          mbar_arrive_cluster_relaxed(map_to_rank(smem_addr(&tmem_empty[which]), leader));
        }
      }
    };
    PairWork work(args, sk_tiles, pair, pairs);
    int tile, kb0, kb1;
    while (next_segment(work, tile, kb0, kb1)) {
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
      const uint32_t lane_tmem = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * S::kAccCols;
      const int64_t tile_end = int64_t(tile + 1) * args.k_blocks;  // stream-K iteration after the tile
      bool released0 = !S::kWide;  // wide tile: first accumulator half reported drained
      if (kb0 > 0) {
        // ---- a later K range of a shared tile: publish it as an FP32 partial ----
        float* slot = slot_of_pair(pair);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(lane_tmem + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            st_global_v4(slot + (static_cast<size_t>(c / 4 + j) * 128 + row) * 4, v[4 * j], v[4 * j + 1],
                         v[4 * j + 2], v[4 * j + 3]);
          }
          if (!released0 && c + 32 == 256) {
            release_acc(0);
            released0 = true;
          }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu_u64(flag_of_pair(pair), sk.token);
      } else {
        // ---- a whole tile, or a shared tile's first K range: its finisher ----
        const bool finisher = kb1 < args.k_blocks;
        bool have = true;
        if (finisher) {
          // The tile's later K ranges belong to pairs pair - 1, pair - 2, ... (adjacent shares).
          int64_t pos = work.it;  // first iteration after this pair's piece
          for (int q = pair - 1; q >= 0 && pos < tile_end && have; --q) {
            const int64_t end = PairWork::share_end(work.total, pairs, q);
            if (end > pos && lane == 0) have = wait_flag_u64(flag_of_pair(q), sk.token, abort_flag);
            pos = end > pos ? end : pos;
          }
          have = __all_sync(0xffffffffu, have);
          if (!have && lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
        }
        // Sub-tile c (64 columns) through staging buffer `buf`: one TMA store, and the peers'
        // copies when the tile fans out.
        auto drain = [&](int c, const uint32_t (&lo)[32], const uint32_t (&hi)[32]) {
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
            for (int q = 0; q < fanout.bulk_count; ++q) tma_store_2d(&fanout.peer_maps[q], dst, n0 + c * 64, row0);
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
        };
        if (!finisher) {
          // A whole tile: sub-tile c + 1's TMEM loads are in flight while sub-tile c is stored.
          uint32_t lo[2][32], hi[2][32];
          tmem_ld_32x32b_x32(lane_tmem, lo[0]);
          tmem_ld_32x32b_x32(lane_tmem + 32, hi[0]);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            const int cur = c & 1;
            if (c + 1 < BN / 64) {
              tmem_ld_32x32b_x32(lane_tmem + (c + 1) * 64, lo[cur ^ 1]);
              tmem_ld_32x32b_x32(lane_tmem + (c + 1) * 64 + 32, hi[cur ^ 1]);
            }
            drain(c, lo[cur], hi[cur]);
            if (c + 1 < BN / 64) {
              tmem_ld_wait();
              tmem_ld_fence_regs(lo[cur ^ 1]);
              tmem_ld_fence_regs(hi[cur ^ 1]);
              if (!released0 && (c + 2) * 64 == 256) {
                release_acc(0);
                released0 = true;
              }
            }
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < BN / 64 && have; ++c) {
            const uint32_t taddr = lane_tmem + c * 64;
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(taddr, lo);
            tmem_ld_32x32b_x32(taddr + 32, hi);
            tmem_ld_wait();
            if (!released0 && c * 64 + 64 == 256) {
              release_acc(0);
              released0 = true;
            }
            // Add the later K ranges in K order (pair - 1 first).
            int64_t pos = work.it;
            for (int q = pair - 1; q >= 0 && pos < tile_end; --q) {
              const int64_t end = PairWork::share_end(work.total, pairs, q);
              if (end > pos) {
                const float* part = slot_of_pair(q) + (static_cast<size_t>(c * 16) * 128 + row) * 4;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float4 p = ld_global_cg_f32x4(part + static_cast<size_t>(j) * 128 * 4);
                  uint32_t* d = j < 8 ? &lo[4 * j] : &hi[4 * (j - 8)];
                  d[0] = __float_as_uint(__uint_as_float(d[0]) + p.x);
                  d[1] = __float_as_uint(__uint_as_float(d[1]) + p.y);
                  d[2] = __float_as_uint(__uint_as_float(d[2]) + p.z);
                  d[3] = __float_as_uint(__uint_as_float(d[3]) + p.w);
                }
                pos = end;
              }
            }
            drain(c, lo, hi);
          }
        }
      }
      if (!released0) release_acc(0);
      if (S::kWide) {
        release_acc(1);
        acc_phase ^= 1u;
      } else {
        release_acc(acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    if (fanout.count > 0 || fanout.bulk_count > 0) __threadfence_system();  // peer writes visible before exit
    __syncwarp();
  }

  if constexpr (SPLIT) {
    const int splits = split_args.splits;
    const int cols = BN / splits;                 // columns each CTA owns (>= 64)
    const int pieces = cols / 64;                 // 64-column pieces of one slice
    constexpr int kPieceBytes = 128 * 64 * 4;     // one 128-row FP32 piece, 256-byte rows
    uint8_t* outgoing = ring;                     // the S - 1 slices this CTA sends
    uint8_t* incoming = ring + (splits - 1) * pieces * kPieceBytes;  // the S - 1 it receives
    // Slot of split `src` among the S - 1 slices CTA `dst` exchanges (its own is never sent).
    auto slot_of = [](int src, int dst) { return src < dst ? src : src - 1; };
    cluster_sync();  // every main loop is done: all rings are free
    if (warp >= 2) {
      const int quarter = warp & 3;
      const uint32_t row = static_cast<uint32_t>(quarter * 32) + lane;
      const uint32_t lane_tmem = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      if (split_ready) tc_fence_after_sync();
      // ---- send: stage each 64-column piece other CTAs own, then copy it while the next is
      // staged; each piece completes on the owner's barrier of that piece ----
#pragma unroll 1
      for (int owner = 0; owner < splits; ++owner) {
        if (owner == split) continue;
        const uint32_t owner_rank = rank + 2u * static_cast<uint32_t>(owner);
#pragma unroll 1
        for (int q = 0; q < pieces; ++q) {
          uint8_t* piece = outgoing + (slot_of(owner, split) * pieces + q) * kPieceBytes;
          if (split_ready) {
            uint32_t v[32];
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              tmem_ld_32x32b_x32(lane_tmem + owner * cols + q * 64 + h * 32, v);
              tmem_ld_wait();
              const uint32_t dst = smem_addr(piece) + row * 256;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t chunk = static_cast<uint32_t>(h * 8 + j);
                st_shared_v4(dst + ((chunk ^ (row & 7u)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                             v[4 * j + 3]);
              }
            }
          }
          fence_proxy_async_smem();
          named_barrier(1, 128);
          if (warp == 2 && lane == 0 && split_ready) {
            bulk_copy_to_cluster(
                map_to_rank(smem_addr(incoming + (slot_of(split, owner) * pieces + q) * kPieceBytes), owner_rank),
                piece, static_cast<uint32_t>(kPieceBytes), map_to_rank(smem_addr(&recv_bar[q]), owner_rank));
          }
        }
      }
      // ---- receive: each owned piece as soon as its S - 1 copies are here ----
      int pm, pn;
      grouped_tile(pair, args.tiles_m, args.tiles_n, args.group_m, pm, pn);
      const int row0 = pm * 256 + static_cast<int>(rank) * 128 + quarter * 32;
      uint8_t* staging = epi + (warp - 2) * 2 * kEpilogueStageBytes;
      int buf = 0;
#pragma unroll 1
      for (int q = 0; q < pieces; ++q) {
        const bool arrived = __all_sync(0xffffffffu, mbar_wait(&recv_bar[q], 0, abort_flag));
        if (!arrived && lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
        if (!split_ready || !arrived) break;
        const int c = q * 64;
        uint32_t own[64];
        tmem_ld_32x32b_x32(lane_tmem + split * cols + c, *reinterpret_cast<uint32_t(*)[32]>(own));
        tmem_ld_32x32b_x32(lane_tmem + split * cols + c + 32, *reinterpret_cast<uint32_t(*)[32]>(own + 32));
        tmem_ld_wait();
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.f;
        for (int src = 0; src < splits; ++src) {  // split order
          if (src == split) {
#pragma unroll
            for (int j = 0; j < 64; ++j) acc[j] = src == 0 ? __uint_as_float(own[j]) : acc[j] + __uint_as_float(own[j]);
          } else {
            const uint32_t base_addr =
                smem_addr(incoming + (slot_of(src, split) * pieces + q) * kPieceBytes) + row * 256;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float4 v = ld_shared_f32x4(base_addr + ((static_cast<uint32_t>(j) ^ (row & 7u)) << 4));
              if (src == 0) {
                acc[4 * j] = v.x; acc[4 * j + 1] = v.y; acc[4 * j + 2] = v.z; acc[4 * j + 3] = v.w;
              } else {
                acc[4 * j] += v.x; acc[4 * j + 1] += v.y; acc[4 * j + 2] += v.z; acc[4 * j + 3] += v.w;
              }
            }
          }
        }
        uint8_t* dst = staging + buf * kEpilogueStageBytes;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        const uint32_t row_addr = smem_addr(dst) + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), pack_half2(acc[8 * j], acc[8 * j + 1]),
                       pack_half2(acc[8 * j + 2], acc[8 * j + 3]), pack_half2(acc[8 * j + 4], acc[8 * j + 5]),
                       pack_half2(acc[8 * j + 6], acc[8 * j + 7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_c, dst, pn * BN + split * cols + c, row0);
          bulk_commit_group();
        }
        buf ^= 1;
      }
      if (lane == 0) bulk_wait_group<0>();
      __syncwarp();
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
