// Weight-streaming GEMM with an in-cluster split-K reduction (the B200 "stream" family).
//
// Same swapped MMA as stream_gemm_kernel (C^T tile = B^T * A^T, UMMA M = 128 columns of C,
// UMMA N = MP rows of A), with two changes for small M:
//   * a CTA may own NA = 2 column atoms (256 columns of C): both UMMAs share the A^T tile of a
//     stage, halving the A bytes each CTA pulls per byte of B;
//   * the S CTAs (1 <= S <= 8) that split one column tile's K range form a thread-block cluster
//     (1, S, 1); CTA r owns columns [r*W, min((r+1)*W, NT)) of the tile, W = ceil(NT/S) rounded
//     up to a multiple of 4. Each CTA pushes every column slice of its FP32 accumulator from TMEM
//     into the owner's shared memory (remote stores, slot = source split, row-major [MP][W] so
//     that a warp's store covers 128 contiguous bytes); each owner sums its S slots in split
//     order 0..S-1 and writes FP16 C. Two ways to meet, by accumulator height:
//       - MP <= 64 (a few stores per thread): asynchronous stores whose bytes complete on the
//         owner's receive mbarrier, pushed as soon as the CTA's own accumulator is complete
//         when the slots fit beside the TMA ring ("early"; a cluster barrier armed at launch
//         guarantees every receive barrier exists), else into the drained ring after a
//         cluster barrier;
//       - MP >= 128: plain remote stores (cheaper per byte than the asynchronous stores once
//         each thread sends 128 words), into slots beside the ring pushed as soon as the CTA's
//         own accumulator is complete when they cost no ring stage (completion by a cluster
//         barrier), else into the drained ring between two cluster barriers.
//     No workspace, no second kernel, no atomics; the result is bitwise reproducible.
// With S = 1 the epilogue writes C straight from TMEM.
//
// RMSNorm prologue (NORM = true): C = RMSNorm(A; gamma, eps) * B for an unnormalised A. While the
// main loop runs, the four epilogue warps take every A^T tile as it lands, add its squares to
// per-row FP32 sums and rewrite it in place as fp16(a * gamma[k]); the UMMAs wait for that
// (a second barrier per stage). The row factors rsqrt(sum / K + eps) are applied to the FP32
// results in the epilogue, after the per-split sums have crossed the cluster with the slices.
#pragma once

#include "ptx.cuh"

namespace hst {

struct ClusterStreamArgs {
  int m, n, k;
  int k_blocks;
  int kb_per_split;
  int splits;  // cluster size along y
  int stages;
  int early;   // exchange slots beside the ring (1) or in it after the main loops (0)
  float eps;            // RMSNorm prologue (NORM): eps and gamma [k]
  const __half* gamma;
  int* status;
  __half* c;
  int64_t ldc;
};

template <int NA, int MP, int BK>
struct ClusterStreamShape {
  static_assert(NA == 1 || NA == 2, "one or two 128-column atoms per CTA");
  static_assert(MP % 16 == 0 && MP >= 16 && MP <= 256, "MP must be a multiple of 16 up to 256");
  static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
  static constexpr int kNT = 128 * NA;
  static constexpr int kAtomsN = kNT / 64;
  static constexpr int kAtomsK = BK / 64;
  static constexpr int kWBoxBytes = BK * 128;
  static constexpr int kXBoxBytes = MP * 128;
  static constexpr int kWBytes = kAtomsN * kWBoxBytes;
  static constexpr int kXBytes = kAtomsK * kXBoxBytes;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  // Columns each CTA of an S-CTA cluster owns (the last may own fewer).
  __host__ __device__ static constexpr int owner_cols(int splits) {
    return ((kNT + splits - 1) / splits + 3) / 4 * 4;
  }
  // The S exchange slots, [MP][owner_cols] FP32 each, then (RMSNorm prologue) S row-sum slots
  // of MP floats.
  __host__ __device__ static constexpr int exchange_bytes(int splits, bool norm) {
    return splits * owner_cols(splits) * MP * 4 + (norm ? splits * MP * 4 : 0);
  }
  static constexpr int kCols = NA * MP;
  static constexpr int kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  static constexpr uint32_t kIdesc = umma_idesc_f16(128, MP, true, false);
  static constexpr int kBarrierBytes = 256 + 16 * kStreamMaxStages;
  static constexpr bool kAsyncPush = MP <= 64;  // see the file comment
  // Shared memory below the barriers: ring and exchange side by side, or overlaid; then the
  // per-stage gamma slices of the RMSNorm prologue.
  __host__ __device__ static constexpr int data_bytes(int stages, int splits, bool early, bool norm) {
    return (early ? stages * kStageBytes + exchange_bytes(splits, norm)
                  : (stages * kStageBytes > exchange_bytes(splits, norm) ? stages * kStageBytes
                                                                         : exchange_bytes(splits, norm))) +
           (norm ? stages * BK * 2 : 0);
  }
  static constexpr int smem_bytes(int stages, int splits, bool early, bool norm) {
    return 1024 + data_bytes(stages, splits, early, norm) + kBarrierBytes;
  }
};

template <int NA, int MP, int BK, bool NORM>
__global__ void __launch_bounds__(kStreamThreads, 1)
    stream_cluster_kernel(const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b, const ClusterStreamArgs args) {
  using S = ClusterStreamShape<NA, MP, BK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = args.stages;
  const bool early = args.early != 0;
  uint8_t* ring = smem;
  uint8_t* exchange = early ? ring + stages * S::kStageBytes : ring;  // the S slots [MP][W]
  static_assert(!NORM || MP <= 128, "the RMSNorm prologue covers up to 128 rows");
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + S::data_bytes(stages, args.splits, early, NORM));
  __half* gamma_ring = reinterpret_cast<__half*>(bars) - stages * BK;  // [stage][BK] (RMSNorm)
  uint64_t* full = bars;
  uint64_t* empty = bars + kStreamMaxStages;
  uint64_t* tmem_full = bars + 2 * kStreamMaxStages;
  uint64_t* mma_done = tmem_full + 1;
  uint64_t* recv_bar = mma_done + 1;  // bytes of the S slots this CTA owns the sum of
  uint64_t* scaled = recv_bar + 1;    // RMSNorm prologue: stage rewritten by the epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(scaled + kStreamMaxStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  const int n0 = blockIdx.x * S::kNT;
  const int split = blockIdx.y;
  const int kb_begin = split * args.kb_per_split;
  const int kb_end = min(kb_begin + args.kb_per_split, args.k_blocks);

  // One stage's loads, completing on full[stage]: the W atoms, the X atoms and, with the RMSNorm
  // prologue, the stage's slice of gamma.
  auto load_stage = [&](int kb, int stage, uint64_t stream_policy, uint64_t keep_policy) {
    uint8_t* st = ring + stage * S::kStageBytes;
    const int k0 = kb * BK;
    const int gamma_bytes = NORM ? min(BK, args.k - k0) * 2 : 0;  // K % 8 == 0: 16-byte multiple
    mbar_arrive_expect_tx(&full[stage], S::kStageBytes + gamma_bytes);
    if (gamma_bytes > 0)
      bulk_load_global(gamma_ring + stage * BK, args.gamma + k0, static_cast<uint32_t>(gamma_bytes), &full[stage]);
#pragma unroll
    for (int na = 0; na < S::kAtomsN; ++na) {
      tma_load_2d(st + na * S::kWBoxBytes, &map_b, &full[stage], n0 + 64 * na, k0, stream_policy);
    }
#pragma unroll
    for (int ka = 0; ka < S::kAtomsK; ++ka) {
      tma_load_2d(st + S::kWBytes + ka * S::kXBoxBytes, &map_a, &full[stage], k0 + 64 * ka, 0,
                  keep_policy);
    }
  };
  // Stages thread 0 (the producer) loaded before the CTA barrier: the first pass over the ring
  // needs no free stage, so its loads overlap TMEM allocation and the barrier.
  int preloaded = 0;

  if (threadIdx.x == 0) {
    // The ring's full barriers and the first pass's loads before anything else, so that the
    // loads' latency overlaps the rest of the set-up.
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbarrier_init();
    preloaded = max(0, min(stages, kb_end - kb_begin));
    {
      const uint64_t stream_policy = l2_policy_evict_first();
      const uint64_t keep_policy = l2_policy_evict_last();
      for (int s = 0; s < preloaded; ++s) load_stage(kb_begin + s, s, stream_policy, keep_policy);
    }
    for (int s = 0; s < stages; ++s) {
      mbar_init(&empty[s], 1);
      mbar_init(&scaled[s], 4);
    }
    mbar_init(tmem_full, 1);
    mbar_init(mma_done, 1);
    mbar_init(recv_bar, 1);
    if (S::kAsyncPush && args.splits > 1) {
      const int w = S::owner_cols(args.splits);
      const int own_cols = min(w, S::kNT - split * w);
      const int sums = NORM ? args.m : 0;  // the row sums travel with the slices
      mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(args.splits * (args.m * own_cols + sums) * 4));
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  // Every CTA's receive barrier is armed before anyone pushes: the arrive here, the wait below.
  if (args.splits > 1 && early) cluster_arrive_relaxed();
  const uint32_t tmem_base = *tmem_slot;
  bool have_result = false;
  constexpr int kTpr = MP >= 128 ? 1 : 128 / MP;  // RMSNorm prologue: threads per row
  float row_ss = 0.f;                            // this thread's part of its row's sum of squares

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t stream_policy = l2_policy_evict_first();
    const uint64_t keep_policy = l2_policy_evict_last();
    int stage = preloaded == stages ? 0 : preloaded;
    uint32_t phase = preloaded == stages ? 1u : 0u;
    uint32_t issued_mask = (1u << preloaded) - 1u, issued_parity = 0;
    bool ok = true;
    for (int kb = kb_begin + preloaded; kb < kb_end; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusProducerTimeout);
        ok = false;
        break;
      }
      load_stage(kb, stage, stream_policy, keep_policy);
      issued_mask |= 1u << stage;
      issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (!ok) {
      for (int s = 0; s < stages; ++s) {
        if ((issued_mask & (1u << s)) &&
            !mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, 200000000ull)) {
          atomicOr(args.status, kStatusDrainTimeout);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- UMMA issuer ----------------
    // Stage 0's operand descriptors at K step 0; any other operand adds its byte offset / 16 to
    // the start-address field (bits 0-13; shared memory stays below 256 KB).
    const uint64_t w_desc0 = smem_desc(smem_addr(ring), S::kWBoxBytes, 1024);
    const uint64_t x_desc0 = smem_desc(smem_addr(ring) + S::kWBytes, 16, 1024);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int kb = kb_begin; kb < kb_end; ++kb) {
      if (!mbar_wait(NORM ? &scaled[stage] : &full[stage], phase, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusMmaTimeout);
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint64_t stage_off = static_cast<uint64_t>(stage * (S::kStageBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t bdesc =
            x_desc0 + stage_off + (((kk >> 2) * S::kXBoxBytes + (kk & 3) * 32) >> 4);
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          const uint64_t adesc =
              w_desc0 + stage_off + ((a * 2 * S::kWBoxBytes + kk * 2048) >> 4);
          umma_f16(tmem_base + a * MP, adesc, bdesc, S::kIdesc,
                   (kb != kb_begin || kk != 0) ? 1u : 0u);
        }
      }
      umma_commit(&empty[stage]);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (ok) umma_commit(tmem_full);
    umma_commit(mma_done);
    if (!mbar_wait(mma_done, 0, nullptr, 200000000ull)) atomicOr(args.status, kStatusDrainTimeout);
  } else if (warp >= 2) {
    if constexpr (NORM) {
      // ---------------- RMSNorm prologue: sum of squares and gamma on every A^T tile ----------
      // Thread t owns row t / kTpr of the tile and every kTpr-th 16-byte chunk of that row.
      const int t = threadIdx.x - 64;
      const int row = t / kTpr;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end && ok; ++kb) {
        ok = mbar_wait(&full[stage], phase, abort_flag);
        if (!ok) {
          if (lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
          break;
        }
        const uint32_t x_base = smem_addr(ring + stage * S::kStageBytes + S::kWBytes);
        const uint32_t g_base = smem_addr(gamma_ring + stage * BK);
        if (row < MP) {
#pragma unroll
          for (int ka = 0; ka < S::kAtomsK; ++ka) {
            const uint32_t row_addr = x_base + ka * S::kXBoxBytes + row * 128;
#pragma unroll
            for (int i = 0; i < 8 / kTpr; ++i) {
              const int p = t % kTpr + i * kTpr;
              const uint32_t addr = row_addr + (static_cast<uint32_t>(p) << 4);
              const int kl = ka * 64 + ((p ^ (row & 7)) << 3);  // swizzled chunk: its K offset in the block
              const float4 raw = ld_shared_f32x4(addr);
              float4 graw = make_float4(0.f, 0.f, 0.f, 0.f);
              if (kb * BK + kl < args.k) graw = ld_shared_f32x4(g_base + kl * 2);
              const uint32_t xw[4] = {__float_as_uint(raw.x), __float_as_uint(raw.y), __float_as_uint(raw.z),
                                      __float_as_uint(raw.w)};
              const uint32_t gw[4] = {__float_as_uint(graw.x), __float_as_uint(graw.y), __float_as_uint(graw.z),
                                      __float_as_uint(graw.w)};
              uint32_t out[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __half2 xh, gh;
                memcpy(&xh, &xw[e], 4);
                memcpy(&gh, &gw[e], 4);
                const float2 v = __half22float2(xh);
                const float2 g2 = __half22float2(gh);
                row_ss = fmaf(v.x, v.x, row_ss);
                row_ss = fmaf(v.y, v.y, row_ss);
                out[e] = pack_half2(v.x * g2.x, v.y * g2.y);
              }
              st_shared_v4(addr, out[0], out[1], out[2], out[3]);
            }
          }
        }
        fence_proxy_async_smem();  // the rewritten tile is visible to the UMMAs
        __syncwarp();
        if (lane == 0) mbar_arrive(&scaled[stage]);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // One partial sum per row for this CTA's K range: the row's kTpr threads are neighbours.
#pragma unroll
      for (int off = 1; off < kTpr; off <<= 1) row_ss += __shfl_xor_sync(0xffffffffu, row_ss, off);
    }
    // ---------------- epilogue: wait for the accumulator ----------------
    have_result = __all_sync(0xffffffffu, mbar_wait(tmem_full, 0, abort_flag));
    if (!have_result && lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
  }

  constexpr int kChunk = MP >= 32 ? 32 : 16;
  const int splits = args.splits;
  const int cols = S::owner_cols(splits);            // columns of C each CTA of the cluster owns
  const int slot_bytes = MP * cols * 4;              // one source split's slice, FP32 [MP][cols]
  const uint32_t base = smem_addr(exchange);
  if (splits > 1) {
    if (early) {
      cluster_wait();  // every receive barrier is armed
    } else {
      cluster_sync();  // every main loop is done: all rings can receive
    }
  }
  const uint32_t sums = base + splits * slot_bytes;  // RMSNorm row sums: [split][MP] FP32
  auto row_factor = [&](int m) {  // rsqrt(mean of squares + eps) of row m, split order
    float ss = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) {
      float v;
      asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(sums + (s2 * MP + m) * 4) : "memory");
      ss = s2 == 0 ? v : ss + v;
    }
    return rsqrtf(ss / static_cast<float>(args.k) + args.eps);
  };
  if (NORM && warp >= 2) {
    // ---- this CTA's row sums to every owner (with the slices), or to its own table ----
    const int t = threadIdx.x - 64;
    const int row = t / kTpr;
    if (have_result && t % kTpr == 0 && row < args.m) {
      if (splits == 1) {
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(sums + row * 4), "f"(row_ss) : "memory");
      } else {
        for (int owner = 0; owner < splits; ++owner) {
          const uint32_t dst = map_to_rank(sums + (split * MP + row) * 4, static_cast<uint32_t>(owner));
          if constexpr (S::kAsyncPush) {
            st_async_b32(dst, __float_as_uint(row_ss), map_to_rank(smem_addr(recv_bar), static_cast<uint32_t>(owner)));
          } else {
            st_dsmem_b32(dst, __float_as_uint(row_ss));
          }
        }
      }
    }
    if (splits == 1) named_barrier(1, 128);  // every row sum is in the table (all four warps)
  }
  if (warp >= 2 && have_result) {
    // ---- TMEM -> C (one split) or -> the owner's slot (asynchronous stores, own one too) ----
    tc_fence_after_sync();
    const int quarter = warp & 3;
#pragma unroll 1
    for (int a = 0; a < NA; ++a) {
      const int nl = a * 128 + quarter * 32 + static_cast<int>(lane);
      const int n = n0 + nl;
      const int owner = nl / cols;
      const uint32_t dst = splits > 1 ? map_to_rank(base + split * slot_bytes + (nl - owner * cols) * 4,
                                                    static_cast<uint32_t>(owner))
                                      : 0u;
      const uint32_t owner_bar = splits > 1 ? map_to_rank(smem_addr(recv_bar), static_cast<uint32_t>(owner)) : 0u;
      const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + a * MP;
#pragma unroll 1
      for (int c0 = 0; c0 < MP; c0 += kChunk) {
        if (c0 >= args.m) break;  // warp-uniform
        uint32_t r[kChunk];
        if constexpr (kChunk == 32) {
          tmem_ld_32x32b_x32(lane_addr + c0, r);
        } else {
          tmem_ld_32x32b_x16(lane_addr + c0, r);
        }
        tmem_ld_wait();
        if (splits == 1) {
          if (n < args.n) {
            if constexpr (!NORM) {
#pragma unroll
              for (int j = 0; j < kChunk; ++j) {
                const int m = c0 + j;
                if (m < args.m) args.c[static_cast<int64_t>(m) * args.ldc + n] = __float2half_rn(__uint_as_float(r[j]));
              }
            } else {
#pragma unroll
              for (int j = 0; j < kChunk; ++j) {
                const int m = c0 + j;
                if (m < args.m)
                  args.c[static_cast<int64_t>(m) * args.ldc + n] = __float2half_rn(__uint_as_float(r[j]) * row_factor(m));
              }
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kChunk; ++j) {
            if (c0 + j < args.m) {
              if constexpr (S::kAsyncPush) {
                st_async_b32(dst + (c0 + j) * cols * 4, r[j], owner_bar);
              } else {
                st_dsmem_b32(dst + (c0 + j) * cols * 4, r[j]);
              }
            }
          }
        }
      }
    }
  }

  if (splits > 1) {
    // ---- wait for the S slots, reduce in split order and write FP16 C ----
    bool arrived = true;
    if constexpr (S::kAsyncPush) {
      arrived = mbar_wait_cluster(recv_bar, 0, abort_flag);
    } else {
      cluster_sync();  // every slice has arrived
    }
    if (!arrived && threadIdx.x == 64) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
    const int rank = split;
    const int own_cols = min(cols, S::kNT - rank * cols);  // the last owner may have fewer
    const int quads = own_cols / 4;
    const int items = args.m * quads;
    const bool vec_store = (args.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(args.c) & 7) == 0);
    // Item i is row i / quads, quad i % quads; a thread takes items t, t + T, t + 2T, ... (T
    // threads), two at a time so both items' shared loads are in flight together.
    const int step = static_cast<int>(blockDim.x);
    const int dm = step / quads, dq = step % quads;
    int m1 = static_cast<int>(threadIdx.x) / quads, q1 = static_cast<int>(threadIdx.x) % quads;
    auto advance = [&](int& m, int& q) {
      m += dm;
      q += dq;
      if (q >= quads) {
        q -= quads;
        ++m;
      }
    };
    auto reduce = [&](int m, int q) {
      const uint32_t offset = static_cast<uint32_t>((m * cols + q * 4) * 4);
      float4 acc = ld_shared_f32x4(base + offset);
      for (int s = 1; s < splits; ++s) {
        const float4 v = ld_shared_f32x4(base + s * slot_bytes + offset);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      return acc;
    };
    auto store = [&](int m, int q, float4 acc) {
      if constexpr (NORM) {
        const float f = row_factor(m);
        acc.x *= f;
        acc.y *= f;
        acc.z *= f;
        acc.w *= f;
      }
      const int n = n0 + rank * cols + q * 4;
      __half* dst = args.c + static_cast<int64_t>(m) * args.ldc + n;
      if (vec_store && n + 3 < args.n) {
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
    };
    for (int i = static_cast<int>(threadIdx.x); arrived && i < items; i += 2 * step) {
      int m2 = m1, q2 = q1;
      advance(m2, q2);
      const bool second = i + step < items;
      const float4 acc1 = reduce(m1, q1);
      const float4 acc2 = second ? reduce(m2, q2) : acc1;
      store(m1, q1, acc1);
      if (second) store(m2, q2, acc2);
      m1 = m2;
      q1 = q2;
      advance(m1, q1);
    }
  }
  (void)have_result;

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace hst
