// Weight-streaming GEMM for small M (decode-shaped projections), C = A[M,K] * B[K,N].
//
// Restates the reference's split-K path (action_expansion.py:56-173) for sm_100a. Small M makes
// the GEMM a stream of B through HBM, so the MMA is swapped: the CTA computes
//     C^T[n0:n0+NT, 0:M] = B[:, n0:n0+NT]^T * A^T
// with UMMA M = NT columns of C (64 or 128) and UMMA N = MP, the rows of A padded to a multiple
// of 16. The large operand B^T is read N-major straight from B's rows; A^T is K-major straight
// from A's rows. K is cut into `splits` contiguous, BK-aligned intervals
// (tiles_per_split = cdiv(cdiv(K, BK), S), as the reference). With one split the epilogue writes
// FP16 C; otherwise each split writes an FP32 partial [split][M][N] and splitk_reduce_kernel sums
// the partials in split order 0..S-1, so the result is bitwise reproducible (no atomics).
//
// CTA of 192 threads: warp 0 TMA producer, warp 1 TMEM owner + UMMA issuer, warps 2..5 epilogue.
#pragma once

#include "ptx.cuh"

namespace hst {

constexpr int kStreamThreads = 192;
constexpr int kStreamMaxStages = 16;

struct StreamArgs {
  int m, n, k;
  int k_blocks;      // cdiv(K, BK)
  int kb_per_split;  // K blocks of one split
  int stages;
  int* status;
  float* partials;   // [splits][M][N] FP32, or nullptr when the epilogue writes C
  __half* c;         // C[M, N] with row stride ldc, written when partials == nullptr
  int64_t ldc;
};

template <int NT, int MP, int BK>
struct StreamShape {
  static_assert(NT == 64 || NT == 128, "UMMA M must be 64 or 128");
  static_assert(MP % 16 == 0 && MP >= 16 && MP <= 256, "MP must be a multiple of 16 up to 256");
  static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
  static constexpr int kAtomsN = NT / 64;       // 64-column atoms of B^T
  static constexpr int kAtomsK = BK / 64;       // 64-deep atoms of A^T
  static constexpr int kWBoxBytes = BK * 128;   // one TMA box of B: BK rows x 64 n
  static constexpr int kXBoxBytes = MP * 128;   // one TMA box of A: MP rows x 64 k
  static constexpr int kWBytes = kAtomsN * kWBoxBytes;
  static constexpr int kXBytes = kAtomsK * kXBoxBytes;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kTmemCols = MP <= 32 ? 32 : MP;
  static constexpr int kRowsPerWarp = NT / 4;
  static constexpr uint32_t kIdesc = umma_idesc_f16(NT, MP, true, false);
  static constexpr int kBarrierBytes = 256 + 16 * kStreamMaxStages;
  static constexpr int smem_bytes(int stages) {
    return 1024 + stages * kStageBytes + kBarrierBytes;
  }
};

template <int NT, int MP, int BK>
__global__ void __launch_bounds__(kStreamThreads, 1)
    stream_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, const StreamArgs args) {
  using S = StreamShape<NT, MP, BK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = args.stages;
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + stages * S::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStreamMaxStages;
  uint64_t* tmem_full = bars + 2 * kStreamMaxStages;
  uint64_t* mma_done = tmem_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  const int n0 = blockIdx.x * NT;
  const int split = blockIdx.y;
  const int kb_begin = split * args.kb_per_split;
  const int kb_end = min(kb_begin + args.kb_per_split, args.k_blocks);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
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
    const uint64_t stream_policy = l2_policy_evict_first();  // B is read once
    const uint64_t keep_policy = l2_policy_evict_last();     // A is re-read by every CTA
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool ok = true;
    for (int kb = kb_begin; kb < kb_end; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusProducerTimeout);
        ok = false;
        break;
      }
      uint8_t* st = ring + stage * S::kStageBytes;
      mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
      const int k0 = kb * BK;
#pragma unroll
      for (int na = 0; na < S::kAtomsN; ++na) {
        tma_load_2d(st + na * S::kWBoxBytes, &map_b, &full[stage], n0 + 64 * na, k0,
                    stream_policy);
      }
#pragma unroll
      for (int ka = 0; ka < S::kAtomsK; ++ka) {
        tma_load_2d(st + S::kWBytes + ka * S::kXBoxBytes, &map_a, &full[stage], k0 + 64 * ka, 0,
                    keep_policy);
      }
      issued_mask |= 1u << stage;
      issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (!ok) {
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
    const uint64_t w_desc0 = smem_desc(smem_addr(ring), S::kWBoxBytes, 1024);
    const uint64_t x_desc0 = smem_desc(smem_addr(ring) + S::kWBytes, 16, 1024);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int kb = kb_begin; kb < kb_end; ++kb) {
      if (!mbar_wait(&full[stage], phase, abort_flag)) {
        raise_abort(args.status, abort_flag, kStatusMmaTimeout);
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint64_t stage_off = static_cast<uint64_t>(stage * (S::kStageBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t adesc = w_desc0 + stage_off + ((kk * 2048) >> 4);
        const uint64_t bdesc =
            x_desc0 + stage_off + (((kk >> 2) * S::kXBoxBytes + (kk & 3) * 32) >> 4);
        umma_f16(tmem_base, adesc, bdesc, S::kIdesc, (kb != kb_begin || kk != 0) ? 1u : 0u);
      }
      umma_commit(&empty[stage]);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (ok) umma_commit(tmem_full);
    umma_commit(mma_done);
    if (!mbar_wait(mma_done, 0, nullptr, 200000000ull)) {
      atomicOr(args.status, kStatusDrainTimeout);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;
    const bool ready = __all_sync(0xffffffffu, mbar_wait(tmem_full, 0, abort_flag));
    if (!ready) {
      if (lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
    } else {
      tc_fence_after_sync();
      const int n = n0 + quarter * S::kRowsPerWarp + static_cast<int>(lane);
      const bool live = static_cast<int>(lane) < S::kRowsPerWarp && n < args.n;
      const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      constexpr int kChunk = MP >= 32 ? 32 : 16;
#pragma unroll 1
      for (int c0 = 0; c0 < MP; c0 += kChunk) {
        if (c0 >= args.m) break;  // warp-uniform
        float v[kChunk];
        if constexpr (kChunk == 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(lane_addr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        } else {
          uint32_t r[16];
          tmem_ld_32x32b_x16(lane_addr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
        }
        if (live) {
          if (args.partials != nullptr) {
            float* out = args.partials + static_cast<int64_t>(split) * args.m * args.n + n;
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
              const int m = c0 + j;
              if (m < args.m) out[static_cast<int64_t>(m) * args.n] = v[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
              const int m = c0 + j;
              if (m < args.m) args.c[static_cast<int64_t>(m) * args.ldc + n] = __float2half_rn(v[j]);
            }
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// C[m, n] = fp16( sum_{s=0}^{S-1} P[s][m][n] ), summed in split order. Four columns per thread.
// Launched as a programmatic dependent of the partials kernel: it waits for that grid's
// memory before reading, while its own launch overlaps the partials kernel's tail.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partials,
                                                            __half* __restrict__ c, int64_t ldc,
                                                            int m, int n, int splits,
                                                            int vector_ok) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int quads = (n + 3) >> 2;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(m) * quads) return;
  const int row = static_cast<int>(idx / quads);
  const int col = static_cast<int>(idx % quads) * 4;
  const int64_t plane = static_cast<int64_t>(m) * n;
  const float* p = partials + static_cast<int64_t>(row) * n + col;
  if (vector_ok) {
    float4 acc = *reinterpret_cast<const float4*>(p);
    for (int s = 1; s < splits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(p + s * plane);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    __half2 lo = __floats2half2_rn(acc.x, acc.y);
    __half2 hi = __floats2half2_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(c + static_cast<int64_t>(row) * ldc + col) = packed;
  } else {
    const int cols = min(4, n - col);
    for (int j = 0; j < cols; ++j) {
      float acc = p[j];
      for (int s = 1; s < splits; ++s) acc += p[s * plane + j];
      c[static_cast<int64_t>(row) * ldc + col + j] = __float2half_rn(acc);
    }
  }
}

}  // namespace hst
