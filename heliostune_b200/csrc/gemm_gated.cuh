// Gated-MLP projection fused with its epilogue: out = bf16(silu(x Wg^T) * (x Wu^T)), for the
// decode regime (M <= 64). BF16 x [M, K] and the nn.Linear weights Wg, Wu [N, K] (row-major,
// so K-major), FP32 accumulation, BF16 output [M, N]. The reference computes it as two FP32
// matmuls, silu and a product (local_executor.py:1970-1979); here it is one launch that streams
// both weights once and never writes the two [M, N] intermediates.
//
// Weight streaming with the MMA swapped, as the stream family: a CTA computes
// acc^T[n0:n0+128, :M] = W[n0:n0+128, k-range] * x[:, k-range]^T with UMMA M = 128 (rows of W =
// columns of out) and UMMA N = MP (M padded to 16, 32 or 64); both operands are K-major tiles
// loaded by TMA with the 128-byte swizzle, kind::f16 with BF16 A and B.
//
// One 128-column tile of out is shared by a cluster of 2S CTAs (1, 2S, 1): CTA y streams the
// gate rows (y < S) or the up rows (y >= S) over K range y mod S. Every CTA pushes each column
// slice of its FP32 accumulator to the CTA owning those columns (asynchronous stores completing
// on the owner's receive barrier, slot = y); the owner sums slots 0..S-1 (gate) and S..2S-1 (up)
// in split order, applies silu(g) * u and stores BF16. No workspace, no second kernel, no atomics:
// bitwise reproducible.
#pragma once

#include <cuda_bf16.h>

#include "gemm_stream.cuh"
#include "ptx.cuh"

namespace hst {

struct GatedStreamArgs {
  int m, n, k;
  int k_blocks;
  int kb_per_split;
  int splits;  // S: K ranges per weight; the cluster holds 2S CTAs
  int stages;
  int* status;
  __nv_bfloat16* out;
  int64_t ldo;
};

// kind::f16 instruction descriptor with BF16 A and B (format 1), FP32 D, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_kmajor(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

template <int MP, int BK>
struct GatedShape {
  static_assert(MP == 16 || MP == 32 || MP == 64, "M is padded to 16, 32 or 64");
  static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
  static constexpr int kNT = 128;                  // columns of out per cluster tile
  static constexpr int kAtomsK = BK / 64;          // 64-wide K atoms (128 bytes of BF16)
  static constexpr int kWAtomBytes = kNT * 128;    // 128 weight rows x 64 K
  static constexpr int kXAtomBytes = MP * 128;     // MP rows of x x 64 K
  static constexpr int kWBytes = kAtomsK * kWAtomBytes;
  static constexpr int kStageBytes = kWBytes + kAtomsK * kXAtomBytes;
  static constexpr int kTmemCols = MP <= 32 ? 32 : 64;
  static constexpr uint32_t kIdesc = umma_idesc_bf16_kmajor(128, MP);
  static constexpr int kBarrierBytes = 256 + 16 * kStreamMaxStages;
  // Columns each of the 2S CTAs owns (the last may own fewer), rounded to 4 for vector loads.
  __host__ __device__ static constexpr int owner_cols(int ctas) { return ((kNT + ctas - 1) / ctas + 3) / 4 * 4; }
  // 2S slots of FP32 [MP][owner_cols], beside the ring.
  __host__ __device__ static constexpr int exchange_bytes(int ctas) { return ctas * MP * owner_cols(ctas) * 4; }
  __host__ __device__ static constexpr int smem_bytes(int stages, int ctas) {
    return 1024 + stages * kStageBytes + exchange_bytes(ctas) + kBarrierBytes;
  }
};

template <int MP, int BK>
__global__ void __launch_bounds__(kStreamThreads, 1)
    gated_stream_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_gate,
                        const __grid_constant__ CUtensorMap map_up, const GatedStreamArgs args) {
  using G = GatedShape<MP, BK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = args.stages;
  const int ctas = 2 * args.splits;
  uint8_t* ring = smem;
  uint8_t* exchange = ring + stages * G::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(exchange + G::exchange_bytes(ctas));
  uint64_t* full = bars;
  uint64_t* empty = bars + kStreamMaxStages;
  uint64_t* tmem_full = bars + 2 * kStreamMaxStages;
  uint64_t* mma_done = tmem_full + 1;
  uint64_t* recv_bar = mma_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  const int n0 = blockIdx.x * G::kNT;
  const int y = blockIdx.y;  // the CTA's rank in the cluster
  const bool up_half = y >= args.splits;
  const CUtensorMap* map_w = up_half ? &map_up : &map_gate;
  const int split = y % args.splits;
  const int kb_begin = split * args.kb_per_split;
  const int kb_end = min(kb_begin + args.kb_per_split, args.k_blocks);
  const int cols = G::owner_cols(ctas);
  const int own_cols = max(0, min(cols, G::kNT - y * cols));

  auto load_stage = [&](int kb, int stage, uint64_t stream_policy, uint64_t keep_policy) {
    uint8_t* st = ring + stage * G::kStageBytes;
    const int k0 = kb * BK;
    mbar_arrive_expect_tx(&full[stage], G::kStageBytes);
#pragma unroll
    for (int ka = 0; ka < G::kAtomsK; ++ka) {
      tma_load_2d(st + ka * G::kWAtomBytes, map_w, &full[stage], k0 + 64 * ka, n0, stream_policy);
      tma_load_2d(st + G::kWBytes + ka * G::kXAtomBytes, &map_x, &full[stage], k0 + 64 * ka, 0, keep_policy);
    }
  };
  int preloaded = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbarrier_init();
    preloaded = max(0, min(stages, kb_end - kb_begin));
    {
      const uint64_t stream_policy = l2_policy_evict_first();
      const uint64_t keep_policy = l2_policy_evict_last();
      for (int s = 0; s < preloaded; ++s) load_stage(kb_begin + s, s, stream_policy, keep_policy);
    }
    for (int s = 0; s < stages; ++s) mbar_init(&empty[s], 1);
    mbar_init(tmem_full, 1);
    mbar_init(mma_done, 1);
    mbar_init(recv_bar, 1);
    // Bytes this CTA receives: every CTA's slice of its columns, M rows each.
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(ctas * args.m * own_cols * 4));
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, G::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  cluster_arrive_relaxed();  // every receive barrier is armed before anyone pushes (wait below)
  const uint32_t tmem_base = *tmem_slot;
  bool have_result = false;

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
    if (!ok) {  // drain the copies in flight before the CTA can exit
      for (int s = 0; s < stages; ++s) {
        if ((issued_mask & (1u << s)) && !mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, 200000000ull)) {
          atomicOr(args.status, kStatusDrainTimeout);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- UMMA issuer ----------------
    // K-major operands: a 16-deep K step is 32 bytes inside a 64-wide atom; atoms follow each
    // other (W: 16 KB, x: MP x 128 bytes). Offsets add to the start-address field (bytes / 16).
    const uint64_t w_desc0 = smem_desc(smem_addr(ring), 16, 1024);
    const uint64_t x_desc0 = smem_desc(smem_addr(ring) + G::kWBytes, 16, 1024);
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
      const uint64_t stage_off = static_cast<uint64_t>(stage * (G::kStageBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t adesc = w_desc0 + stage_off + (((kk >> 2) * G::kWAtomBytes + (kk & 3) * 32) >> 4);
        const uint64_t bdesc = x_desc0 + stage_off + (((kk >> 2) * G::kXAtomBytes + (kk & 3) * 32) >> 4);
        umma_f16(tmem_base, adesc, bdesc, G::kIdesc, (kb != kb_begin || kk != 0) ? 1u : 0u);
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
    have_result = __all_sync(0xffffffffu, mbar_wait(tmem_full, 0, abort_flag));
    if (!have_result && lane == 0) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
  }

  const int slot_bytes = MP * cols * 4;  // one source CTA's slice, FP32 [MP][cols]
  const uint32_t base = smem_addr(exchange);
  cluster_wait();  // every receive barrier of the cluster is armed
  if (warp >= 2 && have_result) {
    // ---- TMEM -> the owner's slot y (asynchronous stores counted on its receive barrier) ----
    tc_fence_after_sync();
    const int quarter = warp & 3;
    const int nl = quarter * 32 + static_cast<int>(lane);  // this lane's column of the tile
    const int owner = nl / cols;
    const uint32_t dst = map_to_rank(base + y * slot_bytes + (nl - owner * cols) * 4, static_cast<uint32_t>(owner));
    const uint32_t owner_bar = map_to_rank(smem_addr(recv_bar), static_cast<uint32_t>(owner));
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr int kChunk = MP >= 32 ? 32 : 16;
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
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        if (c0 + j < args.m) st_async_b32(dst + (c0 + j) * cols * 4, r[j], owner_bar);
      }
    }
  }

  // ---- wait for the 2S slots, sum gate and up in split order, silu(g) * u, BF16 out ----
  const bool arrived = mbar_wait_cluster(recv_bar, 0, abort_flag);
  if (!arrived && threadIdx.x == 64) raise_abort(args.status, abort_flag, kStatusEpilogueTimeout);
  const int quads = own_cols / 4;
  const int items = args.m * quads;
  const bool vec_store = (args.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(args.out) & 7) == 0);
  for (int i = static_cast<int>(threadIdx.x); arrived && i < items; i += static_cast<int>(blockDim.x)) {
    const int m = i / quads, q = i % quads;
    const uint32_t offset = static_cast<uint32_t>((m * cols + q * 4) * 4);
    float4 g = ld_shared_f32x4(base + offset);
    float4 u = ld_shared_f32x4(base + args.splits * slot_bytes + offset);
    for (int s = 1; s < args.splits; ++s) {
      const float4 gs = ld_shared_f32x4(base + s * slot_bytes + offset);
      const float4 us = ld_shared_f32x4(base + (args.splits + s) * slot_bytes + offset);
      g.x += gs.x; g.y += gs.y; g.z += gs.z; g.w += gs.w;
      u.x += us.x; u.y += us.y; u.z += us.z; u.w += us.w;
    }
    const float v[4] = {g.x / (1.0f + expf(-g.x)) * u.x, g.y / (1.0f + expf(-g.y)) * u.y,
                        g.z / (1.0f + expf(-g.z)) * u.z, g.w / (1.0f + expf(-g.w)) * u.w};
    const int n = n0 + y * cols + q * 4;
    __nv_bfloat16* dst = args.out + static_cast<int64_t>(m) * args.ldo + n;
    if (vec_store && n + 3 < args.n) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]);
      const __nv_bfloat162 hi = __floats2bfloat162_rn(v[2], v[3]);
      uint2 packed;
      packed.x = *reinterpret_cast<const uint32_t*>(&lo);
      packed.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(dst) = packed;
    } else {
      for (int j = 0; j < 4 && n + j < args.n; ++j) dst[j] = __float2bfloat16_rn(v[j]);
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, G::kTmemCols);
  }
}

}  // namespace hst
