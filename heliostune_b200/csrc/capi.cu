// C ABI of heliostune_b200: argument checks, TMA tensor maps, workspace planning and the choice
// of kernel instantiation for each configuration. See include/heliostune_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <random>
#include <cstring>
#include <string>

#include "../../include/heliostune_b200.h"
#include "gemm_gated.cuh"
#include "gemm_pair.cuh"
#include "gemm_stream.cuh"
#include "gemm_stream_cluster.cuh"
#include "gemm_tile.cuh"
#include "rmsnorm.cuh"

namespace hst {
namespace {

// ------------------------------------------------------------------------------------------
// Errors
// ------------------------------------------------------------------------------------------

thread_local std::string t_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_error = buf;
  return code;
}

#define HST_CUDA(call)                                                                   \
  do {                                                                                   \
    cudaError_t err_ = (call);                                                           \
    if (err_ != cudaSuccess)                                                             \
      return fail(HST_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(err_));       \
  } while (0)

#define HST_TRY(call)          \
  do {                                \
    int rc_ = (call);                 \
    if (rc_ != HST_OK) return rc_;    \
  } while (0)

// ------------------------------------------------------------------------------------------
// Per-device state
// ------------------------------------------------------------------------------------------

__device__ int g_status_word;  // OR of StatusBits raised by kernels on this device

constexpr int kMaxDevices = 64;
constexpr int kMaxDynamicSmem = 232448;  // 227 KB per CTA on sm_100
constexpr int kSmemPerSm = 233472;       // 228 KB per SM
constexpr int kSmemReservedPerCta = 1024;

struct DeviceState {
  std::atomic<bool> ready{false};
  int sm_count = 0;
  int* status = nullptr;
};
DeviceState g_devices[kMaxDevices];
std::mutex g_device_mutex;

int device_state(DeviceState** out) {
  int dev = 0;
  HST_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(HST_ERR_INVALID, "device %d out of range", dev);
  DeviceState& s = g_devices[dev];
  if (!s.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (!s.ready.load(std::memory_order_relaxed)) {
      HST_CUDA(cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev));
      HST_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&s.status), g_status_word));
      s.ready.store(true, std::memory_order_release);
    }
  }
  *out = &s;
  return HST_OK;
}

// Raises the dynamic shared-memory limit of a kernel once per device.
template <typename Kernel>
int allow_smem(Kernel kernel, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  HST_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << dev;
  if (!(done_mask.load(std::memory_order_acquire) & bit)) {
    HST_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kMaxDynamicSmem));
    done_mask.fetch_or(bit, std::memory_order_release);
  }
  return HST_OK;
}

// Dynamic shared memory to request so that co-resident CTAs never ask for more than the SM's
// 512 TMEM columns in total (tcgen05.alloc would otherwise stall a CTA until another exits).
int smem_for_tmem(int smem, int tmem_cols) {
  const int max_ctas = 512 / tmem_cols;
  const int by_smem = kSmemPerSm / (smem + kSmemReservedPerCta);
  if (by_smem <= max_ctas) return smem;
  return kSmemPerSm / max_ctas - kSmemReservedPerCta + 1;
}

// ------------------------------------------------------------------------------------------
// TMA tensor maps
// ------------------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_error = cudaSuccess;

int encode_tiled_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_FLOAT16) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    g_encode_error = cudaGetDriverEntryPointByVersion(
        "cuTensorMapEncodeTiled", reinterpret_cast<void**>(&g_encode), 12000, cudaEnableDefault,
        &q);
    if (g_encode_error == cudaSuccess && q != cudaDriverEntryPointSuccess) {
      g_encode_error = cudaErrorNotSupported;
    }
  });
  if (g_encode == nullptr) {
    return fail(HST_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s",
                cudaGetErrorString(g_encode_error));
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_elems * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = g_encode(map, type, 2, const_cast<void*>(base),
                              dims, strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(HST_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, row stride %llu, box %u x %u",
                static_cast<int>(r), static_cast<unsigned long long>(inner),
                static_cast<unsigned long long>(outer),
                static_cast<unsigned long long>(row_stride_elems), box_inner, box_outer);
  }
  return HST_OK;
}

// ------------------------------------------------------------------------------------------
// Operand layouts
// ------------------------------------------------------------------------------------------

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }

// A row-major view [rows, cols] with element strides (s0, s1).
struct View {
  const __half* ptr;
  int64_t rows, cols, s0, s1;
};

// Whether a TMA tensor map can describe the view directly: unit inner stride, 16-byte aligned
// base and row stride. Strides of size-1 dimensions do not matter.
bool tma_compatible(const View& v) {
  if (reinterpret_cast<uintptr_t>(v.ptr) & 15) return false;
  if (v.cols > 1 && v.s1 != 1) return false;
  if (v.rows > 1 && (v.s0 < v.cols || (v.s0 * 2) % 16 != 0)) return false;
  return true;
}

// Row stride a tensor map is given for a TMA-compatible view.
int64_t tma_row_stride(const View& v) { return v.rows > 1 ? v.s0 : round_up(v.cols, 8); }

__global__ void pack_fp16_kernel(const __half* __restrict__ src, int64_t s0, int64_t s1,
                                 int64_t rows, int64_t cols, __half* __restrict__ dst,
                                 int64_t ld) {
  const int64_t total = rows * ld;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / ld, c = i % ld;
    dst[i] = c < cols ? src[r * s0 + c * s1] : __float2half_rn(0.f);
  }
}

__global__ void copy_fp16_2d_kernel(const __half* __restrict__ src, int64_t lds, int64_t rows,
                                    int64_t cols, __half* __restrict__ dst, int64_t ldd) {
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    dst[r * ldd + c] = src[r * lds + c];
  }
}

__global__ void fill_zero_fp16_kernel(__half* __restrict__ dst, int64_t ldd, int64_t rows,
                                      int64_t cols) {
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    dst[(i / cols) * ldd + i % cols] = __float2half_rn(0.f);
  }
}

// dst[r, p * cols + c] = src[p][r][c]: puts the rank-ordered chunks an all-gather returns into
// the columns of a row-major C. Eight halves (16 bytes) per thread when rows are aligned.
__global__ void column_assemble_kernel(const __half* __restrict__ src, __half* __restrict__ dst,
                                       int64_t parts, int64_t rows, int64_t cols, int64_t ldd,
                                       int vec8) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec8) {
    const int64_t vcols = cols / 8;
    const int64_t total = parts * rows * vcols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += step) {
      const int64_t v = i % vcols, r = (i / vcols) % rows, p = i / (vcols * rows);
      const uint4 x = __ldcs(reinterpret_cast<const uint4*>(src) + i);
      __stcs(reinterpret_cast<uint4*>(dst + r * ldd + p * cols) + v, x);
    }
  } else {
    const int64_t total = parts * rows * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += step) {
      const int64_t c = i % cols, r = (i / cols) % rows, p = i / (cols * rows);
      dst[r * ldd + p * cols + c] = src[i];
    }
  }
}

__global__ void probe_timeout_kernel(int* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on `bar`: the wait must run out and report.
    if (!mbar_wait(&bar, 0, &abort_flag, limit_ns)) atomicOr(status, kStatusProbeTimeout);
  }
}

// Cross-rank barrier of the fused column-parallel GEMM over CUDA-IPC mappings of every rank's
// barrier words ([2 slots][world] u64 each). Thread q < world, q != rank, stores `epoch` into
// slot `slot`, entry `rank`, of rank q's words (release, system scope), then waits for this
// rank's own entry q of that slot to reach `epoch` (acquire). The stores that came before on this
// stream -- the GEMM's peer writes, whose threads fenced at system scope before they exited --
// are visible to a peer once it sees the word. A wait that runs out sets kStatusPeerTimeout.
struct PeerWords {
  unsigned long long* ranks[kMaxPeers + 1];  // rank q's barrier words as mapped here
};

__global__ void peer_barrier_kernel(const __grid_constant__ PeerWords words, int world, int rank, int slot,
                                    unsigned long long epoch, uint64_t limit_ns, int* status) {
  const int q = static_cast<int>(threadIdx.x);
  if (q >= world || q == rank) return;
  st_release_sys_u64(words.ranks[q] + slot * world + rank, epoch);
  if (!wait_at_least_sys_u64(words.ranks[rank] + slot * world + q, epoch, limit_ns))
    atomicOr(status, kStatusPeerTimeout);
}

int grid_for(int64_t total, int sms) {
  const int64_t blocks = cdiv(total, 256);
  return static_cast<int>(blocks < int64_t(sms) * 8 ? (blocks > 0 ? blocks : 1) : int64_t(sms) * 8);
}

// ------------------------------------------------------------------------------------------
// Workspace plan
// ------------------------------------------------------------------------------------------

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Plan {
  int family;
  // tile / persistent
  int um, ma, bn, bk, stages, group_m;
  // split-K / stream
  int nt, mp, splits, kb_per_split;
  // pair stream-K: tiles shared out along K, pairs launched
  int sk_tiles, sk_pairs;
  // workspace offsets (bytes) and sizes
  bool pack_a, pack_b, c_tmp;
  int64_t lda_p, ldb_p, ldc_p;
  size_t off_a, off_b, off_c, off_p, off_sk, total;
};

// Tiles of a pair GEMM to share out along K (stream-K) over `pairs` persistent pairs: none when
// the tiles fill whole waves; all of them when there is less than one wave; otherwise the
// part-filled last wave, together with one full wave when the last wave holds under a quarter
// of the pairs (so that no tile is cut into more than about five pieces). Zero as well when the
// shared K blocks would give a pair fewer than two.
// Stream-K workspace: one 256 x bn FP32 partial tile per pair, then 8 publication words per pair.
size_t pair_partials_bytes(int pairs, int bn) { return size_t(pairs) * 256 * bn * 4; }
size_t pair_stream_k_bytes(int pairs, int bn) {
  return pair_partials_bytes(pairs, bn) + size_t(pairs) * 8 * sizeof(unsigned long long);
}

int64_t pair_stream_k_tiles(int64_t tiles, int64_t k_blocks, int64_t pairs) {
  if (tiles <= 0 || k_blocks <= 0 || pairs <= 0) return 0;
  const int64_t waves = tiles / pairs, rest = tiles % pairs;
  if (rest == 0) return 0;
  int64_t sk = waves == 0 ? tiles : (rest * 4 >= pairs ? rest : rest + pairs);
  if (sk * k_blocks < 2 * pairs) sk = 0;
  return sk;
}

int split_plan(int64_t k, int bk, int requested, int* kb_per_split, int* splits) {
  const int64_t k_blocks = cdiv(k, bk);
  const int64_t per = cdiv(k_blocks, requested);
  *kb_per_split = static_cast<int>(per);
  *splits = static_cast<int>(cdiv(k_blocks, per));
  return HST_OK;
}

// Clusters of `size` CTAs (one CTA per SM) a B200 keeps resident at once, as
// cudaOccupancyMaxActiveClusters reports them for 1..8 CTAs (its GPCs fit 74 pairs but only 33
// clusters of four and 15 of seven or eight), scaled to `sms`.
int64_t resident_clusters(int size, int sms) {
  static constexpr int64_t kPer148[9] = {148, 148, 74, 45, 33, 26, 22, 15, 15};
  return kPer148[size < 1 ? 1 : (size > 8 ? 8 : size)] * sms / 148;
}

int make_plan(const hst_gemm_config* cfg, const View& a, const View& b, int64_t m, int64_t n,
              int64_t k, int sms, Plan* p) {
  if (cfg == nullptr) return fail(HST_ERR_INVALID, "configuration is null");
  *p = Plan{};
  p->family = cfg->family;
  const int bm = cfg->block_m, bn = cfg->block_n, bk = cfg->block_k;
  auto pow2 = [](int v) { return v > 0 && (v & (v - 1)) == 0; };
  if (!pow2(bm) || !pow2(bn) || !pow2(bk) || cfg->num_stages < 1 || cfg->num_warps < 1)
    return fail(HST_ERR_INVALID, "block sizes must be powers of two and stages/warps positive");
  switch (cfg->family) {
    case HST_FAMILY_TILE:
    case HST_FAMILY_PERSISTENT: {
      if (cfg->group_m < 1) return fail(HST_ERR_INVALID, "group_m must be positive");
      if (bm <= 64) {
        p->um = 64;
        p->ma = 1;
      } else if (bm == 128) {
        p->um = 128;
        p->ma = 1;
      } else if (bm == 256) {
        p->um = 128;
        p->ma = 2;
      } else {
        return fail(HST_ERR_UNSUPPORTED, "block_m %d has no B200 tile kernel (max 256)", bm);
      }
      p->bn = bn < 64 ? 64 : bn;
      p->bk = bk < 64 ? 64 : bk;
      if (p->bn > 256 || p->bk > 128 || (p->ma == 2 && p->bn > 128))
        return fail(HST_ERR_UNSUPPORTED, "tile %dx%dx%d has no B200 kernel", bm, bn, bk);
      p->stages = cfg->num_stages < 2 ? 2 : (cfg->num_stages > kMaxStages ? kMaxStages : cfg->num_stages);
      p->group_m = cfg->group_m;
      break;
    }
    case HST_FAMILY_PAIR: {
      if (cfg->group_m < 1) return fail(HST_ERR_INVALID, "group_m must be positive");
      if (bm != 256) return fail(HST_ERR_UNSUPPORTED, "pair tiles have block_m 256");
      if (bn != 128 && bn != 256 && bn != 512)
        return fail(HST_ERR_UNSUPPORTED, "pair block_n must be 128, 256 or 512");
      if (bk != 64 && bk != 128) return fail(HST_ERR_UNSUPPORTED, "pair block_k must be 64 or 128");
      if (bn == 512 && bk != 64) return fail(HST_ERR_UNSUPPORTED, "the 512-wide pair tile has block_k 64");
      if (bn == 512 && cfg->split_k > 1)
        return fail(HST_ERR_UNSUPPORTED, "the 512-wide pair tile has no cluster split-K (use stream-K)");
      if (cfg->split_k < HST_PAIR_STREAM_K || cfg->split_k > 4 || cfg->split_k == 3)
        return fail(HST_ERR_INVALID, "pair split_k must be -1 (stream-K), 0 (automatic), 1, 2 or 4");
      p->um = 128;
      p->ma = 2;
      p->bn = bn;
      p->bk = bk;
      p->stages = cfg->num_stages < 2 ? 2 : (cfg->num_stages > kMaxStages ? kMaxStages : cfg->num_stages);
      p->group_m = cfg->group_m;
      const int64_t tiles = cdiv(m, 256) * cdiv(n, bn);
      const int64_t k_blocks = cdiv(k, bk);
      const int64_t max_pairs = sms / 2;
      p->sk_pairs = static_cast<int>(tiles < max_pairs ? tiles : max_pairs);
      if (cfg->split_k == HST_PAIR_STREAM_K) {
        p->splits = 1;
        p->kb_per_split = static_cast<int>(k_blocks);
        p->sk_tiles = static_cast<int>(pair_stream_k_tiles(tiles, k_blocks, max_pairs));
        if (p->sk_tiles > 0) p->sk_pairs = static_cast<int>(max_pairs);
        break;
      }
      int splits = bn == 512 ? 1 : cfg->split_k;
      if (splits == 0) {
        // Split K while the tiles leave most SMs idle and a wave of (2, S) clusters holds them:
        // a B200 keeps at most 33 clusters of four and 15 of eight CTAs resident.
        splits = 1;
        if (tiles * 4 <= sms && tiles <= resident_clusters(4, sms)) splits = 2;
        if (tiles * 8 <= sms && tiles <= resident_clusters(8, sms)) splits = 4;
      }
      // Each CTA owns at least 64 columns (one TMA-store sub-tile) of the tile.
      while (splits > 1 && (bn / splits < 64 || splits > k_blocks ||
                            cdiv(k_blocks, cdiv(k_blocks, splits)) != splits))
        splits /= 2;
      p->splits = splits;
      p->kb_per_split = static_cast<int>(cdiv(k_blocks, splits));
      break;
    }
    case HST_FAMILY_SPLIT_K: {
      if (m < 1 || m > 31 || n < 1 || k < 1)
        return fail(HST_ERR_INVALID, "split-K requires 1 <= M <= 31 and positive N and K");
      if (cfg->split_k < 2 || !pow2(cfg->split_k))
        return fail(HST_ERR_INVALID, "split_k must be a power of two of at least 2");
      if (bn != 64 && bn != 128)
        return fail(HST_ERR_UNSUPPORTED, "split-K block_n %d has no B200 kernel (64 or 128)", bn);
      p->nt = bn;
      p->mp = m <= 16 ? 16 : 32;
      p->bk = bk <= 64 ? 64 : 128;
      p->stages = cfg->num_stages < 2 ? 2 : (cfg->num_stages > kStreamMaxStages ? kStreamMaxStages : cfg->num_stages);
      split_plan(k, p->bk, cfg->split_k, &p->kb_per_split, &p->splits);
      break;
    }
    case HST_FAMILY_STREAM: {
      if (m < 1 || m > 256 || n < 1 || k < 1)
        return fail(HST_ERR_INVALID, "the stream family requires 1 <= M <= 256 and positive N and K");
      if (bm < 16 || bm > 256 || bm < m)
        return fail(HST_ERR_INVALID, "stream block_m %d must cover M=%lld (16..256)", bm,
                    static_cast<long long>(m));
      if (bn != 128 && bn != 256) return fail(HST_ERR_UNSUPPORTED, "stream block_n must be 128 or 256");
      if (bn == 256 && (bm < 64 || bm > 128))
        return fail(HST_ERR_UNSUPPORTED, "stream block_n 256 needs block_m 64 or 128");
      if (bk != 64 && bk != 128) return fail(HST_ERR_UNSUPPORTED, "stream block_k must be 64 or 128");
      if (cfg->split_k < 0 || cfg->split_k > 8)
        return fail(HST_ERR_INVALID, "stream split_k must be 0 (automatic) or 1..8");
      p->nt = bn;
      p->mp = bm;
      p->bk = bk;
      p->stages = cfg->num_stages < 2 ? 2 : (cfg->num_stages > kStreamMaxStages ? kStreamMaxStages : cfg->num_stages);
      const int64_t k_blocks = cdiv(k, bk);
      int splits = cfg->split_k;
      // Every split must own at least one K block and all splits the same count but the last.
      auto k_splits_ok = [&](int s) { return s <= k_blocks && cdiv(k_blocks, cdiv(k_blocks, s)) == s; };
      if (splits == 0) {
        // The most CTAs in one wave: the S (1..8) with the largest tiles x S whose clusters are
        // all resident at once, the smallest such S on a tie.
        const int64_t n_tiles = cdiv(n, bn);
        splits = 1;
        for (int s = 2; s <= 8; ++s) {
          if (n_tiles <= resident_clusters(s, sms) && k_splits_ok(s) && s * n_tiles > splits * n_tiles)
            splits = s;
        }
      }
      while (splits > 1 && !k_splits_ok(splits)) --splits;
      p->splits = splits;
      p->kb_per_split = static_cast<int>(cdiv(k_blocks, splits));
      break;
    }
    default:
      return fail(HST_ERR_INVALID, "unknown family %d", cfg->family);
  }

  const bool is_stream = p->family == HST_FAMILY_SPLIT_K || p->family == HST_FAMILY_STREAM;
  p->pack_a = !tma_compatible(a);
  p->pack_b = !tma_compatible(b);
  p->lda_p = round_up(k, 8);
  p->ldb_p = round_up(n, 8);
  p->c_tmp = !is_stream && (n % 8 != 0);
  p->ldc_p = round_up(n, 8);
  size_t off = 0;
  p->off_a = off;
  if (p->pack_a) off = align_up(off + size_t(m) * p->lda_p * 2);
  p->off_b = off;
  if (p->pack_b) off = align_up(off + size_t(k) * p->ldb_p * 2);
  p->off_c = off;
  if (p->c_tmp) off = align_up(off + size_t(m) * p->ldc_p * 2);
  p->off_p = off;
  if (p->family == HST_FAMILY_SPLIT_K && p->splits > 1)
    off = align_up(off + size_t(p->splits) * m * n * 4);
  p->off_sk = off;
  if (p->family == HST_FAMILY_PAIR && p->sk_tiles > 0)
    off = align_up(off + pair_stream_k_bytes(p->sk_pairs, p->bn));
  p->total = off;
  return HST_OK;
}

// ------------------------------------------------------------------------------------------
// Tile / persistent launch
// ------------------------------------------------------------------------------------------

struct Operands {
  const __half* a;
  int64_t lda;  // row stride a tensor map can use
  const __half* b;
  int64_t ldb;
  __half* c;
  int64_t ldc;
  int m, n, k;
};

template <int UM, int MA, int BN, int BK>
int launch_tile(const DeviceState& dev, const Operands& o, int stages, int group_m,
                bool persistent, cudaStream_t stream) {
  using S = TileShape<UM, MA, BN, BK>;
  static std::atomic<uint64_t> smem_done{0};
  HST_TRY(allow_smem(tile_gemm_kernel<UM, MA, BN, BK>, smem_done));
  while (stages > 2 && S::smem_bytes(stages) > kMaxDynamicSmem) --stages;
  if (S::smem_bytes(stages) > kMaxDynamicSmem)
    return fail(HST_ERR_UNSUPPORTED, "tile %dx%dx%d does not fit shared memory", UM * MA, BN, BK);
  CUtensorMap ma_, mb_, mc_;
  HST_TRY(encode_tiled_2d(&ma_, o.a, o.k, o.m, o.lda, 64, UM));
  HST_TRY(encode_tiled_2d(&mb_, o.b, o.n, o.k, o.ldb, 64, BK));
  HST_TRY(encode_tiled_2d(&mc_, o.c, o.n, o.m, o.ldc, 64, S::kRowsPerWarp));
  TileArgs args;
  args.m = o.m;
  args.n = o.n;
  args.k = o.k;
  args.tiles_m = static_cast<int>(cdiv(o.m, UM * MA));
  args.tiles_n = static_cast<int>(cdiv(o.n, BN));
  args.num_tiles = args.tiles_m * args.tiles_n;
  args.k_blocks = static_cast<int>(cdiv(o.k, BK));
  args.group_m = group_m;
  args.stages = stages;
  args.status = dev.status;
  const int smem = smem_for_tmem(S::smem_bytes(stages), S::kTmemCols);
  const int per_sm = kSmemPerSm / (smem + kSmemReservedPerCta);
  int grid = args.num_tiles;
  if (persistent) {
    const int slots = dev.sm_count * (per_sm > 0 ? per_sm : 1);
    grid = grid < slots ? grid : slots;
  }
  tile_gemm_kernel<UM, MA, BN, BK><<<grid, kTileThreads, smem, stream>>>(ma_, mb_, mc_, args);
  HST_CUDA(cudaGetLastError());
  return HST_OK;
}

int dispatch_tile(const DeviceState& dev, const Plan& p, const Operands& o, bool persistent,
                  cudaStream_t stream) {
#define HST_TILE_CASE(UM_, MA_, BN_, BK_)                                          \
  if (p.um == UM_ && p.ma == MA_ && p.bn == BN_ && p.bk == BK_)                    \
    return launch_tile<UM_, MA_, BN_, BK_>(dev, o, p.stages, p.group_m, persistent, stream);
  HST_TILE_CASE(64, 1, 64, 64)
  HST_TILE_CASE(64, 1, 128, 64)
  HST_TILE_CASE(64, 1, 256, 64)
  HST_TILE_CASE(64, 1, 64, 128)
  HST_TILE_CASE(64, 1, 128, 128)
  HST_TILE_CASE(128, 1, 64, 64)
  HST_TILE_CASE(128, 1, 128, 64)
  HST_TILE_CASE(128, 1, 256, 64)
  HST_TILE_CASE(128, 1, 64, 128)
  HST_TILE_CASE(128, 1, 128, 128)
  HST_TILE_CASE(128, 1, 256, 128)
  HST_TILE_CASE(128, 2, 64, 64)
  HST_TILE_CASE(128, 2, 128, 64)
  HST_TILE_CASE(128, 2, 64, 128)
  HST_TILE_CASE(128, 2, 128, 128)
#undef HST_TILE_CASE
  return fail(HST_ERR_UNSUPPORTED, "no tile kernel for UMMA M %d x %d atoms, N %d, K %d", p.um,
              p.ma, p.bn, p.bk);
}

// ------------------------------------------------------------------------------------------
// CTA-pair launch
// ------------------------------------------------------------------------------------------

template <int BN, int BK, bool SPLIT>
int launch_pair(const DeviceState& dev, const Operands& o, int stages, int group_m, int splits,
                int kb_per_split, cudaStream_t stream, const PairFanoutArgs* fanout_in = nullptr,
                const PairStreamKArgs* sk_in = nullptr, int sk_pairs = 0) {
  using S = PairShape<BN, BK>;
  static std::atomic<uint64_t> smem_done{0};
  HST_TRY(allow_smem(pair_gemm_kernel<BN, BK, SPLIT>, smem_done));
  while (stages > 2 && S::smem_bytes(stages) > kMaxDynamicSmem) --stages;
  if (SPLIT) {
    // The staged outgoing and the incoming FP32 slices reuse the drained ring.
    const int exchange = 2 * (splits - 1) * 128 * (BN / splits) * 4;
    while (stages * S::kStageBytes < exchange) ++stages;
  }
  if (S::smem_bytes(stages) > kMaxDynamicSmem)
    return fail(HST_ERR_UNSUPPORTED, "pair tile 256x%dx%d does not fit shared memory", BN, BK);
  CUtensorMap ma_, mb_, mc_;
  HST_TRY(encode_tiled_2d(&ma_, o.a, o.k, o.m, o.lda, 64, 128));
  HST_TRY(encode_tiled_2d(&mb_, o.b, o.n, o.k, o.ldb, 64, BK));
  HST_TRY(encode_tiled_2d(&mc_, o.c, o.n, o.m, o.ldc, 64, 32));
  TileArgs args;
  args.m = o.m;
  args.n = o.n;
  args.k = o.k;
  args.tiles_m = static_cast<int>(cdiv(o.m, 256));
  args.tiles_n = static_cast<int>(cdiv(o.n, BN));
  args.num_tiles = args.tiles_m * args.tiles_n;
  args.k_blocks = static_cast<int>(cdiv(o.k, BK));
  args.group_m = group_m;
  args.stages = stages;
  args.status = dev.status;
  PairFanoutArgs fanout = {};
  if (fanout_in != nullptr) fanout = *fanout_in;
  PairSplitArgs split_args;
  split_args.splits = splits;
  split_args.kb_per_split = kb_per_split;
  split_args.c = o.c;
  split_args.ldc = o.ldc;
  PairStreamKArgs sk = {};
  if (sk_in != nullptr) sk = *sk_in;
  const int max_pairs = dev.sm_count / 2;
  const int pairs = sk.sk_tiles > 0 ? sk_pairs : (args.num_tiles < max_pairs ? args.num_tiles : max_pairs);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = SPLIT ? dim3(static_cast<unsigned>(2 * args.num_tiles), static_cast<unsigned>(splits))
                     : dim3(static_cast<unsigned>(2 * pairs));
  lc.blockDim = dim3(kTileThreads);
  lc.dynamicSmemBytes = S::smem_bytes(stages);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = SPLIT ? static_cast<unsigned>(splits) : 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  HST_CUDA(cudaLaunchKernelEx(&lc, pair_gemm_kernel<BN, BK, SPLIT>, ma_, mb_, mc_, args, split_args,
                              fanout, sk));
  return HST_OK;
}

// Publication value of a stream-K launch: unique per launch within the process, and started
// from a per-process random value so that words left in reused memory by another process (or
// any other data) match with probability ~2^-64.
unsigned long long next_stream_k_token() {
  static std::atomic<unsigned long long> counter{0};
  static const unsigned long long base = [] {
    std::random_device rd;
    return (static_cast<unsigned long long>(rd()) << 32) ^ rd() ^
           static_cast<unsigned long long>(std::chrono::steady_clock::now().time_since_epoch().count());
  }();
  unsigned long long t = 0;
  while (t == 0) t = base + counter.fetch_add(1, std::memory_order_relaxed);
  return t;
}

int dispatch_pair(const DeviceState& dev, const Plan& p, const Operands& o, uint8_t* ws,
                  cudaStream_t stream) {
  PairStreamKArgs sk = {};
  if (p.sk_tiles > 0) {
    sk.sk_tiles = p.sk_tiles;
    sk.partials = reinterpret_cast<float*>(ws + p.off_sk);
    sk.flags = reinterpret_cast<unsigned long long*>(ws + p.off_sk + pair_partials_bytes(p.sk_pairs, p.bn));
    sk.token = next_stream_k_token();
  }
#define HST_PAIR_CASE(BN_, BK_)                                                                \
  if (p.bn == BN_ && p.bk == BK_) {                                                            \
    if (p.splits > 1)                                                                          \
      return launch_pair<BN_, BK_, true>(dev, o, p.stages, p.group_m, p.splits, p.kb_per_split, \
                                         stream);                                              \
    return launch_pair<BN_, BK_, false>(dev, o, p.stages, p.group_m, 1, 0, stream, nullptr,    \
                                        &sk, p.sk_pairs);                                      \
  }
  HST_PAIR_CASE(256, 64)
  HST_PAIR_CASE(128, 64)
  HST_PAIR_CASE(256, 128)
  HST_PAIR_CASE(128, 128)
#undef HST_PAIR_CASE
  if (p.bn == 512 && p.bk == 64)
    return launch_pair<512, 64, false>(dev, o, p.stages, p.group_m, 1, 0, stream, nullptr, &sk, p.sk_pairs);
  return fail(HST_ERR_UNSUPPORTED, "no pair kernel for N %d, K %d", p.bn, p.bk);
}

// ------------------------------------------------------------------------------------------
// Split-K / stream launch
// ------------------------------------------------------------------------------------------

template <int NT, int MP, int BK>
int launch_stream(const DeviceState& dev, const Operands& o, int stages, int splits,
                  int kb_per_split, float* partials, cudaStream_t stream) {
  using S = StreamShape<NT, MP, BK>;
  static std::atomic<uint64_t> smem_done{0};
  HST_TRY(allow_smem(stream_gemm_kernel<NT, MP, BK>, smem_done));
  while (stages > 2 && S::smem_bytes(stages) > kMaxDynamicSmem) --stages;
  if (S::smem_bytes(stages) > kMaxDynamicSmem)
    return fail(HST_ERR_UNSUPPORTED, "stream tile does not fit shared memory");
  CUtensorMap ma_, mb_;
  HST_TRY(encode_tiled_2d(&ma_, o.a, o.k, o.m, o.lda, 64, MP));
  HST_TRY(encode_tiled_2d(&mb_, o.b, o.n, o.k, o.ldb, 64, BK));
  StreamArgs args;
  args.m = o.m;
  args.n = o.n;
  args.k = o.k;
  args.k_blocks = static_cast<int>(cdiv(o.k, BK));
  args.kb_per_split = kb_per_split;
  args.stages = stages;
  args.status = dev.status;
  args.partials = splits > 1 ? partials : nullptr;
  args.c = o.c;
  args.ldc = o.ldc;
  const int smem = smem_for_tmem(S::smem_bytes(stages), S::kTmemCols);
  const dim3 grid(static_cast<unsigned>(cdiv(o.n, NT)), static_cast<unsigned>(splits));
  stream_gemm_kernel<NT, MP, BK><<<grid, kStreamThreads, smem, stream>>>(ma_, mb_, args);
  HST_CUDA(cudaGetLastError());
  if (splits > 1) {
    const int64_t threads = int64_t(o.m) * cdiv(o.n, 4);
    const bool vector_ok = (o.n % 4 == 0) && (o.ldc % 4 == 0) &&
                           (reinterpret_cast<uintptr_t>(o.c) % 8 == 0);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(static_cast<unsigned>(cdiv(threads, 256)));
    lc.blockDim = dim3(256);
    lc.dynamicSmemBytes = 0;
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    HST_CUDA(cudaLaunchKernelEx(&lc, splitk_reduce_kernel, static_cast<const float*>(partials),
                                o.c, o.ldc, o.m, o.n, splits, vector_ok ? 1 : 0));
  }
  return HST_OK;
}

int dispatch_stream(const DeviceState& dev, const Plan& p, const Operands& o, float* partials,
                    cudaStream_t stream) {
#define HST_STREAM_CASE(NT_, MP_, BK_)                                                  \
  if (p.nt == NT_ && p.mp == MP_ && p.bk == BK_)                                        \
    return launch_stream<NT_, MP_, BK_>(dev, o, p.stages, p.splits, p.kb_per_split, partials, \
                                        stream);
  HST_STREAM_CASE(64, 16, 64)
  HST_STREAM_CASE(64, 32, 64)
  HST_STREAM_CASE(128, 16, 64)
  HST_STREAM_CASE(128, 32, 64)
  HST_STREAM_CASE(128, 64, 64)
  HST_STREAM_CASE(128, 128, 64)
  HST_STREAM_CASE(128, 256, 64)
  HST_STREAM_CASE(128, 16, 128)
  HST_STREAM_CASE(128, 32, 128)
  HST_STREAM_CASE(128, 64, 128)
  HST_STREAM_CASE(128, 128, 128)
  HST_STREAM_CASE(128, 256, 128)
#undef HST_STREAM_CASE
  return fail(HST_ERR_UNSUPPORTED, "no stream kernel for UMMA M %d, N %d, K %d", p.nt, p.mp,
              p.bk);
}

// RMSNorm prologue of the stream family: gamma [k] (null = plain GEMM) and eps.
struct RowNorm {
  const __half* gamma = nullptr;
  float eps = 0.f;
};

template <int NA, int MP, int BK, bool NORM>
int launch_stream_cluster(const DeviceState& dev, const Operands& o, int stages, int splits,
                          int kb_per_split, cudaStream_t stream, const RowNorm& norm = RowNorm{}) {
  using S = ClusterStreamShape<NA, MP, BK>;
  static std::atomic<uint64_t> smem_done{0};
  HST_TRY(allow_smem(stream_cluster_kernel<NA, MP, BK, NORM>, smem_done));
  // Exchange slots beside the ring when at least two stages still fit (asynchronous pushes), or
  // when they cost no stage at all (plain remote stores: each CTA then pushes as soon as its own
  // accumulator is complete instead of after the cluster's slowest main loop); else inside it.
  constexpr bool nrm = NORM;
  int early_stages = stages;
  while (early_stages > 2 && S::smem_bytes(early_stages, splits, true, nrm) > kMaxDynamicSmem) --early_stages;
  int ring_stages = stages;
  while (ring_stages > 2 && S::smem_bytes(ring_stages, splits, false, nrm) > kMaxDynamicSmem) --ring_stages;
  const bool early = splits > 1 && S::smem_bytes(early_stages, splits, true, nrm) <= kMaxDynamicSmem &&
                     (S::kAsyncPush || early_stages >= ring_stages);
  if (early) stages = early_stages;
  while (stages > 2 && S::smem_bytes(stages, splits, early, nrm) > kMaxDynamicSmem) --stages;
  if (S::smem_bytes(stages, splits, early, nrm) > kMaxDynamicSmem)
    return fail(HST_ERR_UNSUPPORTED, "stream tile does not fit shared memory");
  CUtensorMap ma_, mb_;
  HST_TRY(encode_tiled_2d(&ma_, o.a, o.k, o.m, o.lda, 64, MP));
  HST_TRY(encode_tiled_2d(&mb_, o.b, o.n, o.k, o.ldb, 64, BK));
  ClusterStreamArgs args;
  args.m = o.m;
  args.n = o.n;
  args.k = o.k;
  args.k_blocks = static_cast<int>(cdiv(o.k, BK));
  args.kb_per_split = kb_per_split;
  args.splits = splits;
  args.stages = stages;
  args.early = early ? 1 : 0;
  args.eps = norm.eps;
  args.gamma = norm.gamma;
  args.status = dev.status;
  args.c = o.c;
  args.ldc = o.ldc;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(cdiv(o.n, S::kNT)), static_cast<unsigned>(splits));
  lc.blockDim = dim3(kStreamThreads);
  lc.dynamicSmemBytes = smem_for_tmem(S::smem_bytes(stages, splits, early, nrm), S::kTmemCols);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = splits > 1 ? 1 : 0;
  HST_CUDA(cudaLaunchKernelEx(&lc, stream_cluster_kernel<NA, MP, BK, NORM>, ma_, mb_, args));
  return HST_OK;
}

// The plain kernel, or its RMSNorm-prologue instantiation when `norm` carries a gamma.
template <int NA, int MP, int BK>
int launch_stream_either(const DeviceState& dev, const Plan& p, const Operands& o,
                         cudaStream_t stream, const RowNorm& norm) {
  if (norm.gamma == nullptr)
    return launch_stream_cluster<NA, MP, BK, false>(dev, o, p.stages, p.splits, p.kb_per_split, stream);
  if constexpr (MP <= 128) {
    return launch_stream_cluster<NA, MP, BK, true>(dev, o, p.stages, p.splits, p.kb_per_split, stream, norm);
  } else {
    return fail(HST_ERR_UNSUPPORTED, "the RMSNorm prologue covers up to 128 rows");
  }
}

int dispatch_stream_cluster(const DeviceState& dev, const Plan& p, const Operands& o,
                            cudaStream_t stream, const RowNorm& norm = RowNorm{}) {
#define HST_CLUSTER_CASE(NA_, MP_, BK_)                        \
  if (p.nt == 128 * NA_ && p.mp == MP_ && p.bk == BK_)         \
    return launch_stream_either<NA_, MP_, BK_>(dev, p, o, stream, norm);
  HST_CLUSTER_CASE(1, 16, 64)
  HST_CLUSTER_CASE(1, 32, 64)
  HST_CLUSTER_CASE(1, 64, 64)
  HST_CLUSTER_CASE(1, 128, 64)
  HST_CLUSTER_CASE(1, 256, 64)
  HST_CLUSTER_CASE(1, 16, 128)
  HST_CLUSTER_CASE(1, 32, 128)
  HST_CLUSTER_CASE(1, 64, 128)
  HST_CLUSTER_CASE(1, 128, 128)
  HST_CLUSTER_CASE(1, 256, 128)
  HST_CLUSTER_CASE(2, 64, 64)
  HST_CLUSTER_CASE(2, 128, 64)
  HST_CLUSTER_CASE(2, 64, 128)
  HST_CLUSTER_CASE(2, 128, 128)
#undef HST_CLUSTER_CASE
  return fail(HST_ERR_UNSUPPORTED, "no stream kernel for %d columns, M %d, K %d", p.nt, p.mp, p.bk);
}

// ------------------------------------------------------------------------------------------
// Gated-MLP weight streaming (BF16, K-major weights)
// ------------------------------------------------------------------------------------------

// A BF16 [outer, inner] row-major tensor in 128-byte-swizzled boxes.
int encode_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  return encode_tiled_2d(map, base, inner, outer, row_stride_elems, box_inner, box_outer,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
}

struct GatedProblem {
  const void* x;
  int64_t ldx;
  const void* gate;
  int64_t ld_gate;
  const void* up;
  int64_t ld_up;
  void* out;
  int64_t ldo;
  int m, n, k;
};

// K splits per weight for an automatic request: of 1, 2 and 4, the most whose 2S-CTA clusters
// still all fit one resident wave, counting how many CTAs share an SM at this shared-memory size.
template <int MP, int BK>
int gated_auto_splits(int n, int k, int stages, int sms) {
  using G = GatedShape<MP, BK>;
  const int64_t tiles = cdiv(n, G::kNT);
  const int64_t k_blocks = cdiv(k, BK);
  int best = 1;
  for (int s : {2, 4}) {
    if (k_blocks < s) break;
    const int64_t per_sm = std::max<int64_t>(1, kSmemPerSm / (G::smem_bytes(stages, 2 * s) + kSmemReservedPerCta));
    if (tiles * 2 * s <= per_sm * sms) best = s;
  }
  return best;
}

template <int MP, int BK>
int launch_gated(const DeviceState& dev, const GatedProblem& p, int stages, int splits, cudaStream_t stream) {
  using G = GatedShape<MP, BK>;
  static std::atomic<uint64_t> smem_done{0};
  HST_TRY(allow_smem(gated_stream_kernel<MP, BK>, smem_done));
  const bool auto_stages = stages == 0;
  if (auto_stages) stages = 4;
  if (stages < 2) stages = 2;
  if (stages > kStreamMaxStages) stages = kStreamMaxStages;
  if (splits == 0) splits = gated_auto_splits<MP, BK>(p.n, p.k, stages, dev.sm_count);
  int kb_per_split = 0, eff = 0;
  HST_TRY(split_plan(p.k, BK, splits, &kb_per_split, &eff));
  if (auto_stages) {
    // More CTAs than SMs: a shallower ring that lets two CTAs share an SM beats a second wave.
    const int64_t ctas = cdiv(p.n, G::kNT) * 2 * eff;
    while (ctas > dev.sm_count && stages > 3 && 2 * (G::smem_bytes(stages, 2 * eff) + kSmemReservedPerCta) > kSmemPerSm)
      --stages;
  }
  while (stages > 2 && G::smem_bytes(stages, 2 * eff) > kMaxDynamicSmem) --stages;
  if (G::smem_bytes(stages, 2 * eff) > kMaxDynamicSmem)
    return fail(HST_ERR_UNSUPPORTED, "gated tile does not fit shared memory");
  CUtensorMap mx, mg, mu;
  HST_TRY(encode_bf16_2d(&mx, p.x, p.k, p.m, p.ldx, 64, MP));
  HST_TRY(encode_bf16_2d(&mg, p.gate, p.k, p.n, p.ld_gate, 64, G::kNT));
  HST_TRY(encode_bf16_2d(&mu, p.up, p.k, p.n, p.ld_up, 64, G::kNT));
  GatedStreamArgs args;
  args.m = p.m;
  args.n = p.n;
  args.k = p.k;
  args.k_blocks = static_cast<int>(cdiv(p.k, BK));
  args.kb_per_split = kb_per_split;
  args.splits = eff;
  args.stages = stages;
  args.status = dev.status;
  args.out = static_cast<__nv_bfloat16*>(p.out);
  args.ldo = p.ldo;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(cdiv(p.n, G::kNT)), static_cast<unsigned>(2 * eff));
  lc.blockDim = dim3(kStreamThreads);
  lc.dynamicSmemBytes = smem_for_tmem(G::smem_bytes(stages, 2 * eff), G::kTmemCols);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(2 * eff);
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  HST_CUDA(cudaLaunchKernelEx(&lc, gated_stream_kernel<MP, BK>, mx, mg, mu, args));
  return HST_OK;
}

// ------------------------------------------------------------------------------------------
// Common GEMM driver
// ------------------------------------------------------------------------------------------

int check_problem(const void* a, const void* b, const void* c, int64_t m, int64_t n, int64_t k,
                  int64_t ldc) {
  if (m < 0 || n < 0 || k < 0) return fail(HST_ERR_INVALID, "negative matrix extent");
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return fail(HST_ERR_INVALID, "matrix extent too large");
  if (m > 0 && n > 0) {
    if (c == nullptr) return fail(HST_ERR_INVALID, "output pointer is null");
    if (ldc < n) return fail(HST_ERR_INVALID, "ldc %lld < n %lld", (long long)ldc, (long long)n);
    if (k > 0 && (a == nullptr || b == nullptr))
      return fail(HST_ERR_INVALID, "input pointer is null");
  }
  return HST_OK;
}

// Launches a planned GEMM: zero-fills C when K is 0, packs the operands TMA cannot read in place
// into the workspace, then runs the plan's kernels. `partials_override`, when not null, replaces
// the workspace's split-K partials slot (the allocation-free entry point passes its fixed array).
int run_plan(const DeviceState* dev, const Plan& p, const View& va, const View& vb, __half* cc,
             int64_t ldc, int64_t m, int64_t n, int64_t k, uint8_t* ws, float* partials_override,
             cudaStream_t stream) {
  const int64_t sa0 = va.s0, sa1 = va.s1, sb0 = vb.s0, sb1 = vb.s1;
  if (m == 0 || n == 0) return HST_OK;
  if (k == 0) {
    fill_zero_fp16_kernel<<<grid_for(m * n, dev->sm_count), 256, 0, stream>>>(cc, ldc, m, n);
    HST_CUDA(cudaGetLastError());
    return HST_OK;
  }

  Operands o;
  o.m = static_cast<int>(m);
  o.n = static_cast<int>(n);
  o.k = static_cast<int>(k);
  if (p.pack_a) {
    __half* dst = reinterpret_cast<__half*>(ws + p.off_a);
    pack_fp16_kernel<<<grid_for(m * p.lda_p, dev->sm_count), 256, 0, stream>>>(
        va.ptr, sa0, sa1, m, k, dst, p.lda_p);
    HST_CUDA(cudaGetLastError());
    o.a = dst;
    o.lda = p.lda_p;
  } else {
    o.a = va.ptr;
    o.lda = tma_row_stride(va);
  }
  if (p.pack_b) {
    __half* dst = reinterpret_cast<__half*>(ws + p.off_b);
    pack_fp16_kernel<<<grid_for(k * p.ldb_p, dev->sm_count), 256, 0, stream>>>(
        vb.ptr, sb0, sb1, k, n, dst, p.ldb_p);
    HST_CUDA(cudaGetLastError());
    o.b = dst;
    o.ldb = p.ldb_p;
  } else {
    o.b = vb.ptr;
    o.ldb = tma_row_stride(vb);
  }

  if (p.family == HST_FAMILY_SPLIT_K) {
    o.c = cc;
    o.ldc = ldc;
    float* partials = partials_override != nullptr ? partials_override
                                                   : reinterpret_cast<float*>(ws + p.off_p);
    return dispatch_stream(*dev, p, o, partials, stream);
  }
  if (p.family == HST_FAMILY_STREAM) {
    o.c = cc;
    o.ldc = ldc;
    return dispatch_stream_cluster(*dev, p, o, stream);
  }

  // Tile and persistent kernels store C with TMA: 16-byte aligned rows, else a padded copy.
  const bool direct_c = !p.c_tmp && (ldc % 8 == 0) && (reinterpret_cast<uintptr_t>(cc) % 16 == 0);
  if (direct_c) {
    o.c = cc;
    o.ldc = ldc;
  } else {
    if (!p.c_tmp) {
      // Aligned N but an unaligned destination: fall back to the padded staging buffer. The plan
      // did not reserve it, so ask the caller for more workspace.
      return fail(HST_ERR_INVALID, "output rows must be 16-byte aligned (ldc %% 8 == 0)");
    }
    o.c = reinterpret_cast<__half*>(ws + p.off_c);
    o.ldc = p.ldc_p;
  }
  if (p.family == HST_FAMILY_PAIR) {
    HST_TRY(dispatch_pair(*dev, p, o, ws, stream));
  } else {
    HST_TRY(dispatch_tile(*dev, p, o, p.family == HST_FAMILY_PERSISTENT, stream));
  }
  if (!direct_c) {
    copy_fp16_2d_kernel<<<grid_for(m * n, dev->sm_count), 256, 0, stream>>>(o.c, o.ldc, m, n, cc,
                                                                            ldc);
    HST_CUDA(cudaGetLastError());
  }
  return HST_OK;
}

int gemm_impl(const hst_gemm_config* cfg, const void* a, int64_t sa0, int64_t sa1, const void* b,
              int64_t sb0, int64_t sb1, void* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  HST_TRY(check_problem(a, b, c, m, n, k, ldc));
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  const View va{static_cast<const __half*>(a), m, k, sa0, sa1};
  const View vb{static_cast<const __half*>(b), k, n, sb0, sb1};
  Plan p;
  HST_TRY(make_plan(cfg, va, vb, m, n, k, dev->sm_count, &p));
  if (m > 0 && n > 0 && k > 0) {
    if (workspace_bytes < p.total || (p.total > 0 && workspace == nullptr))
      return fail(HST_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu required",
                  workspace_bytes, p.total);
    if (p.total > 0 && (reinterpret_cast<uintptr_t>(workspace) % kAlign) != 0)
      return fail(HST_ERR_INVALID, "workspace must be %zu-byte aligned", kAlign);
  }
  return run_plan(dev, p, va, vb, static_cast<__half*>(c), ldc, m, n, k,
                  static_cast<uint8_t*>(workspace), nullptr, stream);
}

}  // namespace
}  // namespace hst

// ============================================================================================
// extern "C"
// ============================================================================================

using namespace hst;

extern "C" {

int hst_abi_version(void) { return HST_ABI_VERSION; }

const char* hst_last_error(void) { return t_error.c_str(); }

int hst_device_sm_count(int device, int* sm_count) {
  if (sm_count == nullptr) return fail(HST_ERR_INVALID, "sm_count is null");
  HST_CUDA(cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, device));
  return HST_OK;
}

int hst_pair_stream_k_tiles(int64_t tiles, int64_t k_blocks, int64_t pairs, int64_t* sk_tiles) {
  if (sk_tiles == nullptr) return fail(HST_ERR_INVALID, "sk_tiles is null");
  if (tiles < 0 || k_blocks < 0 || pairs < 1)
    return fail(HST_ERR_INVALID, "tiles and k_blocks must be >= 0 and pairs >= 1");
  *sk_tiles = pair_stream_k_tiles(tiles, k_blocks, pairs);
  return HST_OK;
}

int hst_gemm_workspace_size(const hst_gemm_config* config, const void* a, int64_t a_stride0,
                            int64_t a_stride1, const void* b, int64_t b_stride0,
                            int64_t b_stride1, int64_t m, int64_t n, int64_t k, int device,
                            size_t* bytes) {
  if (bytes == nullptr) return fail(HST_ERR_INVALID, "bytes is null");
  int sms = 0;
  HST_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const View va{static_cast<const __half*>(a), m, k, a_stride0, a_stride1};
  const View vb{static_cast<const __half*>(b), k, n, b_stride0, b_stride1};
  Plan p;
  HST_TRY(make_plan(config, va, vb, m, n, k, sms, &p));
  *bytes = (m == 0 || n == 0 || k == 0) ? 0 : p.total;
  return HST_OK;
}

int hst_gemm(const hst_gemm_config* config, const void* a, int64_t a_stride0, int64_t a_stride1,
             const void* b, int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc,
             int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
             void* stream) {
  return gemm_impl(config, a, a_stride0, a_stride1, b, b_stride0, b_stride1, c, ldc, m, n, k,
                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int hst_matmul_tile(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_warps,
                    int32_t num_stages, int32_t group_m, const void* a, int64_t a_stride0,
                    int64_t a_stride1, const void* b, int64_t b_stride0, int64_t b_stride1,
                    void* c, int64_t ldc, int64_t m, int64_t n, int64_t k, void* workspace,
                    size_t workspace_bytes, void* stream) {
  const hst_gemm_config cfg{HST_FAMILY_TILE, block_m, block_n, block_k, num_warps, num_stages,
                            group_m, 0};
  return gemm_impl(&cfg, a, a_stride0, a_stride1, b, b_stride0, b_stride1, c, ldc, m, n, k,
                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int hst_matmul_persistent(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_warps,
                          int32_t num_stages, int32_t group_m, const void* a, const void* b,
                          void* c, int64_t m, int64_t n, int64_t k, void* stream) {
  if (k % 8 != 0 || n % 8 != 0)
    return fail(HST_ERR_INVALID,
                "tensor descriptors require 16-byte aligned leading strides: K=%lld and N=%lld "
                "must both be multiples of 8",
                static_cast<long long>(k), static_cast<long long>(n));
  const hst_gemm_config cfg{HST_FAMILY_PERSISTENT, block_m, block_n, block_k, num_warps,
                            num_stages, group_m, 0};
  return gemm_impl(&cfg, a, k, 1, b, n, 1, c, n, m, n, k, nullptr, 0,
                   static_cast<cudaStream_t>(stream));
}

int hst_matmul_split_k(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_warps,
                       int32_t num_stages, int32_t split_k, const void* a, int64_t a_stride0,
                       int64_t a_stride1, const void* b, int64_t b_stride0, int64_t b_stride1,
                       void* c, int64_t ldc, int64_t m, int64_t n, int64_t k, void* workspace,
                       size_t workspace_bytes, void* stream) {
  const hst_gemm_config cfg{HST_FAMILY_SPLIT_K, block_m, block_n, block_k, num_warps,
                            num_stages, 8, split_k};
  return gemm_impl(&cfg, a, a_stride0, a_stride1, b, b_stride0, b_stride1, c, ldc, m, n, k,
                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int hst_matmul_stream(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_stages,
                      int32_t split_k, const void* a, int64_t a_stride0, int64_t a_stride1, const void* b,
                      int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc, int64_t m,
                      int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                      void* stream) {
  const hst_gemm_config cfg{HST_FAMILY_STREAM, block_m, block_n, block_k, 4, num_stages, 8, split_k};
  return gemm_impl(&cfg, a, a_stride0, a_stride1, b, b_stride0, b_stride1, c, ldc, m, n, k,
                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int hst_rmsnorm_matmul_stream(int32_t block_m, int32_t block_n, int32_t block_k,
                              int32_t num_stages, int32_t split_k, const void* x, int64_t ldx,
                              const void* gamma, float eps, const void* w, int64_t ldw, void* c,
                              int64_t ldc, int64_t m, int64_t n, int64_t k, void* stream) {
  HST_TRY(check_problem(x, w, c, m, n, k, ldc));
  if (gamma == nullptr) return fail(HST_ERR_INVALID, "gamma is null");
  if (block_m > 128) return fail(HST_ERR_UNSUPPORTED, "the RMSNorm prologue needs block_m <= 128");
  if (k % 8 != 0 || (reinterpret_cast<uintptr_t>(gamma) & 15) != 0)
    return fail(HST_ERR_INVALID, "the RMSNorm prologue needs K %% 8 == 0 and a 16-byte aligned gamma");
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  const hst_gemm_config cfg{HST_FAMILY_STREAM, block_m, block_n, block_k, 4, num_stages, 8, split_k};
  const View vx{static_cast<const __half*>(x), m, k, m > 1 ? ldx : k, 1};
  const View vw{static_cast<const __half*>(w), k, n, ldw, 1};
  Plan p;
  HST_TRY(make_plan(&cfg, vx, vw, m, n, k, dev->sm_count, &p));
  if (p.pack_a || p.pack_b)
    return fail(HST_ERR_INVALID, "x and W must be row-major with 16-byte aligned rows");
  if (m == 0 || n == 0) return HST_OK;
  Operands o;
  o.m = static_cast<int>(m);
  o.n = static_cast<int>(n);
  o.k = static_cast<int>(k);
  o.a = vx.ptr;
  o.lda = tma_row_stride(vx);
  o.b = vw.ptr;
  o.ldb = tma_row_stride(vw);
  o.c = static_cast<__half*>(c);
  o.ldc = ldc;
  RowNorm norm;
  norm.gamma = static_cast<const __half*>(gamma);
  norm.eps = eps;
  return dispatch_stream_cluster(*dev, p, o, static_cast<cudaStream_t>(stream), norm);
}

int hst_matmul_pair(int32_t block_n, int32_t block_k, int32_t num_stages, int32_t group_m,
                    int32_t split_k, const void* a, int64_t a_stride0, int64_t a_stride1, const void* b,
                    int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc, int64_t m,
                    int64_t n, int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  const hst_gemm_config cfg{HST_FAMILY_PAIR, 256, block_n, block_k, 4, num_stages, group_m,
                            split_k};
  return gemm_impl(&cfg, a, a_stride0, a_stride1, b, b_stride0, b_stride1, c, ldc, m, n, k,
                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int hst_matmul_pair_fanout(int32_t block_n, int32_t block_k, int32_t num_stages, int32_t group_m,
                           const void* a, const void* b_slice, void* const* c_ranks, int32_t world,
                           int32_t rank, int64_t m, int64_t n_total, int64_t k, int32_t peer_writes,
                           void* stream) {
  if (peer_writes != HST_PEER_STORES && peer_writes != HST_PEER_BULK)
    return fail(HST_ERR_INVALID, "peer_writes must be HST_PEER_STORES or HST_PEER_BULK");
  if (world < 1 || world > kMaxPeers + 1 || rank < 0 || rank >= world)
    return fail(HST_ERR_INVALID, "world %d / rank %d out of range (at most %d ranks)", world, rank,
                kMaxPeers + 1);
  if (n_total % world != 0) return fail(HST_ERR_INVALID, "N must split evenly over the ranks");
  const int64_t cols = n_total / world;
  if (cols % 8 != 0 || k % 8 != 0)
    return fail(HST_ERR_INVALID, "the column slice and K must be multiples of 8");
  if (c_ranks == nullptr || a == nullptr || b_slice == nullptr)
    return fail(HST_ERR_INVALID, "null pointer");
  HST_TRY(check_problem(a, b_slice, c_ranks[rank], m, cols, k, n_total));
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  const hst_gemm_config cfg{HST_FAMILY_PAIR, 256, block_n, block_k, 4, num_stages, group_m, 1};
  const View va{static_cast<const __half*>(a), m, k, k, 1};
  const View vb{static_cast<const __half*>(b_slice), k, cols, cols, 1};
  Plan p;
  HST_TRY(make_plan(&cfg, va, vb, m, cols, k, dev->sm_count, &p));
  if (p.pack_a || p.pack_b) return fail(HST_ERR_INVALID, "operands must be 16-byte aligned row-major");
  if (m == 0) return HST_OK;
  PairFanoutArgs fanout = {};
  fanout.ldc = n_total;
  // Peers in the order rank + 1, rank + 2, ...: at any moment the ranks write to different peers.
  for (int j = 1; j < world; ++j) {
    const int q = (rank + j) % world;
    if (c_ranks[q] == nullptr) return fail(HST_ERR_INVALID, "null peer output");
    __half* slice = static_cast<__half*>(c_ranks[q]) + rank * cols;
    if (peer_writes == HST_PEER_STORES) {
      fanout.peers[fanout.count++] = reinterpret_cast<uint64_t>(slice);
    } else {
      if ((reinterpret_cast<uintptr_t>(slice) & 15) != 0) return fail(HST_ERR_INVALID, "peer output rows must be 16-byte aligned");
      HST_TRY(encode_tiled_2d(&fanout.peer_maps[fanout.bulk_count++], slice, cols, m, n_total, 64, 32));
    }
  }
  Operands o;
  o.m = static_cast<int>(m);
  o.n = static_cast<int>(cols);
  o.k = static_cast<int>(k);
  o.a = va.ptr;
  o.lda = k;
  o.b = vb.ptr;
  o.ldb = cols;
  o.c = static_cast<__half*>(c_ranks[rank]) + rank * cols;
  o.ldc = n_total;
  if ((reinterpret_cast<uintptr_t>(o.c) & 15) != 0 || n_total % 8 != 0)
    return fail(HST_ERR_INVALID, "output rows must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.bn == 256 && p.bk == 64) return launch_pair<256, 64, false>(*dev, o, p.stages, p.group_m, 1, 0, s, &fanout);
  if (p.bn == 128 && p.bk == 64) return launch_pair<128, 64, false>(*dev, o, p.stages, p.group_m, 1, 0, s, &fanout);
  if (p.bn == 256 && p.bk == 128) return launch_pair<256, 128, false>(*dev, o, p.stages, p.group_m, 1, 0, s, &fanout);
  if (p.bn == 128 && p.bk == 128) return launch_pair<128, 128, false>(*dev, o, p.stages, p.group_m, 1, 0, s, &fanout);
  if (p.bn == 512 && p.bk == 64) return launch_pair<512, 64, false>(*dev, o, p.stages, p.group_m, 1, 0, s, &fanout);
  return fail(HST_ERR_UNSUPPORTED, "no pair kernel for N %d, K %d", p.bn, p.bk);
}

int hst_rmsnorm(const void* x, int64_t ldx, const void* gamma, void* y, int64_t ldy,
                int64_t rows, int64_t hidden, float eps, void* stream) {
  if (rows < 0 || hidden < 1) return fail(HST_ERR_INVALID, "rows must be >= 0 and hidden >= 1");
  if (rows > INT32_MAX) return fail(HST_ERR_INVALID, "too many rows");
  if (ldx < hidden || ldy < hidden) return fail(HST_ERR_INVALID, "row strides must be >= hidden");
  if (!(eps >= 0.f)) return fail(HST_ERR_INVALID, "eps must be non-negative");
  if (rows == 0) return HST_OK;
  if (x == nullptr || gamma == nullptr || y == nullptr)
    return fail(HST_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* xp = static_cast<const __half*>(x);
  const __half* gp = static_cast<const __half*>(gamma);
  __half* yp = static_cast<__half*>(y);
  const bool aligned = hidden % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(gamma) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(y) % 16) == 0;
  const int64_t vecs = hidden / 8;
  const int h = static_cast<int>(hidden);
  if (aligned && vecs <= 256 * 16) {
    int chunks = 1;
    while (cdiv(vecs, chunks) > 256) chunks *= 2;
    const int threads = static_cast<int>(round_up(cdiv(vecs, chunks), 32));
    const dim3 grid(static_cast<unsigned>(rows));
    switch (chunks) {
      case 1: rmsnorm_vec_kernel<1><<<grid, threads, 0, s>>>(xp, gp, yp, h, ldx, ldy, eps); break;
      case 2: rmsnorm_vec_kernel<2><<<grid, threads, 0, s>>>(xp, gp, yp, h, ldx, ldy, eps); break;
      case 4: rmsnorm_vec_kernel<4><<<grid, threads, 0, s>>>(xp, gp, yp, h, ldx, ldy, eps); break;
      case 8: rmsnorm_vec_kernel<8><<<grid, threads, 0, s>>>(xp, gp, yp, h, ldx, ldy, eps); break;
      default: rmsnorm_vec_kernel<16><<<grid, threads, 0, s>>>(xp, gp, yp, h, ldx, ldy, eps); break;
    }
  } else {
    rmsnorm_scalar_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(xp, gp, yp, h, ldx, ldy, eps);
  }
  HST_CUDA(cudaGetLastError());
  return HST_OK;
}

int hst_residual_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                         const void* gamma, void* y, int64_t ldy, int64_t rows, int64_t hidden,
                         float eps, int32_t num_warps, void* stream) {
  if (rows < 0 || hidden < 1) return fail(HST_ERR_INVALID, "rows must be >= 0 and hidden >= 1");
  if (rows > INT32_MAX || hidden > INT32_MAX) return fail(HST_ERR_INVALID, "extent too large");
  if (ldx < hidden || ldr < hidden || ldy < hidden)
    return fail(HST_ERR_INVALID, "row strides must be >= hidden");
  if (!(eps >= 0.f)) return fail(HST_ERR_INVALID, "eps must be non-negative");
  if (num_warps < 1 || num_warps > 32)
    return fail(HST_ERR_INVALID, "num_warps %d outside 1..32", num_warps);
  if (rows == 0) return HST_OK;
  if (x == nullptr || residual == nullptr || gamma == nullptr || y == nullptr)
    return fail(HST_ERR_INVALID, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* rp = static_cast<const __nv_bfloat16*>(residual);
  const auto* gp = static_cast<const __nv_bfloat16*>(gamma);
  auto* yp = static_cast<__nv_bfloat16*>(y);
  const int threads = num_warps * 32;
  const int h = static_cast<int>(hidden);
  const bool aligned = hidden % 8 == 0 && ldx % 8 == 0 && ldr % 8 == 0 && ldy % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(residual) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(gamma) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(y) % 16) == 0;
  const int64_t vecs = hidden / 8;
  const dim3 grid(static_cast<unsigned>(rows));
  int chunks = 1;
  while (chunks < 16 && int64_t(threads) * chunks < vecs) chunks *= 2;
  if (aligned && int64_t(threads) * chunks >= vecs && threads <= residual_rmsnorm_max_threads(chunks)) {
    switch (chunks) {
      case 1: residual_rmsnorm_bf16_kernel<1><<<grid, threads, 0, s>>>(xp, rp, gp, yp, h, ldx, ldr, ldy, eps); break;
      case 2: residual_rmsnorm_bf16_kernel<2><<<grid, threads, 0, s>>>(xp, rp, gp, yp, h, ldx, ldr, ldy, eps); break;
      case 4: residual_rmsnorm_bf16_kernel<4><<<grid, threads, 0, s>>>(xp, rp, gp, yp, h, ldx, ldr, ldy, eps); break;
      case 8: residual_rmsnorm_bf16_kernel<8><<<grid, threads, 0, s>>>(xp, rp, gp, yp, h, ldx, ldr, ldy, eps); break;
      default: residual_rmsnorm_bf16_kernel<16><<<grid, threads, 0, s>>>(xp, rp, gp, yp, h, ldx, ldr, ldy, eps); break;
    }
  } else {
    residual_rmsnorm_bf16_scalar_kernel<<<grid, threads, 0, s>>>(xp, rp, gp, yp, h, ldx, ldr, ldy, eps);
  }
  HST_CUDA(cudaGetLastError());
  return HST_OK;
}

int hst_gated_mlp_stream(int32_t block_m, int32_t block_k, int32_t num_stages, int32_t split_k,
                         const void* x, int64_t ldx, const void* w_gate, int64_t ld_gate,
                         const void* w_up, int64_t ld_up, void* out, int64_t ldo, int64_t m,
                         int64_t n, int64_t k, void* stream) {
  if (m < 1 || m > 64) return fail(HST_ERR_INVALID, "the gated MLP stream kernel needs 1 <= M <= 64 (got %lld)", (long long)m);
  if (n < 1 || k < 1 || n > INT32_MAX / 2 || k > INT32_MAX / 2) return fail(HST_ERR_INVALID, "bad N or K");
  if (block_m == 0) block_m = m <= 16 ? 16 : (m <= 32 ? 32 : 64);
  if ((block_m != 16 && block_m != 32 && block_m != 64) || m > block_m)
    return fail(HST_ERR_INVALID, "block_m must be 16, 32 or 64 and at least M");
  if (block_k != 64 && block_k != 128) return fail(HST_ERR_INVALID, "block_k must be 64 or 128");
  if (split_k != 0 && split_k != 1 && split_k != 2 && split_k != 4)
    return fail(HST_ERR_INVALID, "split_k must be 0 (automatic), 1, 2 or 4");
  if (num_stages < 0 || num_stages > kStreamMaxStages) return fail(HST_ERR_INVALID, "num_stages outside 0..%d", kStreamMaxStages);
  if (x == nullptr || w_gate == nullptr || w_up == nullptr || out == nullptr) return fail(HST_ERR_INVALID, "null pointer");
  if (k % 8 != 0 || ldx % 8 != 0 || ld_gate % 8 != 0 || ld_up % 8 != 0 || ldx < k || ld_gate < k || ld_up < k ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w_gate) & 15) ||
      (reinterpret_cast<uintptr_t>(w_up) & 15))
    return fail(HST_ERR_INVALID, "x and the weights must be row-major with 16-byte aligned rows (K and leading dimensions multiples of 8)");
  if (ldo < n) return fail(HST_ERR_INVALID, "ldo < N");
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  const GatedProblem p{x, ldx, w_gate, ld_gate, w_up, ld_up, out, ldo, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k)};
  const int stages = num_stages;  // 0: automatic
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define HST_GATED_CASE(MP_, BK_) \
  if (block_m == MP_ && block_k == BK_) return launch_gated<MP_, BK_>(*dev, p, stages, split_k, s);
  HST_GATED_CASE(16, 64)
  HST_GATED_CASE(32, 64)
  HST_GATED_CASE(64, 64)
  HST_GATED_CASE(16, 128)
  HST_GATED_CASE(32, 128)
  HST_GATED_CASE(64, 128)
#undef HST_GATED_CASE
  return fail(HST_ERR_UNSUPPORTED, "no gated kernel for block_m %d, block_k %d", block_m, block_k);
}

int hst_column_assemble(const void* src, void* dst, int64_t parts, int64_t rows,
                        int64_t cols_per_part, int64_t ldd, void* stream) {
  if (parts < 1 || rows < 0 || cols_per_part < 0) return fail(HST_ERR_INVALID, "negative extent");
  if (ldd < parts * cols_per_part) return fail(HST_ERR_INVALID, "ldd smaller than parts x cols");
  if (rows == 0 || cols_per_part == 0) return HST_OK;
  if (src == nullptr || dst == nullptr) return fail(HST_ERR_INVALID, "null pointer");
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  const bool vec8 = cols_per_part % 8 == 0 && ldd % 8 == 0 &&
                    reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(dst) % 16 == 0;
  const int64_t work = parts * rows * (vec8 ? cols_per_part / 8 : cols_per_part);
  column_assemble_kernel<<<grid_for(work, dev->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(src), static_cast<__half*>(dst), parts, rows, cols_per_part, ldd,
      vec8 ? 1 : 0);
  HST_CUDA(cudaGetLastError());
  return HST_OK;
}

// ---- peer mappings for the fused column-parallel GEMM (CUDA IPC, no multicast objects) ----

typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

int hst_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(HST_ERR_INVALID, "null pointer");
  static PfnMemGetAddressRange get_range = nullptr;
  if (get_range == nullptr) {
    cudaDriverEntryPointQueryResult q;
    HST_CUDA(cudaGetDriverEntryPointByVersion("cuMemGetAddressRange",
                                              reinterpret_cast<void**>(&get_range), 12000,
                                              cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || get_range == nullptr)
      return fail(HST_ERR_CUDA, "cuMemGetAddressRange unavailable");
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(HST_ERR_CUDA, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t handle;
  HST_CUDA(cudaIpcGetMemHandle(&handle, reinterpret_cast<void*>(base)));
  memcpy(handle_out, &handle, sizeof(handle));
  *offset_out = reinterpret_cast<uint64_t>(ptr) - static_cast<uint64_t>(base);
  return HST_OK;
}

int hst_ipc_import(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return fail(HST_ERR_INVALID, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  HST_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return HST_OK;
}

int hst_ipc_close(void* base) {
  if (base == nullptr) return fail(HST_ERR_INVALID, "null pointer");
  HST_CUDA(cudaIpcCloseMemHandle(base));
  return HST_OK;
}

int hst_peer_barrier(void* const* words_ranks, int32_t world, int32_t rank, int32_t slot, uint64_t epoch,
                     uint64_t limit_ns, void* stream) {
  if (limit_ns == 0) limit_ns = 10000000000ull;
  if (limit_ns > 60000000000ull) return fail(HST_ERR_INVALID, "barrier limit above one minute");
  if (world < 1 || world > kMaxPeers + 1 || rank < 0 || rank >= world)
    return fail(HST_ERR_INVALID, "world %d / rank %d out of range (at most %d ranks)", world, rank, kMaxPeers + 1);
  if (slot != 0 && slot != 1) return fail(HST_ERR_INVALID, "slot must be 0 or 1");
  if (epoch == 0) return fail(HST_ERR_INVALID, "epoch must be >= 1");
  if (words_ranks == nullptr) return fail(HST_ERR_INVALID, "null pointer");
  PeerWords words = {};
  for (int q = 0; q < world; ++q) {
    if (words_ranks[q] == nullptr || (reinterpret_cast<uintptr_t>(words_ranks[q]) & 7) != 0)
      return fail(HST_ERR_INVALID, "barrier words of rank %d null or not 8-byte aligned", q);
    words.ranks[q] = static_cast<unsigned long long*>(words_ranks[q]);
  }
  if (world == 1) return HST_OK;
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(words, world, rank, slot, epoch, limit_ns,
                                                                       dev->status);
  HST_CUDA(cudaGetLastError());
  return HST_OK;
}

int hst_status(int device, int* bits, int clear) {
  if (bits == nullptr) return fail(HST_ERR_INVALID, "bits is null");
  int prev = 0;
  HST_CUDA(cudaGetDevice(&prev));
  HST_CUDA(cudaSetDevice(device));
  DeviceState* dev = nullptr;
  int rc = device_state(&dev);
  if (rc == HST_OK) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(bits, dev->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(dev->status, 0, sizeof(int));
    if (e != cudaSuccess) rc = fail(HST_ERR_CUDA, "reading the status word failed: %s", cudaGetErrorString(e));
  }
  cudaSetDevice(prev);
  return rc;
}

int hst_probe_wait_timeout(uint64_t limit_ns, void* stream) {
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  if (limit_ns > 1000000000ull) return fail(HST_ERR_INVALID, "probe limit above one second");
  probe_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev->status, limit_ns);
  HST_CUDA(cudaGetLastError());
  return HST_OK;
}

}  // extern "C"

// ============================================================================================
// Allocation-free split-K entry point
//
// Some callers cannot allocate device memory at the moment they want a GEMM: a host process
// that reserved the whole GPU up front and hands out no new buffers, an FFI binding of this C
// ABI with no device allocator of its own, or code running where a cudaMalloc would stall or
// be refused. They still own their inputs and outputs; what they cannot provide is the FP32
// split-K partials buffer. This entry point keeps that buffer in a fixed file-scope device
// array instead, so it allocates nothing.
//
// Limits and sharing:
//   * The array holds kNoAllocScratchFloats FP32 values (16 MiB). Every GPU that loads this
//     library keeps it for the life of the process. A call whose effective splits x M x N
//     exceed it is rejected with HST_ERR_INVALID before anything is launched.
//   * Every call on a device uses the same array. Nothing in it has to start at zero: each
//     launch writes every partial it later reads. Two calls whose kernels overlap on the GPU
//     (different streams, or different host threads) race on the array and corrupt each
//     other's results; serialise them.
//   * Operands must already be TMA-describable (unit inner stride, 16-byte aligned base and row
//     stride), because repacking them would need more scratch.
//   * The first call on each device looks up the device address of the array with
//     cudaGetSymbolAddress (the array's name in host code is only a stand-in for it); make that
//     first call before any stream capture.
// ============================================================================================

namespace hst {
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;  // 4 Mi floats = 16 MiB
static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchFloats];

std::atomic<float*> g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mutex;

// Device address of the scratch array on the current device. The first call on a device looks
// it up under the mutex; later calls read the cached address without locking.
int noalloc_scratch(float** out) {
  int dev = 0;
  HST_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(HST_ERR_INVALID, "device %d out of range", dev);
  float* cached = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (cached == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    cached = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (cached == nullptr) {
      void* ptr = nullptr;
      const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_partials);
      if (err != cudaSuccess || ptr == nullptr) {
        return fail(HST_ERR_CUDA, "cudaGetSymbolAddress of the split-K scratch array failed: %s",
                    cudaGetErrorString(err));
      }
      cached = static_cast<float*>(ptr);
      g_noalloc_ptr[dev].store(cached, std::memory_order_release);
    }
  }
  *out = cached;
  return HST_OK;
}

}  // namespace
}  // namespace hst

extern "C" int hst_matmul_split_k_noalloc(int32_t block_m, int32_t block_n, int32_t block_k,
                                          int32_t num_warps, int32_t num_stages, int32_t split_k,
                                          const void* a, int64_t a_stride0, int64_t a_stride1,
                                          const void* b, int64_t b_stride0, int64_t b_stride1,
                                          void* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                                          void* stream) {
  using namespace hst;
  HST_TRY(check_problem(a, b, c, m, n, k, ldc));
  DeviceState* dev = nullptr;
  HST_TRY(device_state(&dev));
  const hst_gemm_config cfg{HST_FAMILY_SPLIT_K, block_m, block_n, block_k, num_warps,
                            num_stages, 8, split_k};
  const View va{static_cast<const __half*>(a), m, k, a_stride0, a_stride1};
  const View vb{static_cast<const __half*>(b), k, n, b_stride0, b_stride1};
  Plan p;
  HST_TRY(make_plan(&cfg, va, vb, m, n, k, dev->sm_count, &p));
  if (p.pack_a || p.pack_b) {
    return fail(HST_ERR_INVALID,
                "the allocation-free split-K needs row-major operands with unit inner stride and "
                "16-byte aligned base and rows");
  }
  const size_t needed = p.splits > 1 ? size_t(p.splits) * size_t(m) * size_t(n) : 0;
  if (needed > kNoAllocScratchFloats) {
    return fail(HST_ERR_INVALID,
                "the allocation-free split-K needs %zu FP32 partials (%d splits x M=%lld x "
                "N=%lld) but its scratch array holds %zu",
                needed, p.splits, static_cast<long long>(m), static_cast<long long>(n),
                kNoAllocScratchFloats);
  }
  float* scratch = nullptr;
  HST_TRY(noalloc_scratch(&scratch));
  return run_plan(dev, p, va, vb, static_cast<__half*>(c), ldc, m, n, k, nullptr, scratch,
                  static_cast<cudaStream_t>(stream));
}
