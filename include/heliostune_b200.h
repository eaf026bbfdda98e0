/*
 * heliostune_b200 -- C ABI of the B200 FP16 matmul path.
 *
 * Plain pointers, 64-bit sizes and strides (in elements), a CUDA stream passed as void*.
 * Every entry point returns HST_OK or an HST_ERR_* code; hst_last_error() gives the message of
 * the calling thread's last failure. No entry point allocates device memory: outputs and
 * workspaces are the caller's (the Python layer allocates them with torch, per call, as the
 * reference does). Launches are asynchronous on the given stream; nothing synchronises.
 *
 * Each GEMM entry point replaces one reference launcher (file:line in mottopanikeiku/heliostune):
 *   hst_matmul_tile        <- heliostune.kernel.matmul                     src/heliostune/kernel.py:83
 *   hst_matmul_persistent  <- heliostune.hopper_kernel.hopper_matmul      src/heliostune/hopper_kernel.py:250
 *   hst_matmul_split_k     <- heliostune.action_expansion._split_k_matmul src/heliostune/action_expansion.py:124
 *   hst_gemm               <- heliostune.action_expansion.launch          src/heliostune/action_expansion.py:176
 *   hst_rmsnorm            <- heliostune_fusion_v2::residual_rmsnorm      src/heliostune/_fusion_gpu.py:76
 *                             (FP16 form without the residual, as BASELINE config 4 measures it)
 *   hst_residual_rmsnorm   <- heliostune_fusion_v2::residual_rmsnorm_w{4,8,16,32}
 *                                                                        src/heliostune/_fusion_gpu.py:49-94
 *   hst_gated_mlp_stream   <- the gated-MLP epilogue suite's candidate    src/heliostune/local_executor.py:1970-1979
 * hst_matmul_stream has no reference counterpart (B200 weight-streaming family, M <= 256).
 */
#ifndef HELIOSTUNE_B200_H_
#define HELIOSTUNE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HST_ABI_VERSION 1

/* Return codes. INVALID and UNSUPPORTED map to ValueError, CUDA and TIMEOUT to RuntimeError. */
#define HST_OK 0
#define HST_ERR_INVALID 1      /* bad shape, stride, pointer or configuration value */
#define HST_ERR_UNSUPPORTED 2  /* a configuration this library has no kernel for */
#define HST_ERR_WORKSPACE 3    /* the workspace given is smaller than hst_gemm_workspace_size */
#define HST_ERR_CUDA 4         /* a CUDA runtime or driver call failed */
#define HST_ERR_TIMEOUT 5      /* a kernel's bounded wait ran out (see hst_status) */

/* Candidate families, as ActionCandidate.family in src/heliostune/action_configs.py:70-77. */
#define HST_FAMILY_TILE 0       /* KernelConfig        -> tcgen05 tile GEMM, one CTA per tile */
#define HST_FAMILY_PERSISTENT 1 /* HopperGemmConfig    -> persistent tcgen05 GEMM, grid = #SMs */
#define HST_FAMILY_SPLIT_K 2    /* SplitKConfig        -> swap-AB split-K + fixed-order reduce */
#define HST_FAMILY_STREAM 3     /* StreamConfig        -> swap-AB weight streaming, M <= 256 */
#define HST_FAMILY_PAIR 4       /* PairConfig          -> CTA-pair (cta_group::2) 256 x N tiles */

/* split_k of the pair family that selects its stream-K schedule (no reference counterpart). */
#define HST_PAIR_STREAM_K (-1)

/* Field names and meaning follow the reference's config dataclasses
 * (configs.py:11-51, configs.py:269-356, action_configs.py:20-59). group_m is ignored by the
 * split-K and stream families; split_k by the tile and persistent families (0 = automatic for
 * the stream family). */
typedef struct hst_gemm_config {
  int32_t family;
  int32_t block_m;
  int32_t block_n;
  int32_t block_k;
  int32_t num_warps;
  int32_t num_stages;
  int32_t group_m;
  int32_t split_k;
} hst_gemm_config;

int hst_abi_version(void);

/* Message of the calling thread's last failed call (empty string if none). */
const char* hst_last_error(void);

/* Number of SMs of a device (148 on a B200). */
int hst_device_sm_count(int device, int* sm_count);

/* Bytes of workspace hst_gemm needs for these operands: FP32 split-K partials, plus packed
 * copies of operands whose layout a TMA tensor map cannot describe (unit inner stride,
 * 16-byte aligned base and row stride). a and b are only inspected for alignment. */
int hst_gemm_workspace_size(const hst_gemm_config* config, const void* a, int64_t a_stride0,
                            int64_t a_stride1, const void* b, int64_t b_stride0,
                            int64_t b_stride1, int64_t m, int64_t n, int64_t k, int device,
                            size_t* bytes);

/* C[m, n] (row stride ldc, unit column stride) = A[m, k] * B[k, n], FP16 in and out, FP32
 * accumulation. A and B may have any strides. Replaces action_expansion.launch. */
int hst_gemm(const hst_gemm_config* config, const void* a, int64_t a_stride0, int64_t a_stride1,
             const void* b, int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc,
             int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
             void* stream);

/* Tile family (kernel.py:83-118). */
int hst_matmul_tile(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_warps,
                    int32_t num_stages, int32_t group_m, const void* a, int64_t a_stride0,
                    int64_t a_stride1, const void* b, int64_t b_stride0, int64_t b_stride1,
                    void* c, int64_t ldc, int64_t m, int64_t n, int64_t k, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Persistent family (hopper_kernel.py:250-290): A and B row-major contiguous, K % 8 == 0 and
 * N % 8 == 0, as the reference requires of its tensor descriptors. */
int hst_matmul_persistent(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_warps,
                          int32_t num_stages, int32_t group_m, const void* a, const void* b,
                          void* c, int64_t m, int64_t n, int64_t k, void* stream);

/* Split-K family (action_expansion.py:124-173): 1 <= m <= 31, any strides; the FP32 partials
 * [split_k][m][n] live in the workspace. */
int hst_matmul_split_k(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_warps,
                       int32_t num_stages, int32_t split_k, const void* a, int64_t a_stride0,
                       int64_t a_stride1, const void* b, int64_t b_stride0, int64_t b_stride1,
                       void* c, int64_t ldc, int64_t m, int64_t n, int64_t k, void* workspace,
                       size_t workspace_bytes, void* stream);

/* B200 weight-streaming family (no reference counterpart): 1 <= m <= 256, block_n 128 or 256
 * columns of C per CTA (256 needs block_m 64 or 128). split_k (1..8; 0 = the count putting the
 * most CTAs in one resident wave) CTAs form a cluster whose partials are summed in split order
 * through distributed shared memory: no workspace for aligned operands. */
int hst_matmul_stream(int32_t block_m, int32_t block_n, int32_t block_k, int32_t num_stages,
                      int32_t split_k,
                      const void* a, int64_t a_stride0, int64_t a_stride1, const void* b,
                      int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc, int64_t m,
                      int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                      void* stream);

/* B200 CTA-pair family (no reference counterpart): clusters of two CTAs computing 256 x block_n
 * tiles (block_n 128, 256, or 512 with block_k 64) with tcgen05.mma.cta_group::2, persistent over
 * the tiles. split_k 2 or 4 (block_n 128 or 256; 0 = automatic when the tiles leave most SMs
 * idle) makes clusters of 2 x split_k CTAs
 * that divide K and sum their partials in split order through distributed shared memory.
 * split_k HST_PAIR_STREAM_K balances a part-filled last wave: the tiles
 * hst_pair_stream_k_tiles names are cut along K into one equal run of K blocks per pair, the
 * rest stay whole; pieces meet through FP32 partial tiles and publication words in the
 * workspace (hst_gemm_workspace_size covers them; no zeroing needed: each launch publishes a
 * value of its own). Calls that share a workspace must not overlap on the GPU. Any strides
 * (packed through the workspace when a TMA tensor map cannot describe them). */
int hst_matmul_pair(int32_t block_n, int32_t block_k, int32_t num_stages, int32_t group_m,
                    int32_t split_k, const void* a, int64_t a_stride0, int64_t a_stride1, const void* b,
                    int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc, int64_t m,
                    int64_t n, int64_t k, void* workspace, size_t workspace_bytes, void* stream);

/* RMSNorm(x; gamma, eps) @ W with the normalisation inside the weight-streaming GEMM (no
 * reference counterpart: the reference runs its RMSNorm op, _fusion_gpu.py:76, then the GEMM).
 * While the main loop streams W, the GEMM rescales each x tile it loads by gamma and sums the
 * squares of its rows; the FP32 results are multiplied by rsqrt(sum / k + eps) per row. Same
 * tiles and split_k as hst_matmul_stream, block_m <= 128; x [m, k] and W [k, n] row-major with
 * 16-byte aligned rows, k % 8 == 0, gamma [k] 16-byte aligned. x is read, never written. */
int hst_rmsnorm_matmul_stream(int32_t block_m, int32_t block_n, int32_t block_k,
                              int32_t num_stages, int32_t split_k, const void* x, int64_t ldx,
                              const void* gamma, float eps, const void* w, int64_t ldw, void* c,
                              int64_t ldc, int64_t m, int64_t n, int64_t k, void* stream);

/* Host-only planning query of the stream-K schedule: how many of `tiles` pair tiles (each
 * k_blocks K blocks deep) are shared out along K over `pairs` persistent pairs (0 = none). */
int hst_pair_stream_k_tiles(int64_t tiles, int64_t k_blocks, int64_t pairs, int64_t* sk_tiles);

/* y[r, :] = fp16((x[r, :] * rsqrt(mean(x[r, :]^2) + eps)) * gamma), FP32 row sum.
 * Replaces the residual RMSNorm op (_fusion_gpu.py:49-94) in the form measured here: FP16,
 * no residual, caller-chosen eps. */
int hst_rmsnorm(const void* x, int64_t ldx, const void* gamma, void* y, int64_t ldy,
                int64_t rows, int64_t hidden, float eps, void* stream);

/* The reference's residual RMSNorm (_fusion_gpu.py:49-73, launched by _fusion_gpu.py:76-94):
 * z = fp32(x) + fp32(residual), y = bf16((z * rsqrt(mean(z^2) + eps)) * gamma), BF16 in and out,
 * FP32 row sum, one CTA of num_warps (1..32) warps per row -- the reference's w4/w8/w16/w32
 * variants are num_warps 4/8/16/32. Row strides in elements. Inputs are never written. */
int hst_residual_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                         const void* gamma, void* y, int64_t ldy, int64_t rows, int64_t hidden,
                         float eps, int32_t num_warps, void* stream);

/* Gated-MLP projection with its epilogue, out = bf16(silu(x Wg^T) * (x Wu^T)), in one
 * weight-streaming launch (replaces the two FP32 matmuls, silu and product of the reference's
 * gated-MLP epilogue suite, local_executor.py:1970-1979). BF16 x [m, k] (row stride ldx), the
 * nn.Linear weights w_gate and w_up [n, k] (row strides ld_gate, ld_up), BF16 out [m, n] (row
 * stride ldo); FP32 accumulation. 1 <= m <= 64 (the decode regime); k and the input row
 * strides multiples of 8 with 16-byte aligned bases. block_m 16, 32 or 64 (0: the smallest
 * >= m), block_k 64 or 128, num_stages the ring depth (0: 4, or 3 where that lets two CTAs
 * share an SM because the grid holds more CTAs than SMs), split_k the K ranges per weight
 * (1, 2, 4; 0: automatic) -- a cluster of 2 x split_k CTAs shares each 128-column tile. */
int hst_gated_mlp_stream(int32_t block_m, int32_t block_k, int32_t num_stages, int32_t split_k,
                         const void* x, int64_t ldx, const void* w_gate, int64_t ld_gate,
                         const void* w_up, int64_t ld_up, void* out, int64_t ldo, int64_t m,
                         int64_t n, int64_t k, void* stream);

/* Peer writes of hst_matmul_pair_fanout: coalesced 16-byte stores from the epilogue warps, or
 * one TMA tensor store per peer of each staged sub-tile. */
#define HST_PEER_STORES 0
#define HST_PEER_BULK 1

/* Fused column-parallel GEMM (no reference counterpart). Rank `rank` of `world` (<= 9) holds
 * A [m, k] and its column slice B_r [k, n_total / world], both row-major contiguous. c_ranks[q]
 * is rank q's full output C [m, n_total] (row-major, ldc = n_total) as mapped into this process
 * (e.g. CUDA IPC); the CTA-pair GEMM writes C_r = A B_r into columns
 * [rank * n_total / world, (rank + 1) * n_total / world) of its own C by TMA and of every peer's
 * C (peer_writes: HST_PEER_STORES or HST_PEER_BULK) as each tile finishes, so the exchange
 * overlaps the GEMM. The caller orders the ranks afterwards (a cross-rank barrier on the stream)
 * before reading C. */
int hst_matmul_pair_fanout(int32_t block_n, int32_t block_k, int32_t num_stages, int32_t group_m,
                           const void* a, const void* b_slice, void* const* c_ranks, int32_t world,
                           int32_t rank, int64_t m, int64_t n_total, int64_t k, int32_t peer_writes,
                           void* stream);

/* Peer mappings for hst_matmul_pair_fanout (CUDA IPC; no multicast objects). hst_ipc_export
 * writes the 64-byte IPC handle of the allocation containing `ptr` and ptr's offset in it;
 * another process opens it with hst_ipc_import (the mapped base) and releases it with
 * hst_ipc_close. */
int hst_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
int hst_ipc_import(const void* handle, void** base_out);
int hst_ipc_close(void* base);

/* Column-parallel assembly (no reference counterpart: the reference has no multi-GPU path).
 * dst[r, p * cols_per_part + c] = src[p][r][c] for the rank-ordered [parts][rows][cols_per_part]
 * chunks an all-gather of per-rank C slices returns; dst has row stride ldd. */
int hst_column_assemble(const void* src, void* dst, int64_t parts, int64_t rows,
                        int64_t cols_per_part, int64_t ldd, void* stream);

/* Cross-rank barrier on a stream, for hst_matmul_pair_fanout's callers (no reference
 * counterpart). words_ranks[q] is rank q's array of 2 * world uint64 barrier words as mapped into
 * this process (hst_ipc_* for the peers), all zero before the first call. One small kernel
 * stores `epoch` into word slot * world + rank of every peer's array and waits until this rank's
 * words slot * world + q have all reached it; `epoch` grows by one per barrier round and the
 * ranks pass the same one. Work enqueued after it on the stream starts once every rank has
 * reached the barrier, and sees what the ranks' earlier kernels wrote. The wait is bounded by
 * limit_ns (0: ten seconds; at most one minute); when it runs out the kernel sets status bit 64
 * and returns. */
int hst_peer_barrier(void* const* words_ranks, int32_t world, int32_t rank, int32_t slot, uint64_t epoch,
                     uint64_t limit_ns, void* stream);

/* Status word of a device: bits set by kernels whose bounded waits ran out (1 producer,
 * 2 UMMA issuer, 4 epilogue, 8 drain, 16 timeout probe, 64 peer barrier). Synchronises the
 * device. clear != 0 resets it afterwards. */
int hst_status(int device, int* bits, int clear);

/* Allocation-free split-K (no counterpart in the reference). For callers that cannot allocate
 * device memory when they call -- a process that reserved the whole GPU up front, or an FFI
 * caller with no device allocator -- but still own A, B and C. The FP32 partials live in a
 * fixed 16 MiB device array inside this library instead of a caller workspace, so nothing is
 * allocated. Same arguments and result as hst_matmul_split_k without the workspace; operands
 * must be row-major with 16-byte aligned rows. Rejects (HST_ERR_INVALID) calls whose
 * splits x M x N partials exceed 4 Mi floats. All calls on a device share the array: calls
 * that overlap on the GPU race and must be serialised. The first call on a device looks up the
 * array's device address; make it before any stream capture. */
int hst_matmul_split_k_noalloc(int32_t block_m, int32_t block_n, int32_t block_k,
                               int32_t num_warps, int32_t num_stages, int32_t split_k,
                               const void* a, int64_t a_stride0, int64_t a_stride1, const void* b,
                               int64_t b_stride0, int64_t b_stride1, void* c, int64_t ldc,
                               int64_t m, int64_t n, int64_t k, void* stream);

/* Test hook for the failure path: launches one CTA that waits on an mbarrier nobody arrives at,
 * bounded by limit_ns; when the bound runs out the kernel sets status bit 16 and returns. */
int hst_probe_wait_timeout(uint64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HELIOSTUNE_B200_H_ */
