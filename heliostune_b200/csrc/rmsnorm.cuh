// HBM-bound RMSNorm: y[r, :] = fp16( (x[r, :] * rsqrt(mean(x[r, :]^2) + eps)) * gamma ).
//
// Restates the reference row kernel (_fusion_gpu.py:49-73, eager formula local_executor.py:
// 1982-1985) in the form this build measures: FP16 input without a residual, FP32 row sum,
// eps given by the caller (1e-6 for the measured configuration). One CTA owns one row; each
// thread keeps CHUNKS 16-byte vectors of the row in registers, so x is read from HBM once.
// The row sum is a warp-shuffle tree then a cross-warp pass through shared memory.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace hst {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Sum of `v` over the CTA; every thread receives the total.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < warps; ++w) total += scratch[w];  // fixed order: reproducible
  __syncthreads();
  return total;
}

// hidden % 8 == 0, 16-byte aligned rows; blockDim.x * CHUNKS * 8 >= hidden, blockDim.x <= 256.
template <int CHUNKS>
__global__ void __launch_bounds__(256) rmsnorm_vec_kernel(const __half* __restrict__ x,
                                                           const __half* __restrict__ gamma,
                                                           __half* __restrict__ y, int hidden,
                                                           int64_t ldx, int64_t ldy, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
  const int vecs = hidden >> 3;
  uint4 v[CHUNKS];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < vecs) {
      v[i] = __ldcs(xr + idx);  // streamed: x is read exactly once
      const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < vecs) {
      const uint4 g = __ldg(gr + idx);
      const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
      const __half2* gh = reinterpret_cast<const __half2*>(&g);
      uint4 out;
      uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        const float2 gf = __half22float2(gh[j]);
        o[j] = pack_half2((f.x * inv) * gf.x, (f.y * inv) * gf.y);
      }
      __stcs(yr + idx, out);
    }
  }
}

// Any hidden size and alignment: two passes over the row, scalar loads.
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const __half* __restrict__ x,
                                                             const __half* __restrict__ gamma,
                                                             __half* __restrict__ y, int hidden,
                                                             int64_t ldx, int64_t ldy, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const __half* xr = x + row * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float f = __half2float(xr[i]);
    ss = fmaf(f, f, ss);
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    y[row * ldy + i] = __float2half_rn((__half2float(xr[i]) * inv) * __half2float(gamma[i]));
  }
}

// Residual RMSNorm in the reference's own form (_fusion_gpu.py:49-73; eager formula
// local_executor.py:1982-1985): z = fp32(x) + fp32(r), y = bf16((z * rsqrt(mean(z^2) + eps)) *
// gamma), BF16 in and out, FP32 row sum. One CTA per row; each thread holds CHUNKS 16-byte
// vectors of x and of r (8 BF16 values each), all issued before the first use, so every byte is
// read from HBM once; z is formed again from them for the output (the same FP32 sums). Needs
// hidden % 8 == 0, 16-byte aligned rows, blockDim.x * CHUNKS * 8 >= hidden and blockDim.x <=
// residual_rmsnorm_max_threads(CHUNKS).
__host__ __device__ constexpr int residual_rmsnorm_max_threads(int chunks) {
  return chunks >= 16 ? 256 : chunks >= 8 ? 512 : 1024;
}

__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int CHUNKS>
__global__ void __launch_bounds__(residual_rmsnorm_max_threads(CHUNKS)) residual_rmsnorm_bf16_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r,
    const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ y, int hidden,
    int64_t ldx, int64_t ldr, int64_t ldy, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const uint4* rr = reinterpret_cast<const uint4*>(r + row * ldr);
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
  const int vecs = hidden >> 3;
  uint4 xv[CHUNKS], rv[CHUNKS];
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < vecs) {
      xv[i] = __ldcs(xr + idx);  // streamed: read exactly once
      rv[i] = __ldcs(rr + idx);
    }
  }
  // z of the 8 values of chunk i, pair j: the reference's FP32 sum x + r.
  auto z_pair = [&](int i, int j) {
    const float2 a = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&xv[i])[j]);
    const float2 b = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&rv[i])[j]);
    return make_float2(a.x + b.x, a.y + b.y);
  };
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < vecs) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 z = z_pair(i, j);
        ss = fmaf(z.x, z.x, ss);
        ss = fmaf(z.y, z.y, ss);
      }
    }
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int idx = threadIdx.x + i * blockDim.x;
    if (idx < vecs) {
      const uint4 g = __ldg(gr + idx);
      const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&g);
      uint4 out;
      uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 z = z_pair(i, j);
        const float2 gf = __bfloat1622float2(gh[j]);
        o[j] = pack_bf162((z.x * inv) * gf.x, (z.y * inv) * gf.y);
      }
      __stcs(yr + idx, out);
    }
  }
}

// Any hidden size and alignment: two passes over the row, scalar loads.
__global__ void __launch_bounds__(1024) residual_rmsnorm_bf16_scalar_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r,
    const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ y, int hidden,
    int64_t ldx, int64_t ldr, int64_t ldy, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float zi = __bfloat162float(x[row * ldx + i]) + __bfloat162float(r[row * ldr + i]);
    ss = fmaf(zi, zi, ss);
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float zi = __bfloat162float(x[row * ldx + i]) + __bfloat162float(r[row * ldr + i]);
    y[row * ldy + i] = __float2bfloat16_rn((zi * inv) * __bfloat162float(gamma[i]));
  }
}

}  // namespace hst
