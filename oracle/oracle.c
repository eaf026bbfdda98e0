/*
 * CPU oracle of the FP16 matmul path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only the tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this file's
 * library, and only as the checker; the product path never calls it.
 *
 * Restated from the reference (mottopanikeiku/heliostune):
 *   hst_oracle_gemm        the FP32 check value torch.mm(a, b, out_dtype=float32) with TF32 off
 *                          (src/heliostune/action_expansion.py:206-211): products of FP16
 *                          values are exact in FP64, summed in FP64, rounded once to FP32.
 *   hst_oracle_gemm_splitk the split-K algorithm (src/heliostune/action_expansion.py:56-121):
 *                          contiguous BK-aligned K intervals, tiles_per_split =
 *                          cdiv(cdiv(K, BK), S) (:79-80); each split accumulates in FP32; the
 *                          S partials are summed in FP32 in split order and narrowed once to FP16.
 *   hst_oracle_rmsnorm     the eager formula of src/heliostune/local_executor.py:1982-1985:
 *                          z = x + residual (FP32 sum; no residual in the FP16 form measured
 *                          here), y = cast((z * rsqrt(mean(z^2) + eps)) * gamma), the row sum in
 *                          FP64 and the output rounded to FP16 or BF16.
 * Conversions are IEEE round-to-nearest-even, written out from the format definitions.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  float out;
  if (exp == 0) {
    /* zero or subnormal: man * 2^-24 */
    out = ldexpf((float)man, -24);
    if (sign) out = -out;
    return out;
  }
  uint32_t bits;
  if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  memcpy(&out, &bits, sizeof(out));
  return out;
}

/* Round a finite or infinite double to the nearest FP16 value (ties to even). */
static uint16_t f64_to_f16(double v) {
  if (isnan(v)) return 0x7E00u;
  uint16_t sign = signbit(v) ? 0x8000u : 0u;
  double a = fabs(v);
  if (a >= 65520.0) return sign | 0x7C00u; /* rounds to infinity */
  if (a < ldexp(1.0, -25)) {
    /* below half the smallest subnormal; exactly half rounds to zero (even) */
    return sign;
  }
  int e;
  frexp(a, &e); /* a = f * 2^e, f in [0.5, 1) */
  int exp_unbiased = e - 1;
  double quantum = exp_unbiased < -14 ? ldexp(1.0, -24) : ldexp(1.0, exp_unbiased - 10);
  double q = a / quantum;
  double r = nearbyint(q); /* default rounding mode: nearest, ties to even */
  double rounded = r * quantum;
  if (rounded >= 65520.0) return sign | 0x7C00u;
  /* re-encode */
  if (rounded < ldexp(1.0, -14)) {
    return sign | (uint16_t)(rounded / ldexp(1.0, -24));
  }
  frexp(rounded, &e);
  exp_unbiased = e - 1;
  uint16_t man = (uint16_t)(rounded / ldexp(1.0, exp_unbiased - 10) - 1024.0);
  return sign | (uint16_t)((exp_unbiased + 15) << 10) | man;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t bits;
  memcpy(&bits, &f, sizeof(bits));
  if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x7FFFFFu)) return (uint16_t)((bits >> 16) | 0x40u);
  const uint32_t lsb = (bits >> 16) & 1u;
  bits += 0x7FFFu + lsb;
  return (uint16_t)(bits >> 16);
}

uint16_t hst_oracle_f32_to_f16(float v) { return f64_to_f16((double)v); }
float hst_oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

/* C[m][n] = fp32( sum_k a[m,k] * b[k,n] ) in FP64. Strides in elements. */
void hst_oracle_gemm(const uint16_t* a, int64_t sa0, int64_t sa1, const uint16_t* b, int64_t sb0,
                     int64_t sb1, float* c, int64_t m, int64_t n, int64_t k) {
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      double acc = 0.0;
      for (int64_t p = 0; p < k; ++p) {
        acc += (double)f16_to_f32(a[i * sa0 + p * sa1]) * (double)f16_to_f32(b[p * sb0 + j * sb1]);
      }
      c[i * n + j] = (float)acc;
    }
  }
}

/* The reference split-K algorithm; writes FP16 bit patterns to c[m][n]. */
void hst_oracle_gemm_splitk(const uint16_t* a, int64_t sa0, int64_t sa1, const uint16_t* b,
                            int64_t sb0, int64_t sb1, uint16_t* c, int64_t m, int64_t n, int64_t k,
                            int64_t block_k, int64_t splits) {
  const int64_t k_tiles = (k + block_k - 1) / block_k;
  const int64_t tiles_per_split = (k_tiles + splits - 1) / splits;
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      float total = 0.0f;
      for (int64_t s = 0; s < splits; ++s) {
        float partial = 0.0f;
        const int64_t k0 = s * tiles_per_split * block_k;
        const int64_t k1 = k0 + tiles_per_split * block_k;
        for (int64_t p = k0; p < k1 && p < k; ++p) {
          partial += f16_to_f32(a[i * sa0 + p * sa1]) * f16_to_f32(b[p * sb0 + j * sb1]);
        }
        total = (s == 0) ? partial : total + partial;
      }
      c[i * n + j] = f64_to_f16((double)total);
    }
  }
}

static float bf16_to_f32(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

/* Element i of a row as FP32: z = x (no residual) or z = fp32(x) + fp32(residual), the sum
 * rounded to FP32 as the reference's x.float() + residual.float() rounds it. */
static float row_value(const uint16_t* xr, const uint16_t* rr, int64_t i, int in_bf16) {
  const float v = in_bf16 ? bf16_to_f32(xr[i]) : f16_to_f32(xr[i]);
  if (rr == NULL) return v;
  return v + (in_bf16 ? bf16_to_f32(rr[i]) : f16_to_f32(rr[i]));
}

/* y[r][:] = cast((z * rsqrt(mean(z^2) + eps)) * gamma) with z = x or x + residual (residual may
 * be NULL); out_bf16 selects the output format. */
void hst_oracle_rmsnorm(const uint16_t* x, const uint16_t* residual, const uint16_t* gamma,
                        uint16_t* y, int64_t rows, int64_t hidden, double eps, int in_bf16,
                        int out_bf16) {
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * hidden;
    const uint16_t* rr = residual == NULL ? NULL : residual + r * hidden;
    double ss = 0.0;
    for (int64_t i = 0; i < hidden; ++i) {
      const double v = row_value(xr, rr, i, in_bf16);
      ss += v * v;
    }
    const double inv = 1.0 / sqrt(ss / (double)hidden + eps);
    for (int64_t i = 0; i < hidden; ++i) {
      const double v = row_value(xr, rr, i, in_bf16);
      const double g = in_bf16 ? bf16_to_f32(gamma[i]) : f16_to_f32(gamma[i]);
      const double out = v * inv * g;
      y[r * hidden + i] = out_bf16 ? f32_to_bf16((float)out) : f64_to_f16(out);
    }
  }
}
