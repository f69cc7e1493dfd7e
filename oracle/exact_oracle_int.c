/*
 * Second CPU restatement of the exact_int8 linear layer -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain C with integer accumulation: no floating point takes part in the dot products. It exists to cross-check
 * oracle/exact_oracle.py, whose dot products are float64 BLAS products (exact only because every partial sum stays
 * below 2^53). Only tests load it (oracle/c_oracle.py builds it with gcc); the product never does.
 *
 *   eo_digitize      follows digitize_torch      (reference: src/vllm_exact/kernels.py:22-39)
 *   eo_exact_linear  follows exact_linear_torch  (reference: src/vllm_exact/kernels.py:89-100)
 *
 * Semantics, per row of x (float32): a = max|x| (or the caller's amax), e = frexp exponent of a (0 when a == 0),
 * sh = F - e, scale = the float32 whose bits are ((sh + 127) << 23) modulo 2^32, q = trunc(x * scale) as int32.
 * F = 14: l = ((q + 128) & 255) - 128, h = (q - l) >> 8, cs = 0. F = 15: l = (q & 255) - 128, h = (q - l - 128) >> 8,
 * cs = sum(256 h + l) wrapped to int32. The product:
 *   tot = 2^16 xh.wh + 2^8 (xh.wl + xl.wh) [+ xl.wl unless truncated] [+ 128 (cx + cw) + 2^14 K when F = 15]
 *   y   = float32(float64(tot) * 2^-(sx + sw)), the power of two built from float64 bits ((e + 1023) << 52).
 * Each digit dot product is accumulated in int32: |d| <= 128, so |sum| <= 2^14 K < 2^31 for K <= 65536.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define EO_MAX_K 65536

static int32_t eo_frexp_exponent(float a) {
  if (!(a > 0.0f)) return 0;
  int e = 0;
  (void)frexpf(a, &e);
  return (int32_t)e;
}

static float eo_pow2_f32(int32_t sh) {
  const uint32_t bits = (uint32_t)((uint64_t)((int64_t)sh + 127) << 23);
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

static double eo_pow2_neg_f64(int64_t s) {
  const uint64_t bits = (uint64_t)(-s + 1023) << 52;
  double d;
  memcpy(&d, &bits, sizeof d);
  return d;
}

/* x: R rows of K floats (row-major). amax: NULL, or R row maxima to use instead of the rows' own. */
int eo_digitize(const float* x, int64_t R, int64_t K, int F, const float* amax, int8_t* h, int8_t* l, int32_t* cs,
                int32_t* sh) {
  if (F != 14 && F != 15) return 1;
  for (int64_t r = 0; r < R; ++r) {
    const float* xr = x + r * K;
    float a = 0.0f;
    if (amax) {
      a = amax[r];
    } else {
      for (int64_t k = 0; k < K; ++k) {
        const float v = fabsf(xr[k]);
        if (v > a) a = v;
      }
    }
    const int32_t s = F - eo_frexp_exponent(a);
    const float scale = eo_pow2_f32(s);
    int64_t sum = 0;
    for (int64_t k = 0; k < K; ++k) {
      const float p = xr[k] * scale;
      const int32_t q = (int32_t)(int64_t)truncf(p);
      int32_t lo, hi;
      if (F == 15) {
        lo = (q & 255) - 128;
        hi = (q - lo - 128) >> 8;
        sum += 256 * (int64_t)hi + lo;
      } else {
        lo = ((q + 128) & 255) - 128;
        hi = (q - lo) >> 8;
      }
      h[r * K + k] = (int8_t)hi;
      l[r * K + k] = (int8_t)lo;
    }
    cs[r] = (F == 15) ? (int32_t)(uint32_t)(uint64_t)sum : 0;
    sh[r] = s;
  }
  return 0;
}

static int32_t eo_dot(const int8_t* a, const int8_t* b, int64_t K) {
  int32_t s = 0;
  for (int64_t k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)b[k];
  return s;
}

/* Digits row-major with leading dimension K; tot (M x N int64) and y (M x N float32) may each be NULL. */
int eo_exact_linear(const int8_t* xh, const int8_t* xl, const int32_t* cx, const int32_t* sx, const int8_t* wh,
                    const int8_t* wl, const int32_t* cw, const int32_t* sw, int64_t M, int64_t N, int64_t K, int F,
                    int trunc, int64_t* tot, float* y) {
  if ((F != 14 && F != 15) || K > EO_MAX_K) return 1;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      const int8_t *ah = xh + m * K, *al = xl + m * K, *bh = wh + n * K, *bl = wl + n * K;
      int64_t t = 65536 * (int64_t)eo_dot(ah, bh, K) + 256 * ((int64_t)eo_dot(ah, bl, K) + eo_dot(al, bh, K));
      if (!trunc) t += eo_dot(al, bl, K);
      if (F == 15) t += 128 * ((int64_t)cx[m] + cw[n]) + 128 * 128 * K;
      if (tot) tot[m * N + n] = t;
      if (y) y[m * N + n] = (float)((double)t * eo_pow2_neg_f64((int64_t)sx[m] + sw[n]));
    }
  }
  return 0;
}
