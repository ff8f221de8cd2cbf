// Deterministic fp32 transcendentals for the index-deciding stages (ErrorGate score, water-filling
// weights, proxy log-counts).  Each is evaluated in double precision by a fixed sequence of IEEE
// operations written with explicit round-to-nearest intrinsics (no FMA contraction), then rounded
// to fp32 once, so the result is reproducible bit for bit by any IEEE implementation of the same
// sequence:
//   ln(x)  = e*ln2 + 2*atanh(s),  s = (m-1)/(m+1),  m in [sqrt(1/2), sqrt(2)),  odd series to s^27
//   exp(x) = 2^k * exp(r),  r = (x - k*ln2_hi) - k*ln2_lo  (Cody-Waite),  Taylor series to r^17
//   erf(x) = 2/sqrt(pi) * exp(-x^2) * sum_n (2x^2)^n x / (1*3*...*(2n+1))  (Abramowitz & Stegun
//            7.1.6, all terms positive), 1 for x >= 6
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace oa {

__device__ __forceinline__ double pow2d(int k) {  // exact 2^k, -1022 <= k <= 1023
  return __longlong_as_double((long long)(k + 1023) << 52);
}

__device__ __noinline__ double ln_d(double x) {  // x > 0 and normal
  long long bits = __double_as_longlong(x);
  int e = (int)((bits >> 52) & 0x7ff) - 1022;
  double m = __longlong_as_double((bits & 0x000fffffffffffffLL) | 0x3fe0000000000000LL);
  if (m < 0.70710678118654752440) {
    m = __dmul_rn(m, 2.0);
    e = e - 1;
  }
  const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
  const double s2 = __dmul_rn(s, s);
  double term = s, sum = s;
#pragma unroll 1
  for (int k = 1; k <= 13; ++k) {
    term = __dmul_rn(term, s2);
    sum = __dadd_rn(sum, __ddiv_rn(term, (double)(2 * k + 1)));
  }
  return __dadd_rn(__dmul_rn(2.0, sum), __dmul_rn((double)e, 0.69314718055994530942));
}

__device__ __noinline__ double exp_d(double x) {
  if (x < -745.0) return 0.0;
  if (x > 709.0) return __longlong_as_double(0x7ff0000000000000LL);
  const double k = rint(__dmul_rn(x, 1.44269504088896338700));
  const double t1 = __dmul_rn(k, 6.93147180369123816490e-01);
  const double t2 = __dmul_rn(k, 1.90821492927058770002e-10);
  const double r = __dsub_rn(__dsub_rn(x, t1), t2);
  double p = 1.0, term = 1.0;
#pragma unroll 1
  for (int i = 1; i <= 17; ++i) {
    term = __dmul_rn(term, r);
    term = __ddiv_rn(term, (double)i);
    p = __dadd_rn(p, term);
  }
  const int ki = (int)k;
  if (ki < -1022) return 0.0;
  return __dmul_rn(p, pow2d(ki));
}

__device__ __noinline__ double erf_d(double x) {  // x >= 0
  if (x >= 6.0) return 1.0;
  const double x2 = __dmul_rn(x, x);
  const double tx2 = __dmul_rn(2.0, x2);
  double term = x, sum = x;
#pragma unroll 1
  for (int n = 1; n < 400; ++n) {
    term = __dmul_rn(term, tx2);
    term = __ddiv_rn(term, (double)(2 * n + 1));
    sum = __dadd_rn(sum, term);
    if (term < __dmul_rn(sum, 1e-17)) break;
  }
  return __dmul_rn(__dmul_rn(1.1283791670955126, exp_d(-x2)), sum);
}

__device__ __forceinline__ float ln_f(float x) { return __double2float_rn(ln_d((double)x)); }
__device__ __forceinline__ float exp_f(float x) {
  if (x == -INFINITY) return 0.0f;
  return __double2float_rn(exp_d((double)x));
}
__device__ __forceinline__ float erf_f(float x) { return __double2float_rn(erf_d((double)x)); }

}  // namespace oa
