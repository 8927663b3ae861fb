// Deterministic fp64 exp / log / softplus for the routing scores: the same IEEE operations,
// in the same order, as the CPU oracle's numpy restatement (no fused multiply-add: every
// product and sum is an explicit __dmul_rn / __dadd_rn), so both round identically.
// exp: Cody-Waite reduction x = k ln2 + r (ln2 split in a 32-bit head and a tail), then the
// Taylor series of e^r to degree 17 by Horner. log: u = m 2^e with m in [sqrt(1/2), sqrt(2)),
// log m = 2 atanh(s), s = (m - 1) / (m + 1), the atanh series to s^27. log1p(y) via
// Goldberg's correction log(u) * y / (u - 1), u = 1 + y.
#pragma once

#include <math.h>
#include <stdint.h>

namespace dsv41 {

__device__ __forceinline__ double det_exp(double x) {
  const double kLn2Hi = 0x1.62e42fee00000p-1;
  const double kLn2Lo = 0.6931471805599453 - 0x1.62e42fee00000p-1;
  const double kInvLn2 = 1.4426950408889634;
  const double k = rint(__dmul_rn(x, kInvLn2));
  const double r = __dadd_rn(__dadd_rn(x, -__dmul_rn(k, kLn2Hi)), -__dmul_rn(k, kLn2Lo));
  // 1/n! for n = 17 .. 0
  const double c[18] = {
      1.0 / 355687428096000.0, 1.0 / 20922789888000.0, 1.0 / 1307674368000.0,
      1.0 / 87178291200.0,     1.0 / 6227020800.0,     1.0 / 479001600.0,
      1.0 / 39916800.0,        1.0 / 3628800.0,        1.0 / 362880.0,
      1.0 / 40320.0,           1.0 / 5040.0,           1.0 / 720.0,
      1.0 / 120.0,             1.0 / 24.0,             1.0 / 6.0,
      1.0 / 2.0,               1.0,                    1.0};
  double p = c[0];
#pragma unroll
  for (int i = 1; i < 18; ++i) p = __dadd_rn(__dmul_rn(p, r), c[i]);
  const double two_k = __longlong_as_double(((long long)k + 1023) << 52);
  return __dmul_rn(p, two_k);
}

__device__ __forceinline__ double det_log(double u) {
  const long long kSqrtHalf = 0x3FE6A09E667F3BCDLL;
  long long bits = __double_as_longlong(u);
  long long e = (bits >> 52) - 1023;
  long long mb = (bits & 0x000FFFFFFFFFFFFFLL) | 0x3FF0000000000000LL;
  if (mb > kSqrtHalf + (1LL << 52)) {
    mb -= (1LL << 52);
    e += 1;
  }
  const double m = __longlong_as_double(mb);
  const double s = __ddiv_rn(__dadd_rn(m, -1.0), __dadd_rn(m, 1.0));
  const double s2 = __dmul_rn(s, s);
  // 1/(2n+1) for n = 13 .. 0
  double p = 1.0 / 27.0;
  const double c[13] = {1.0 / 25.0, 1.0 / 23.0, 1.0 / 21.0, 1.0 / 19.0, 1.0 / 17.0,
                        1.0 / 15.0, 1.0 / 13.0, 1.0 / 11.0, 1.0 / 9.0,  1.0 / 7.0,
                        1.0 / 5.0,  1.0 / 3.0,  1.0};
#pragma unroll
  for (int i = 0; i < 13; ++i) p = __dadd_rn(__dmul_rn(p, s2), c[i]);
  return __dadd_rn(__dmul_rn((double)e, 0.6931471805599453), __dmul_rn(__dmul_rn(2.0, s), p));
}

// softplus(x) in fp64 for x <= 20.
__device__ __forceinline__ double det_softplus(double x) {
  const double y = det_exp(fmax(x, -700.0));
  const double u = __dadd_rn(1.0, y);
  const double d = __dadd_rn(u, -1.0);
  if (d == 0.0) return y;
  return __dmul_rn(det_log(u), __ddiv_rn(y, d));
}

// The sqrtsoftplus routing score of an fp32 logit (NaN stays NaN).
__device__ __forceinline__ float route_score(float x) {
  if (isnan(x)) return x;
  const float sp = x > 20.0f ? x : (float)det_softplus((double)x);
  return __fsqrt_rn(sp);
}

}  // namespace dsv41
