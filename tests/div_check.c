/* Checks the divisions used by the codec kernels.
 *
 * Markstein's correction step: q1 = fma(x - q0*c, r, q0) with q0 = x*r,
 * r = RN(1/c), must equal the IEEE quotient RN(x/c) whenever
 * 2^-100 <= |x| <= 2^120 (outside that range, and for NaN, the kernels take the
 * IEEE division).
 *
 * Brisebarre-Muller multiplication by 1/c: RN(x*ch + RN(x*cl)) with ch = RN(1/c),
 * cl = RN((1 - c*ch) / c) = RN(1/c - ch), must equal RN(x/c) for
 * 2^-98 <= |x| <= 2^120 (the 512-value encode uses it for c = float32(sqrt(512))).
 *
 * Modes:
 *   const <c>           every float32 x, Markstein only (slow: ~40 s)
 *   sig <c>             every significand at exponents -98, -60, -20, 0, 20, 60, 119
 *                       and both signs; prints "<markstein mismatches> <bm mismatches>"
 *   random <n> <seed>   n (x, c) pairs, c in the range of the quantizer's scales and
 *                       x in [-8c, 8c], Markstein only
 * Both methods are invariant under x -> 2^k x while no intermediate is
 * subnormal or overflows, so "sig" covers the whole stated range. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static float markstein(float x, float c, float r) {
  const float ax = fabsf(x);
  if (!(ax >= 0x1p-100f && ax <= 0x1p120f)) {
    volatile float q = x / c; /* the kernels take the IEEE division here */
    return q;
  }
  volatile float q0 = x * r;
  float e = fmaf(-q0, c, x);
  return fmaf(e, r, q0);
}

static int same(float a, float b) { return f2u(a) == f2u(b) || (isnan(a) && isnan(b)); }

int main(int argc, char** argv) {
  if (argc >= 3 && strcmp(argv[1], "const") == 0) {
    const float c = strtof(argv[2], NULL);
    volatile float one = 1.0f;
    const float r = one / c;
    uint64_t bad = 0;
    for (uint64_t u = 0; u <= 0xffffffffull; ++u) {
      const float x = u2f((uint32_t)u);
      volatile float exact = x / c;
      if (!same(markstein(x, c, r), exact)) ++bad;
    }
    printf("%llu\n", (unsigned long long)bad);
    return 0;
  }
  if (argc >= 3 && strcmp(argv[1], "sig") == 0) {
    const float c = strtof(argv[2], NULL);
    volatile float one = 1.0f;
    const float r = one / c;
    const float ch = r;
    volatile float resid = fmaf(-c, ch, 1.0f); /* exact */
    const float cl = resid / c;
    static const int exps[] = {-98, -60, -20, 0, 20, 60, 119};
    uint64_t bad_m = 0, bad_bm = 0;
    for (unsigned e = 0; e < sizeof(exps) / sizeof(exps[0]); ++e) {
      for (uint32_t m = 0; m < (1u << 23); ++m) {
        for (int sgn = 0; sgn < 2; ++sgn) {
          const uint32_t u = ((uint32_t)sgn << 31) | ((uint32_t)(exps[e] + 127) << 23) | m;
          const float x = u2f(u);
          volatile float exact = x / c;
          if (!same(markstein(x, c, r), exact)) ++bad_m;
          volatile float lo = x * cl;
          const float bm = fmaf(x, ch, lo);
          if (!same(bm, exact)) ++bad_bm;
        }
      }
    }
    printf("%llu %llu\n", (unsigned long long)bad_m, (unsigned long long)bad_bm);
    return 0;
  }
  if (argc >= 4 && strcmp(argv[1], "random") == 0) {
    const uint64_t n = strtoull(argv[2], NULL, 10);
    uint64_t s = strtoull(argv[3], NULL, 10) * 2654435761ull + 1;
    uint64_t bad = 0;
    for (uint64_t i = 0; i < n; ++i) {
      s ^= s << 13; s ^= s >> 7; s ^= s << 17;
      /* divisor: random significand, exponent in [-30, 20] */
      const uint32_t cu = (uint32_t)(((s >> 8) & 0x7fffff) | ((uint32_t)(97 + (s >> 40) % 51) << 23));
      const float c = u2f(cu);
      s ^= s << 13; s ^= s >> 7; s ^= s << 17;
      const float x = ((float)(int32_t)(s >> 32) / 2147483648.0f) * 8.0f * c;
      volatile float one = 1.0f;
      const float r = one / c;
      volatile float exact = x / c;
      if (!same(markstein(x, c, r), exact)) ++bad;
    }
    printf("%llu\n", (unsigned long long)bad);
    return 0;
  }
  fprintf(stderr, "usage: div_check const <c> | sig <c> | random <n> <seed>\n");
  return 2;
}
