/* Checks the division used by the codec kernels: q1 = fma(x - q0*c, r, q0) with
 * q0 = x*r, r = RN(1/c) (Markstein's correction step) must equal the IEEE
 * quotient RN(x/c) whenever 2^-100 <= |x| <= 2^120 (outside that range, and for
 * NaN, the kernels fall back to the IEEE division).  Mode "const <c>" walks every float32 x; mode
 * "random <n> <seed>" draws n (x, c) pairs with c in the range of the
 * quantizer's scales and x in [-8c, 8c]. Prints the number of mismatches. */
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
  fprintf(stderr, "usage: div_check const <c> | random <n> <seed>\n");
  return 2;
}
