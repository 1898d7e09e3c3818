// Exhaustive check of the branch-free quotient of two f16-valued f32 numbers used for
// r = M / S in the requantization: with y any f32 within K ulp of 1/b (the reciprocal
// approximation is documented to be within 1 ulp; K = 2 is checked), e = fma(-b, y, 1)
// (exact: b has at most 11 significant bits), yl = RN(e * y) and
// r = RN(a*y + RN(a*yl)) (one fma), r equals RN(a / b) for every finite f16 a >= 0 and
// every finite nonzero f16 b > 0.  Both signs follow by symmetry of every step.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
static float h2f(uint16_t h) {
  uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023, f;
  if (e == 0) { if (m == 0) f = s << 31; else { float v = ldexpf((float)m, -24); if (s) v = -v; return v; } }
  else if (e == 31) f = (s << 31) | 0x7f800000 | (m << 13);
  else f = (s << 31) | ((e - 15 + 127) << 23) | (m << 13);
  float r; memcpy(&r, &f, 4); return r;
}
static uint32_t bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float from_bits(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }
#define K 2
int main(void) {
  static float av[31744];
  int na = 0;
  for (uint32_t h = 0; h < 0x7C00; ++h) av[na++] = h2f((uint16_t)h);   // +0 .. 65504
  long bad = 0, n = 0;
#pragma omp parallel for reduction(+ : bad, n) schedule(dynamic, 64)
  for (uint32_t hb = 1; hb < 0x7C00; ++hb) {
    const float b = h2f((uint16_t)hb);
    const float y0 = 1.0f / b;
    for (int d = -K; d <= K; ++d) {
      const float y = from_bits(bits(y0) + d);
      const float e = fmaf(-b, y, 1.0f);
      const float yl = e * y;
      for (int i = 0; i < na; ++i) {
        const float a = av[i];
        const float r = fmaf(a, y, a * yl);
        const float want = a / b;
        ++n;
        if (bits(r) != bits(want)) {
#pragma omp critical
          if (bad < 5) printf("a=%a b=%a y=%a got %a want %a\n", a, b, y, r, want);
          ++bad;
        }
      }
    }
  }
  printf("checked %ld, mismatches %ld\n", n, bad);
  return bad != 0;
}
