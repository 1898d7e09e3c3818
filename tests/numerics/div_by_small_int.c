// Exhaustive check of the division used for block scales: for every finite f32 value S
// that is a widened f16 and every integer k in 1..16, with y = RN(1/k), q0 = RN(S*y) and
// r = fma(-k, q0, S) (exact), q = (r == 0 ? q0 : RN(q0 + r*y)) equals RN(S/k).
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
int main(void) {
  long bad = 0, n = 0;
  for (int k = 1; k <= 16; ++k) {
    volatile float kf = (float)k;
    volatile float y = 1.0f / kf;
    for (uint32_t h = 0; h < 65536; ++h) {
      float S = h2f((uint16_t)h);
      if (!isfinite(S)) continue;
      volatile float q0 = S * y;
      float r = fmaf(-kf, q0, S);
      float q1 = (r == 0.0f) ? q0 : fmaf(r, y, q0);
      volatile float want = S / kf;
      uint32_t a, b; memcpy(&a, &q1, 4); memcpy(&b, (const void*)&want, 4);
      ++n;
      if (a != b) { if (bad < 5) printf("k=%d S=%a got %a want %a\n", k, S, q1, want); ++bad; }
    }
  }
  printf("checked %ld, mismatches %ld\n", n, bad);
  return bad != 0;
}
