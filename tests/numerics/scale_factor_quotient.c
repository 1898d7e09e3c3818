// Exhaustive check of the division behind the requantization scale factor on the fast
// path, sf0 = min(16, c / b) with c = 127 (b = qmax + r > 127/16) or c = -128
// (b = qmin + r < -8).
//
// Method (Markstein's division with a refined reciprocal: P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990):
//   y   ~ 1/b                      (the hardware approximation, documented within 1 ulp;
//                                   every y within K = 2 ulp of RN(1/b) is checked, and
//                                   y = 0 where RN(1/b) is subnormal)
//   e   = fma(-b, y, 1)
//   y1  = fma(e, y, y)
//   q0  = RN(c * y1)
//   rem = fma(-b, q0, c)           (exact)
//   q1  = fma(rem, y1, q0)
//
// What the kernel relies on, checked for c = 127 and c = 128 (c = -128 with b < 0: every
// step is odd in the signs of c and b together):
//   (1) 127/16 < b <= 1024 (c = 127) or 8 < b <= 1024 (c = 128), every f32 b:
//       (q1 > 0.98) == (RN(c/b) > 0.98), and when so floor(min(16, q1)) equals
//       floor(min(16, RN(c/b))) -- the integer scale factor and the fast / rare decision;
//   (2) b > 1024 (every 61st f32 up to 2^126, every f32 above): q1 <= 0.98, as RN(c/b) is.
// q1 itself is not always RN(c/b): for c = 128 and b = 2^k (1 - 2^-24) it is one ulp
// low (b = 2^4 - ulp ... 2^10 - ulp: 28 (b, y) cases of range (1)), which moves no floor
// and no 0.98 decision.
// Where the kernel needs the quotient itself (sf0 <= 0.98 on the rare-block path) it
// recomputes it with an IEEE division.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static uint32_t bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float from_bits(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }
#define K 2

static float quotient(float c, float b, float y) {
  const float e = fmaf(-b, y, 1.0f);
  const float y1 = fmaf(e, y, y);
  const float q0 = c * y1;
  const float rem = fmaf(-b, q0, c);
  return fmaf(rem, y1, q0);
}

// returns the number of violations of (1) / (2); counts inexact quotients in *inexact
static long check(float c, float b_lo, long* inexact) {
  const int64_t first = bits(b_lo) + 1, last = bits(3.4028235e38f), split = bits(1024.0f);
  const int64_t sub = bits(0x1p126f);
  long bad = 0, n = 0, ne = 0;
#pragma omp parallel for reduction(+ : bad, n, ne) schedule(dynamic, 1)
  for (int64_t chunk = first; chunk <= last; chunk += 1 << 16) {
    for (int64_t u = chunk; u < chunk + (1 << 16) && u <= last; ++u) {
      if (u > split && u < sub && (u % 61) != 0) continue;
      const float b = from_bits((uint32_t)u);
      const float y0 = 1.0f / b;
      const float want = c / b;
      for (int d = -K; d <= K + 1; ++d) {
        float y;
        if (d == K + 1) {
          if (u < sub) continue;
          y = 0.0f;   // a flushed subnormal reciprocal
        } else {
          if ((int64_t)bits(y0) + d < 0) continue;
          y = from_bits(bits(y0) + d);
        }
        const float q1 = quotient(c, b, y);
        ++n;
        int ok;
        if (u <= split) {
          const int big = q1 > 0.98f, want_big = want > 0.98f;
          ok = big == want_big && (!big || floorf(fminf(16.0f, q1)) == floorf(fminf(16.0f, want)));
          if (bits(q1) != bits(want)) {
#pragma omp critical
            if (ne < 4) printf("  inexact: c=%g b=%a y=%a q1=%a want %a\n", c, b, y, q1, want);
            ++ne;
          }
        } else {
          ok = q1 <= 0.98f;
        }
        if (!ok) {
#pragma omp critical
          if (bad < 5) printf("VIOLATION c=%g b=%a y=%a q1=%a want %a\n", c, b, y, q1, want);
          ++bad;
        }
      }
    }
  }
  printf("c=%g: checked %ld, violations %ld, inexact quotients %ld\n", c, n, bad, ne);
  *inexact += ne;
  return bad;
}

int main(void) {
  long inexact = 0;
  long bad = check(127.0f, 127.0f / 16.0f, &inexact);
  bad += check(128.0f, 8.0f, &inexact);
  return bad != 0;
}
