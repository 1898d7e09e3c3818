// Exhaustive check of the packed integer requantization in process_k45 (gq_kernels.cu) for
// blocks with an integer scale factor and no clipping, over every scale factor sfi in 1..16,
// every offset rm and every pair of codes that share a 32-bit operation.  The kernel keeps
// the codes of a word in 16-bit lanes at their place in the word (no shift down), computes
// q * sfi + rm + 0x400 per lane, the odd bytes with a multiply-high that undoes their shift,
// and gathers the low bytes with a byte permute:
//   Q4_K low nibbles:  codes_word(EL * sfi + K, mad_hi(OL, sfi << 24, K))
//   Q4_K high nibbles: codes_word((EH * sfi + (K << 4)) >> 4, mad_hi(OH, sfi << 20, K))
//   Q5_K (codes as bytes, one mask per layout): codes_word(E * sfi + K, mad_hi(O, sfi << 24, K))
// with K = (rm + 0x400) * 0x00010001.  Each result byte must equal int8(q * sfi + rm), which
// is requantize_symmetric's code for such a block (ggml_quant.py:866-875).
//
// Bytes 0 and 2 of a word go through one multiply-add (E) and bytes 1 and 3 through one
// multiply-high (O); the two results are separate registers until the permute, which moves
// bytes independently.  So every pair of codes that shares an operation is checked in full
// (all pairs the block's code range allows), with the other pair at the range's ends, and
// with the other nibble of each byte (Q4_K) at 0, 15 and a mixed pattern, which the masks
// must remove.
#include <stdint.h>
#include <stdio.h>

static uint32_t byte_perm(uint32_t x, uint32_t y, uint32_t s) {
  // PTX prmt (default mode): result byte i = byte (selector nibble i & 7) of {y:x}
  const uint64_t v = ((uint64_t)y << 32) | x;
  uint32_t r = 0;
  for (int i = 0; i < 4; ++i) r |= (uint32_t)((v >> (8 * ((s >> (4 * i)) & 7))) & 0xFF) << (8 * i);
  return r;
}
static uint32_t mad_hi(uint32_t a, uint32_t b, uint32_t c) { return (uint32_t)(((uint64_t)a * b) >> 32) + c; }
static uint32_t codes_word(uint32_t e, uint32_t o) { return byte_perm(e, o, 0x6240); }

static long n = 0, bad = 0;

static void expect(const char* what, uint32_t got, const int q[4], int sfi, int rm) {
  for (int b = 0; b < 4; ++b) {
    ++n;
    if ((uint8_t)(got >> (8 * b)) != (uint8_t)(int8_t)(q[b] * sfi + rm)) {
      if (bad < 5) printf("%s sfi=%d rm=%d q=%d,%d,%d,%d byte %d got %02x\n", what, sfi, rm, q[0], q[1], q[2], q[3],
                          b, (unsigned)(uint8_t)(got >> (8 * b)));
      ++bad;
    }
  }
}

// one word of a block with code range [lo, hi]: Q5_K (codes 0..31, one per byte) or the
// low / high nibbles of a Q4_K word, the other nibbles set to `other`
static void check(int qmax, int sfi, int rm, const int q[4], uint32_t other) {
  const uint32_t K = (uint32_t)(rm + 0x400) * 0x00010001u;
  if (qmax == 31) {
    const uint32_t w = (uint32_t)q[0] | (uint32_t)q[1] << 8 | (uint32_t)q[2] << 16 | (uint32_t)q[3] << 24;
    expect("Q5_K", codes_word((w & 0x00FF00FFu) * sfi + K, mad_hi(w & 0xFF00FF00u, (uint32_t)sfi << 24, K)), q, sfi, rm);
    return;
  }
  uint32_t wl = 0, wh = 0;
  for (int b = 0; b < 4; ++b) {
    const uint32_t o = (other >> (4 * b)) & 15;
    wl |= ((uint32_t)q[b] | o << 4) << (8 * b);   // codes in the low nibbles
    wh |= (o | (uint32_t)q[b] << 4) << (8 * b);   // codes in the high nibbles
  }
  expect("Q4_K low", codes_word((wl & 0x000F000Fu) * sfi + K, mad_hi(wl & 0x0F000F00u, (uint32_t)sfi << 24, K)), q,
         sfi, rm);
  expect("Q4_K high",
         codes_word(((wh & 0x00F000F0u) * sfi + (K << 4)) >> 4, mad_hi(wh & 0xF000F000u, (uint32_t)sfi << 20, K)), q,
         sfi, rm);
}

// Q5_K's 5-bit codes as bytes (process_k45): with t = qh_word >> 2g, the low-nibble block's
// codes are (t & 0x01010101) * 16 + (qs_word & 0x0F0F0F0F) and the high-nibble block's
// (t & 0x02020202) * 8 + ((qs_word >> 4) & 0x0F0F0F0F); byte j must be nibble | bit << 4 with
// bit 2g (low) or 2g + 1 (high) of qh byte j (ggml_quant.py:311-349).  Bytes cannot carry
// into each other (each is at most 31), and every byte pair (qs byte, qh byte) is checked in
// every byte position against the other positions' bytes at 0x00 and 0xFF.
static void check_q5_codes(void) {
  for (int g = 0; g < 4; ++g)
    for (int pos = 0; pos < 4; ++pos)
      for (uint32_t fill = 0; fill <= 0xFF; fill += 0xFF)
        for (uint32_t qs = 0; qs < 256; ++qs)
          for (uint32_t qh = 0; qh < 256; ++qh) {
            uint32_t w = 0, h = 0;
            for (int b = 0; b < 4; ++b) {
              w |= (b == pos ? qs : fill) << (8 * b);
              h |= (b == pos ? qh : (fill ^ 0xA5)) << (8 * b);
            }
            const uint32_t t = h >> (2 * g);
            const uint32_t lo = (t & 0x01010101u) * 16u + (w & 0x0F0F0F0Fu);
            const uint32_t hi = (t & 0x02020202u) * 8u + ((w >> 4) & 0x0F0F0F0Fu);
            for (int b = 0; b < 4; ++b) {
              const uint32_t wb = (w >> (8 * b)) & 0xFF, hb = (h >> (8 * b)) & 0xFF;
              const uint32_t want_lo = (wb & 15) | ((hb >> (2 * g)) & 1) << 4;
              const uint32_t want_hi = (wb >> 4) | ((hb >> (2 * g + 1)) & 1) << 4;
              n += 2;
              if (((lo >> (8 * b)) & 0xFF) != want_lo || ((hi >> (8 * b)) & 0xFF) != want_hi) {
                if (bad < 5) printf("Q5_K codes g=%d pos=%d qs=%02x qh=%02x byte %d\n", g, pos, qs, qh, b);
                ++bad;
              }
            }
          }
}

int main(void) {
  check_q5_codes();
  const uint32_t others[3] = {0x0000u, 0xFFFFu, 0x5A3Cu};
  for (int qmax = 15; qmax <= 31; qmax += 16) {
    for (int sfi = 1; sfi <= 16; ++sfi) {
      for (int rm = -128 - qmax * 16; rm <= 127; ++rm) {
        int lo = 0, hi = qmax;   // the codes a good block with these parameters can hold
        while (lo <= qmax && lo * sfi + rm < -128) ++lo;
        while (hi >= 0 && hi * sfi + rm > 127) --hi;
        if (lo > hi) continue;
        for (int a = lo; a <= hi; ++a) {
          for (int b = lo; b <= hi; ++b) {
            for (int k = 0; k < (qmax == 15 ? 3 : 1); ++k) {
              const int even[4] = {a, lo, b, hi}, odd[4] = {hi, a, lo, b};   // pair (0,2), pair (1,3)
              check(qmax, sfi, rm, even, others[k]);
              check(qmax, sfi, rm, odd, others[k]);
            }
          }
        }
      }
    }
  }
  printf("checked %ld codes, mismatches %ld\n", n, bad);
  return bad != 0;
}
