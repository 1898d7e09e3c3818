// Check of the invariant-divisor parameters (gq::fast_div_params) used by the head
// permutation: q = (t1 + ((n - t1) >> sh1)) >> sh2 with t1 = mulhi(m, n) equals n / d for
// n below 2^31 (dense below 2^24, strided above) and a range of divisors.
#include <stdio.h>

#include "gq_internal.h"

static uint32_t fdiv(uint32_t n, uint32_t mul, uint32_t shift) {
    const uint32_t t1 = static_cast<uint32_t>((static_cast<uint64_t>(mul) * n) >> 32);
    return (t1 + ((n - t1) >> (shift & 0xFF))) >> (shift >> 8);
}

int main() {
    long bad = 0, n_checked = 0;
    const uint32_t ds[] = {1, 2, 3, 5, 7, 10, 14, 16, 28, 32, 56, 64, 96, 100, 127, 128, 129, 255, 256, 1000, 4096,
                           65535, 65536, 1u << 20, 3000017, 2147483647u};
    for (uint32_t d : ds) {
        uint32_t m, s;
        gq::fast_div_params(d, m, s);
        for (uint64_t n = 0; n < (1ull << 31); n += (n < (1u << 24) ? 1 : 9973)) {
            ++n_checked;
            if (fdiv(static_cast<uint32_t>(n), m, s) != static_cast<uint32_t>(n / d) && bad++ < 5)
                printf("d=%u n=%llu\n", d, static_cast<unsigned long long>(n));
        }
    }
    printf("checked %ld, mismatches %ld\n", n_checked, bad);
    return bad != 0;
}
