/* rsqrt_check.c -- TEST INFRASTRUCTURE: the norm factor of Gemma's router
 * (engines/gemma.c:313-317, powf((float)(ms/n) + eps, -0.5f)).
 *
 * The device (overhang_b200/csrc/prenorm.cu) and the oracle's RSQRT_CR mode
 * compute r = (float)(1.0 / sqrt((double)y)): one IEEE double sqrt, one
 * IEEE double divide, one rounding to float.  This program checks, on every
 * stride-th positive finite float y, that this r equals the 64-bit-mantissa
 * long double 1/sqrtl(y) rounded to float (the correctly rounded value up to
 * that precision), and counts how often this host's libm powf(y, -0.5f)
 * differs from it (libm is not correctly rounded).
 *
 * Usage: rsqrt_check [stride]; prints both counts and exits 0 only when the
 * double formula never differs from the long double one. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int main(int argc, char **argv) {
    const uint32_t stride = argc > 1 ? (uint32_t)strtoul(argv[1], NULL, 10) : 1u;
    unsigned long long n = 0, bad = 0, libm = 0;
    #pragma omp parallel for reduction(+:n,bad,libm) schedule(static)
    for (int64_t b = 1; b < 0x7f800000LL; b += stride) {
        const uint32_t u = (uint32_t)b;
        float y;
        memcpy(&y, &u, 4);
        const float d = (float)(1.0 / sqrt((double)y));
        const float l = (float)(1.0L / sqrtl((long double)y));
        const float p = powf(y, -0.5f);
        if (memcmp(&d, &l, 4)) ++bad;
        if (memcmp(&p, &d, 4)) ++libm;
        ++n;
    }
    printf("rsqrt_check: %llu floats, %llu double/long-double mismatches, %llu libm powf differences\n", n, bad,
           libm);
    return bad == 0 ? 0 : 1;
}
