/* expf_check.c -- TEST INFRASTRUCTURE: checks that the restated expf used on
 * the device (overhang_b200/csrc/omc_common.cuh, omc_expf_glibc) gives the
 * same bits as this host's glibc expf, the function the reference's softmax
 * calls (engines/olmoe.c:172, engines/qwen.c:163).
 *
 * The restatement follows the published ARM optimized-routines expf
 * (Szabolcs Nagy, 2017; in glibc since 2.28): x*32/ln2 = k + r, 2^(k/32)
 * from a table, 2^(r/32) by a cubic, all in double, with the FMAs the x86-64
 * FMA build of glibc forms.  Usage: expf_check [stride] -- compares every
 * stride-th float bit pattern (stride 1 = all 2^32), prints the mismatch
 * count and exits 0 only when it is zero. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static const uint64_t tab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

static double asd(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static uint64_t asu(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

static float restated_expf(float x) {
    uint32_t ix; memcpy(&ix, &x, 4);
    const uint32_t abstop = (ix >> 20) & 0x7ff;
    if (abstop >= 0x42b) {
        if (ix == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8) return x + x;
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double InvLn2N = 0x1.71547652b82fep+0 * 32.0, Shift = 0x1.8p+52;
    const double C0 = 0x1.c6af84b912394p-5 / 32768.0, C1 = 0x1.ebfce50fac4f3p-3 / 1024.0,
                 C2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = x;
    double kd = fma(InvLn2N, xd, Shift);
    const uint64_t ki = asu(kd);
    kd -= Shift;
    const double r = fma(InvLn2N, xd, -kd);
    const double s = asd(tab[ki & 31] + (ki << 47));
    const double z = fma(C0, r, C1), r2 = r * r;
    double y = fma(C2, r, 1.0);
    y = fma(z, r2, y);
    return (float)(y * s);
}

int main(int argc, char **argv) {
    const long long stride = argc > 1 ? atoll(argv[1]) : 1;
    long long bad = 0, n = 0;
    #pragma omp parallel for reduction(+:bad, n) schedule(static, 1 << 16)
    for (long long b = 0; b < (1LL << 32); b += stride) {
        const uint32_t bits = (uint32_t)b;
        float x; memcpy(&x, &bits, 4);
        const float r = expf(x), m = restated_expf(x);
        n++;
        if (memcmp(&r, &m, 4) && !(isnan(r) && isnan(m))) bad++;
    }
    printf("expf_check: %lld inputs, %lld mismatches\n", n, bad);
    return bad ? 1 : 0;
}
