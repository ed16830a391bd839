// omc_rms.cuh -- Gemma's rms factor (mean(x^2) + eps)^-0.5 of one row, as a
// warp-level device function (every lane gets the same value).
//
// engines/gemma.c:313-317: ms = the double sum of (double)x[i]*x[i] in index
// order, (float)(ms/n) + eps, powf(., -0.5f).  Each product is exact in
// double; the warp adds them in another order, within 2(D-1)u of the
// sequential sum (all terms are >= 0, u = 2^-53), so float(ms/D) can only
// differ when ms/D lies within that distance of a point halfway between two
// floats; for those rows (about 2 in 10^5 at D = 2816) one lane redoes the
// sum in index order.  The factor is 1/sqrt(y) in double rounded once to
// float: the correctly rounded value (libm's powf is 1 ulp off it on 0.06% of
// floats; the oracle has both).  x may be in global or shared memory, 16-byte
// aligned, D a multiple of 4.
#pragma once
#include "omc_common.cuh"

__device__ __forceinline__ double omc_sq(float v) { return __dmul_rn((double)v, (double)v); }

__device__ inline float omc_gemma_rms_factor(const float *xt, int D, float eps) {
    const int lane = threadIdx.x & 31;
    const float4 *x4 = reinterpret_cast<const float4 *>(xt);
    const int n4 = D >> 2;
    double s = 0.0;
    for (int i = lane; i < n4; i += 32) {
        const float4 v = x4[i];
        s = __dadd_rn(s, omc_sq(v.x));
        s = __dadd_rn(s, omc_sq(v.y));
        s = __dadd_rn(s, omc_sq(v.z));
        s = __dadd_rn(s, omc_sq(v.w));
    }
    // xor butterfly: every lane ends with the same bits (a + b == b + a)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    double q = __ddiv_rn(s, (double)D);
    float f = __double2float_rn(q);
    const uint32_t fb = __float_as_uint(f);
    bool sure = q >= 0.0 && fb < 0x7f7fffffu;   // finite, below FLT_MAX
    if (sure) {
        const double tol = (double)(D + 2) * 0x1p-51 * q;
        const double lo = fb == 0u ? -1.0 : 0.5 * ((double)__uint_as_float(fb - 1u) + (double)f);
        const double hi = 0.5 * ((double)f + (double)__uint_as_float(fb + 1u));
        sure = (q - lo > tol) && (hi - q > tol);
    }
    if (!sure) {   // warp-uniform: every lane holds the same q
        double sq_seq = 0.0;
        if (lane == 0)
            for (int i = 0; i < D; ++i) sq_seq = __dadd_rn(sq_seq, omc_sq(xt[i]));
        s = __shfl_sync(0xffffffffu, sq_seq, 0);
        q = __ddiv_rn(s, (double)D);
        f = __double2float_rn(q);
    }
    const float y = __fadd_rn(f, eps);
    return __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn((double)y)));
}
