// prenorm.cu -- the Gemma MoE block's two inputs from the residual rows.
//
// engines/gemma.c routes on the residual row x (route_token, :455-460) and
// feeds the experts another norm of the same row (:608):
//   r  = (mean(x^2) + eps)^-0.5        rmsnorm, :313-317
//   xr = (x*r) * (router.scale * D^-0.5)   router input, :458-460
//   xe = (x*r) * pre_feedforward_layernorm_2   expert input, :608
// One warp per token writes xr (f32, the router's operand), and xe as f32
// (CUDA-core expert paths) and/or f16 (the tensor-core path's token operand).
//
// The sum of squares.  The reference adds (double)x[i]*x[i] in index order
// and rounds ms/D to float.  Each product is exact in double; the warp adds
// them in another order, whose result is within 2(D-1)u of the sequential
// one (all terms are >= 0, u = 2^-53).  The float rounding of ms/D can only
// differ when ms/D lies within that distance of a point halfway between two
// floats; for those rows (about 2 in 10^5 for D = 2816) one lane redoes the
// sum in index order.  So float(ms/D) is the reference's in every case.
//
// The factor.  The reference calls powf(y, -0.5f), which libm does not round
// correctly (glibc 2.39 x86-64 is 1 ulp off for 0.06% of floats).  Here r is
// 1/sqrt(y) in double, rounded once to float: the correctly rounded value
// (it equals the 64-bit long double result rounded to float on every
// positive float).  Routing indices are unaffected in practice; top-k weights
// move by a few ulps on the rows where the two differ.
#include "omc_rms.cuh"

namespace {

constexpr int PN_WARPS = 8;

__global__ void __launch_bounds__(PN_WARPS * 32)
    gemma_prenorm_kernel(const float *__restrict__ x, int T, int D, float eps, const float *__restrict__ s2,
                         const float *__restrict__ en, float *__restrict__ xr, float *__restrict__ xe,
                         __half *__restrict__ xh, float *__restrict__ rout, int *err) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * PN_WARPS + (threadIdx.x >> 5);
    if (t >= T) return;
    const float *xt = x + (size_t)t * D;
    const float4 *x4 = reinterpret_cast<const float4 *>(xt);
    const int n4 = D >> 2;
    const float r = omc_gemma_rms_factor(xt, D, eps);
    if (rout && lane == 0) rout[t] = r;
    const float4 *s24 = reinterpret_cast<const float4 *>(s2);
    const float4 *en4 = reinterpret_cast<const float4 *>(en);
    for (int i = lane; i < n4; i += 32) {
        const float4 v = __ldg(x4 + i);
        const float4 n = make_float4(__fmul_rn(v.x, r), __fmul_rn(v.y, r), __fmul_rn(v.z, r), __fmul_rn(v.w, r));
        if (xr) {
            const float4 c = __ldg(s24 + i);
            reinterpret_cast<float4 *>(xr + (size_t)t * D)[i] =
                make_float4(__fmul_rn(n.x, c.x), __fmul_rn(n.y, c.y), __fmul_rn(n.z, c.z), __fmul_rn(n.w, c.w));
        }
        float4 e = n;
        if (en) {
            const float4 w = __ldg(en4 + i);
            e = make_float4(__fmul_rn(n.x, w.x), __fmul_rn(n.y, w.y), __fmul_rn(n.z, w.z), __fmul_rn(n.w, w.w));
        }
        if (xe) reinterpret_cast<float4 *>(xe + (size_t)t * D)[i] = e;
        if (xh) {
            if (omc_f16_outside(e.x) || omc_f16_outside(e.y) || omc_f16_outside(e.z) || omc_f16_outside(e.w))
                omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_ROUTER, t);
            uint2 o;
            o.x = f32x2_to_f16x2_sat(e.x, e.y);
            o.y = f32x2_to_f16x2_sat(e.z, e.w);
            reinterpret_cast<uint2 *>(xh + (size_t)t * D)[i] = o;
        }
    }
}

}  // namespace

// xr (router input, f32), xe (expert input, f32) and xh (expert input, f16)
// are each nullable; r receives the norm factor per row (nullable).
extern "C" int omc_launch_gemma_prenorm(const omc_layer_dev *L, const float *x, int T, float *xr, float *xe,
                                        uint16_t *xh, float *r, int *err, cudaStream_t s) {
    if (T <= 0) return 0;
    if (L->family != OMC_FAMILY_GEMMA || (L->D & 3) || !L->g_s2) return OMC_EINVAL;
    gemma_prenorm_kernel<<<(T + PN_WARPS - 1) / PN_WARPS, PN_WARPS * 32, 0, s>>>(
        x, T, L->D, L->eps, L->g_s2, L->g_en, xr, xe, reinterpret_cast<__half *>(xh), r, err);
    omc_g_launches += 1;
    omc_prof_mark(s, "prenorm");
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
